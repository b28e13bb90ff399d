// w4.cu -- INT4 nibble-packed weight GEMM with f32 activations.
//
// Reference semantics: dequantize_i4_symmetric_per_channel
// (crates/tpt-infer-quantize/src/dequant.rs:56-71) followed by the f32 matmul
// (crates/tpt-infer-ops/src/avx512.rs:55-78) and the runtime's bias add:
//   y[m,n] = sum_k x[m,k] * (q[n,k] * s[n]) + bias[n], then act.
// The device computes s[n] * sum_k x[m,k]*q[n,k] (the per-channel scale
// factored out of the sum, q exact as a small integer), which differs from the
// reference only by f32 rounding; parity is checked at max-abs 1e-3 x output
// scale.
//
// Weight layout in HBM: n rows of k/2 bytes, low nibble first along k -- the
// bytes quantize_i4_symmetric_per_channel(W^T, rows = n) emits
// (quant.rs:192-204), uploaded once, never repacked.
//
// 3 <= M <= 8 with K % 256 == 0, K <= 4096 goes to the small-batch kernel of
// w4_gemv.cu; other M >= 3 to the tensor-core kernel (w4_tc.cu) when
// K % 128 == 0 and x is 16-byte aligned. M <= 2 uses the TMA-ring GEMV with integer digit planes
// (w4_gemv.cu) for K % 256 == 0, K <= 8192, else k_w4_gemv: one warp streams 8
// weight rows with 128-bit loads, reusing each activation chunk across the 8
// rows. Other shapes use the SIMT tile kernel.
#include <new>

#include "common.cuh"

namespace tpt {

int launch_w4_simt(tpt_cuda_ctx *ctx, const float *x, const uint8_t *packed, const float *scales, const float *bias,
                   int act, float *y, size_t m, size_t n, size_t k);
int launch_w4_tc(tpt_cuda_ctx *ctx, const float *x, size_t m, const tpt_cuda_weights *w, const float *bias, int act,
                 float *y, bool *handled);
int launch_w4_gemv_tma(tpt_cuda_ctx *ctx, const float *x, size_t m, const tpt_cuda_weights *w, const float *bias,
                       int act, float *y, bool *handled);
int launch_w4_small(tpt_cuda_ctx *ctx, const float *x, size_t m, const tpt_cuda_weights *w, const float *bias,
                    int act, float *y, bool *handled);

namespace {

constexpr int W4_ROWS = 8;  // weight rows per warp

// signed nibble j (0..7) of a 32-bit word, low nibble first
__device__ __forceinline__ float nib(unsigned w, int j) { return (float)((int)(w << (28 - 4 * j)) >> 28); }

// Each lane covers 32 consecutive k (one 16-byte chunk of a weight row).
template <int MM>
__global__ void __launch_bounds__(256) k_w4_gemv(const float *__restrict__ X, const uint8_t *__restrict__ Wp,
                                                 const float *__restrict__ scales, const float *__restrict__ bias,
                                                 int M, int N, int K, int act, float *__restrict__ Y) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int chunks = K >> 5;          // 32 k per 16-byte chunk
    const size_t row_bytes = (size_t)K >> 1;
    for (int n0 = warp * W4_ROWS; n0 < N; n0 += nwarps * W4_ROWS) {
        float acc[MM][W4_ROWS];
#pragma unroll
        for (int i = 0; i < MM; i++)
#pragma unroll
            for (int r = 0; r < W4_ROWS; r++) acc[i][r] = 0.0f;
        for (int c = lane; c < chunks; c += 32) {
            uint4 w[W4_ROWS];
#pragma unroll
            for (int r = 0; r < W4_ROWS; r++) {
                const int n = n0 + r < N ? n0 + r : N - 1;
                w[r] = __ldcs(reinterpret_cast<const uint4 *>(Wp + (size_t)n * row_bytes) + c);
            }
#pragma unroll
            for (int i = 0; i < MM; i++) {
                if (i >= M) break;
                const float4 *xr = reinterpret_cast<const float4 *>(X + (size_t)i * K + (size_t)c * 32);
#pragma unroll
                for (int q = 0; q < 4; q++) {  // 8 k per 32-bit word
                    float4 x0 = __ldg(xr + 2 * q), x1 = __ldg(xr + 2 * q + 1);
#pragma unroll
                    for (int r = 0; r < W4_ROWS; r++) {
                        unsigned word = q == 0 ? w[r].x : q == 1 ? w[r].y : q == 2 ? w[r].z : w[r].w;
                        float a = acc[i][r];
                        a = fmaf(x0.x, nib(word, 0), a);
                        a = fmaf(x0.y, nib(word, 1), a);
                        a = fmaf(x0.z, nib(word, 2), a);
                        a = fmaf(x0.w, nib(word, 3), a);
                        a = fmaf(x1.x, nib(word, 4), a);
                        a = fmaf(x1.y, nib(word, 5), a);
                        a = fmaf(x1.z, nib(word, 6), a);
                        a = fmaf(x1.w, nib(word, 7), a);
                        acc[i][r] = a;
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < MM; i++)
#pragma unroll
            for (int r = 0; r < W4_ROWS; r++) acc[i][r] = warp_sum(acc[i][r]);
        if (lane < W4_ROWS && n0 + lane < N) {
            const int n = n0 + lane;
            const float s = __ldg(scales + n), b = bias ? __ldg(bias + n) : 0.0f;
#pragma unroll
            for (int i = 0; i < MM; i++) {
                if (i >= M) break;
                float v = 0.0f;
#pragma unroll
                for (int r = 0; r < W4_ROWS; r++)
                    if (r == lane) v = acc[i][r];
                float y = v * s;
                if (bias) y += b;
                Y[(size_t)i * N + n] = apply_act(y, act);
            }
        }
    }
}

}  // namespace

int launch_w4(tpt_cuda_ctx *ctx, const float *x, size_t m, const tpt_cuda_weights *w, const float *bias, int act,
              float *y) {
    const size_t n = w->n, k = w->k;
    if (m == 0 || n == 0) return TPT_OK;
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return TPT_UNSUPPORTED;
    const uint8_t *p = (const uint8_t *)w->data;
    if (m > 2 && m <= 8) {
        bool handled = false;
        int st = launch_w4_small(ctx, x, m, w, bias, act, y, &handled);
        if (st || handled) return st;
    }
    if (m > 2) {
        bool handled = false;
        int st = launch_w4_tc(ctx, x, m, w, bias, act, y, &handled);
        if (st || handled) return st;
    }
    if (m <= 2) {
        bool handled = false;
        int st = launch_w4_gemv_tma(ctx, x, m, w, bias, act, y, &handled);
        if (st || handled) return st;
    }
    if (m <= 2 && ((uintptr_t)x & 15) == 0) {
        size_t warps = (n + W4_ROWS - 1) / W4_ROWS;
        unsigned g = grid_1d(warps * 32, 256, (unsigned)ctx->sm_count * 8);
        if (m == 1)
            k_w4_gemv<1><<<g, 256, 0, ctx->stream>>>(x, p, w->scales, bias, (int)m, (int)n, (int)k, act, y);
        else
            k_w4_gemv<2><<<g, 256, 0, ctx->stream>>>(x, p, w->scales, bias, (int)m, (int)n, (int)k, act, y);
        return after_launch(ctx, "w4_gemv");
    }
    return launch_w4_simt(ctx, x, p, w->scales, bias, act, y, m, n, k);
}

}  // namespace tpt

using namespace tpt;

#define CHECK_CTX(c)                  \
    do {                              \
        if (!(c)) return TPT_INVALID; \
        cudaSetDevice((c)->device);   \
    } while (0)
#define TRY(x)               \
    do {                     \
        int _st = (x);       \
        if (_st) return _st; \
    } while (0)

extern "C" {

int tpt_cuda_weights_upload_i4(tpt_cuda_ctx *ctx, const uint8_t *packed, size_t packed_len, const float *scales,
                               size_t n, size_t k, tpt_cuda_weights **out) {
    CHECK_CTX(ctx);
    if (!out || !packed || !scales || n == 0 || k == 0 || k % 32 != 0) return TPT_INVALID;
    *out = nullptr;
    size_t bytes;
    if (!checked_mul(n, k / 2, &bytes)) return TPT_INVALID;
    if (packed_len != bytes) return set_size_mismatch(ctx, bytes, packed_len);
    tpt_cuda_weights *w = new (std::nothrow) tpt_cuda_weights();
    if (!w) return TPT_OUT_OF_MEMORY;
    w->ctx = ctx;
    w->device = ctx->device;
    w->kind = 4;
    w->n = n;
    w->k = k;
    w->bytes = bytes;
    cudaError_t e = cudaMalloc(&w->data, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&w->scales, n * sizeof(float));
    if (e == cudaSuccess) e = cudaMemcpy(w->data, packed, bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(w->scales, scales, n * sizeof(float), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaGetLastError();
        if (w->data) cudaFree(w->data);
        if (w->scales) cudaFree(w->scales);
        delete w;
        return cuda_fail(ctx, e, "i4 weights upload");
    }
    *out = w;
    return TPT_OK;
}

int tpt_cuda_w4_gemm(tpt_cuda_ctx *ctx, const float *x, size_t m, size_t k, const tpt_cuda_weights *w,
                     const float *bias, int act, float *out) {
    CHECK_CTX(ctx);
    if (!w || w->kind != 4 || act < 0 || act > 2) return TPT_INVALID;
    if (k != w->k) return TPT_SHAPE_MISMATCH;
    size_t xn, on;
    if (!checked_mul(m, k, &xn) || !checked_mul(m, w->n, &on)) return TPT_INVALID;
    if (on == 0) return TPT_OK;
    Staging st(ctx);
    st.reserve(xn * 4);
    st.reserve(on * 4);
    st.reserve(bias ? w->n * 4 : 0);
    TRY(st.commit());
    float *dx = st.take<float>(xn), *dy = st.take<float>(on);
    float *db = bias ? st.take<float>(w->n) : nullptr;
    TRY(h2d(ctx, dx, x, xn * 4));
    if (bias) TRY(h2d(ctx, db, bias, w->n * 4));
    TRY(launch_w4(ctx, dx, m, w, db, act, dy));
    TRY(d2h(ctx, out, dy, on * 4));
    return sync_and_check(ctx);
}

int tpt_cuda_w4_gemm_dev(tpt_cuda_ctx *ctx, const float *x, size_t m, const tpt_cuda_weights *w, const float *bias,
                         int act, float *out) {
    CHECK_CTX(ctx);
    if (!w || w->kind != 4 || act < 0 || act > 2) return TPT_INVALID;
    return launch_w4(ctx, x, m, w, bias, act, out);
}

}  // extern "C"
