// eltwise.cu -- element-wise and row-normalisation kernels: Add, Relu,
// Sigmoid, Gelu (crates/tpt-infer-ops/src/naive.rs:86-146) and Softmax
// (naive.rs:104-125). HBM-bound: 128-bit loads/stores, grid-stride loops
// sized to the SM count, warp-shuffle reductions.
#include "common.cuh"

namespace tpt {
namespace {

__device__ __forceinline__ float unary_op(int op, float x) {
    if (op == 1) return x > 0.0f ? x : 0.0f;                       // naive.rs:95-101
    if (op == 2) return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));  // naive.rs:128-134
    return gelu_det(x);                                              // naive.rs:137-146 (det_math.cuh)
}

__global__ void k_add_vec(const float4 *__restrict__ a, const float4 *__restrict__ b,
                          float4 *__restrict__ o, size_t n4) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
         i += (size_t)gridDim.x * blockDim.x) {
        float4 x = __ldg(a + i), y = __ldg(b + i);
        o[i] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
    }
}

__global__ void k_add(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ o,
                      size_t n) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        o[i] = a[i] + b[i];
}

template <int OP>
__global__ void k_unary_vec(const float4 *__restrict__ a, float4 *__restrict__ o, size_t n4) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4;
         i += (size_t)gridDim.x * blockDim.x) {
        float4 x = __ldg(a + i);
        o[i] = make_float4(unary_op(OP, x.x), unary_op(OP, x.y), unary_op(OP, x.z), unary_op(OP, x.w));
    }
}

template <int OP>
__global__ void k_unary(const float *__restrict__ a, float *__restrict__ o, size_t n) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        o[i] = unary_op(OP, a[i]);
}

// One warp per row: running max (NaN ignored, as `v > max` in the reference),
// exp(v - max), warp-tree sum, then an IEEE divide by the sum.
__global__ void k_softmax_warp(const float *__restrict__ a, float *__restrict__ o, size_t rows,
                               size_t L) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    size_t row = (blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5;
    const size_t nwarps = ((size_t)gridDim.x * blockDim.x) >> 5;
    for (; row < rows; row += nwarps) {
        const float *src = a + row * L;
        float *dst = o + row * L;
        float mx = -INFINITY;
        for (size_t j = lane; j < L; j += 32) mx = fmaxf(mx, __ldg(src + j));
        mx = warp_max(mx);
        float s = 0.0f;
        for (size_t j = lane; j < L; j += 32) {
            float e = expf(src[j] - mx);
            dst[j] = e;
            s += e;
        }
        s = warp_sum(s);
        for (size_t j = lane; j < L; j += 32) dst[j] = __fdiv_rn(dst[j], s);
    }
}

// One block per row for long rows.
__global__ void k_softmax_block(const float *__restrict__ a, float *__restrict__ o, size_t rows,
                                size_t L) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[32];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, nw = blockDim.x >> 5;
    for (size_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const float *src = a + row * L;
        float *dst = o + row * L;
        float mx = -INFINITY;
        for (size_t j = tid; j < L; j += blockDim.x) mx = fmaxf(mx, src[j]);
        mx = warp_max(mx);
        if (lane == 0) red[wid] = mx;
        __syncthreads();
        mx = lane < nw ? red[lane] : -INFINITY;
        mx = warp_max(mx);
        __syncthreads();
        float s = 0.0f;
        for (size_t j = tid; j < L; j += blockDim.x) {
            float e = expf(src[j] - mx);
            dst[j] = e;
            s += e;
        }
        s = warp_sum(s);
        if (lane == 0) red[wid] = s;
        __syncthreads();
        s = lane < nw ? red[lane] : 0.0f;
        s = warp_sum(s);
        __syncthreads();
        for (size_t j = tid; j < L; j += blockDim.x) dst[j] = __fdiv_rn(dst[j], s);
    }
}

bool aligned16(const void *p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

int launch_add(tpt_cuda_ctx *ctx, const float *a, const float *b, float *out, size_t n) {
    const unsigned bs = 256;
    unsigned cap = (unsigned)ctx->sm_count * 8;
    if (n % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(out)) {
        launch_pdl(k_add_vec, grid_1d(n / 4, bs, cap), bs, 0, ctx->stream, (const float4 *)a, (const float4 *)b,
                                                                    (float4 *)out, n / 4);
    } else {
        launch_pdl(k_add, grid_1d(n, bs, cap), bs, 0, ctx->stream, a, b, out, n);
    }
    return after_launch(ctx, "add");
}

int launch_unary(tpt_cuda_ctx *ctx, int op, const float *a, float *out, size_t n) {
    const unsigned bs = 256;
    unsigned cap = (unsigned)ctx->sm_count * 8;
    bool vec = n % 4 == 0 && aligned16(a) && aligned16(out);
    unsigned g = grid_1d(vec ? n / 4 : n, bs, cap);
#define TPT_UNARY(OPN)                                                                                 \
    if (vec)                                                                                           \
        launch_pdl(k_unary_vec<OPN>, g, bs, 0, ctx->stream, (const float4 *)a, (float4 *)out, n / 4);          \
    else                                                                                               \
        launch_pdl(k_unary<OPN>, g, bs, 0, ctx->stream, a, out, n);
    if (op == 1) {
        TPT_UNARY(1)
    } else if (op == 2) {
        TPT_UNARY(2)
    } else {
        TPT_UNARY(3)
    }
#undef TPT_UNARY
    return after_launch(ctx, "unary");
}

int launch_softmax(tpt_cuda_ctx *ctx, const float *a, float *out, size_t rows, size_t row_len) {
    if (row_len <= 2048) {
        const unsigned bs = 256;
        unsigned g = grid_1d(rows * 32, bs, (unsigned)ctx->sm_count * 16);
        launch_pdl(k_softmax_warp, g, bs, 0, ctx->stream, a, out, rows, row_len);
    } else {
        unsigned g = (unsigned)(rows < (size_t)ctx->sm_count * 8 ? rows : (size_t)ctx->sm_count * 8);
        launch_pdl(k_softmax_block, g, 512, 0, ctx->stream, a, out, rows, row_len);
    }
    return after_launch(ctx, "softmax");
}

}  // namespace tpt
