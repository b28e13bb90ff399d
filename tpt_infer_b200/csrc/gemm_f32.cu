// gemm_f32.cu -- the f32 contractions of the Backend trait: MatMul
// (crates/tpt-infer-ops/src/naive.rs:13-33, avx512.rs:55-78) and Conv2d as an
// implicit GEMM (naive.rs:36-83), plus the general-M W4 path.
//
// Numerics (MatMul, Conv2d): each output is accumulated by one thread in
// increasing k order, acc = acc + a*b with a round-to-nearest multiply and a
// separate round-to-nearest add (__fmul_rn / __fadd_rn, never an FMA). That is
// exactly the reference's arithmetic (the Rust code never contracts to FMA and
// the AVX backends use _mm512_mul_ps then _mm512_add_ps), so results are
// bit-identical to the reference for finite inputs. For conv the implicit
// GEMM's k index is (ci, ky, kx) in the reference's loop order; padded taps
// contribute a +-0 product, which leaves the running sum unchanged (the
// reference skips them; the two differ only for non-finite weights).
//
// Tiling: 128x128 output tile per 256-thread CTA, 8x8 outputs per thread,
// k-slices of 8 staged through double-buffered shared memory.
#include "common.cuh"

namespace tpt {
namespace {

constexpr int BM = 128, BN = 128, BK = 8, NT = 256;

struct ConvGeom {
    int C, H, W, KH, KW, OH, OW, sh, sw, ph, pw, OC;
};

// W4 epilogue parameters (MODE 2).
struct W4Epi {
    const float *scales;
    const float *bias;
    int act;
};

// MODE 0: A [m,k] row-major, B [k,n] row-major, C [m,n].
// MODE 1: conv; A(m, kk) gathered from NCHW input, B(kk, oc) = w[oc*K + kk],
//         C(m, oc) scattered to NCHW output.
// MODE 2: W4; A = x [m,k] f32, B(kk, n) = signed nibble kk of weight row n
//         (rows of K/2 bytes, low nibble first), y = acc*scale[n] + bias[n], act.
//         FFMA accumulation (the W4 path is tolerance-checked, not bit-exact).
template <int MODE>
__global__ void __launch_bounds__(NT) k_gemm_f32(const float *__restrict__ A, const float *__restrict__ B,
                                                 float *__restrict__ Cout, int M, int N, int K,
                                                 ConvGeom g, W4Epi epi) {
    pdl_wait();
    pdl_trigger();
    __shared__ __align__(16) float As[2][BK][BM];
    __shared__ __align__(16) float Bs[2][BK][BN];
    const int tid = threadIdx.x;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int tx = tid & 15, ty = tid >> 4;

    // loader mapping: A tile BMxBK = 1024 values, 4 per thread (rows a_r + 32*i, k = tid%8)
    const int a_k = tid & 7, a_r = tid >> 3;
    // B tile BKxBN: 4 per thread, row b_k, cols b_c + 32*i
    const int b_k = tid >> 5, b_c = tid & 31;

    float ra[4], rb[4];
    auto load_tile = [&](int k0) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int m = m0 + a_r + 32 * i, kk = k0 + a_k;
            float v = 0.0f;
            if (m < M && kk < K) {
                if (MODE != 1) {
                    v = A[(size_t)m * K + kk];
                } else {
                    int hw = g.OH * g.OW;
                    int n = m / hw, p = m - n * hw;
                    int oy = p / g.OW, ox = p - oy * g.OW;
                    int khw = g.KH * g.KW;
                    int ci = kk / khw, r = kk - ci * khw;
                    int ky = r / g.KW, kx = r - ky * g.KW;
                    int iy = oy * g.sh + ky - g.ph, ix = ox * g.sw + kx - g.pw;
                    if (iy >= 0 && iy < g.H && ix >= 0 && ix < g.W)
                        v = A[(((size_t)n * g.C + ci) * g.H + iy) * g.W + ix];
                }
            }
            ra[i] = v;
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int kk = k0 + b_k, n = n0 + b_c + 32 * i;
            float v = 0.0f;
            if (kk < K && n < N) {
                if (MODE == 0) {
                    v = B[(size_t)kk * N + n];
                } else if (MODE == 1) {
                    v = B[(size_t)n * K + kk];
                } else {
                    unsigned byte = reinterpret_cast<const uint8_t *>(B)[(size_t)n * (K >> 1) + (kk >> 1)];
                    unsigned nib = (kk & 1) ? (byte >> 4) : (byte & 15u);
                    v = (float)((int)(nib << 28) >> 28);
                }
            }
            rb[i] = v;
        }
    };
    auto store_tile = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 4; i++) As[buf][a_k][a_r + 32 * i] = ra[i];
#pragma unroll
        for (int i = 0; i < 4; i++) Bs[buf][b_k][b_c + 32 * i] = rb[i];
    };

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0.0f;

    const int ktiles = (K + BK - 1) / BK;
    load_tile(0);
    store_tile(0);
    __syncthreads();
    for (int t = 0; t < ktiles; t++) {
        const int buf = t & 1;
        if (t + 1 < ktiles) load_tile((t + 1) * BK);
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float av[8], bv[8];
            // rows ty*4 + {0..3} and 64 + ty*4 + {0..3}; cols tx*4 + {0..3} and 64 + tx*4 + {0..3}
            float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][kk][ty * 4]);
            float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][kk][64 + ty * 4]);
            float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][tx * 4]);
            float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][64 + tx * 4]);
            av[0] = a0.x; av[1] = a0.y; av[2] = a0.z; av[3] = a0.w;
            av[4] = a1.x; av[5] = a1.y; av[6] = a1.z; av[7] = a1.w;
            bv[0] = b0.x; bv[1] = b0.y; bv[2] = b0.z; bv[3] = b0.w;
            bv[4] = b1.x; bv[5] = b1.y; bv[6] = b1.z; bv[7] = b1.w;
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    if (MODE == 2)
                        acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
                    else
                        acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(av[i], bv[j]));
                }
        }
        if (t + 1 < ktiles) store_tile(buf ^ 1);
        __syncthreads();
    }

#pragma unroll
    for (int i = 0; i < 8; i++) {
        int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
            if (n >= N) continue;
            if (MODE == 0) {
                Cout[(size_t)m * N + n] = acc[i][j];
            } else if (MODE == 2) {
                float y = acc[i][j] * __ldg(epi.scales + n);
                if (epi.bias) y += __ldg(epi.bias + n);
                Cout[(size_t)m * N + n] = apply_act(y, epi.act);
            } else {
                int hw = g.OH * g.OW;
                int b = m / hw, p = m - b * hw;
                Cout[((size_t)b * g.OC + n) * hw + p] = acc[i][j];
            }
        }
    }
}

// Small-output MatMul (MODE 0 arithmetic): 16x16 outputs per 256-thread CTA,
// one output per thread, k-slices of 32 through shared memory. Used when the
// 128x128 tiling would leave most SMs idle (e.g. [64,784]x[784,512]): the
// outputs are latency-bound sequential chains, so more of them run at once;
// the per-output RN multiply-then-add order is unchanged.
constexpr int SB = 16, SK = 32;
__global__ void __launch_bounds__(256) k_gemm_f32_small(const float *__restrict__ A, const float *__restrict__ B,
                                                       float *__restrict__ Cout, int M, int N, int K) {
    pdl_wait();
    pdl_trigger();
    __shared__ float As[SK][SB + 1];
    __shared__ float Bs[SK][SB + 1];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * SB, n0 = blockIdx.x * SB;
    float acc = 0.0f;
    for (int k0 = 0; k0 < K; k0 += SK) {
        // A tile [16 rows][32 k] and B tile [32 k][16 cols]: 2 values per thread each
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int e = tid + 256 * i;
            const int ar = e >> 5, ac = e & 31;
            const int m = m0 + ar, ka = k0 + ac;
            As[ac][ar] = (m < M && ka < K) ? A[(size_t)m * K + ka] : 0.0f;
            const int br = e >> 4, bc = e & 15;
            const int kb = k0 + br, n = n0 + bc;
            Bs[br][bc] = (kb < K && n < N) ? B[(size_t)kb * N + n] : 0.0f;
        }
        __syncthreads();
        if (K - k0 >= SK) {
#pragma unroll
            for (int kk = 0; kk < SK; kk++) acc = __fadd_rn(acc, __fmul_rn(As[kk][ty], Bs[kk][tx]));
        } else {
            for (int kk = 0; kk < K - k0; kk++) acc = __fadd_rn(acc, __fmul_rn(As[kk][ty], Bs[kk][tx]));
        }
        __syncthreads();
    }
    const int m = m0 + ty, n = n0 + tx;
    if (m < M && n < N) Cout[(size_t)m * N + n] = acc;
}

// ONNX Gemm, Y = alpha * op(A) op(B) + beta * C (C: none, [N] broadcast, or
// [M,N]): the small-tile structure above with transposable operands (each tile
// load walks the operand's contiguous dimension with consecutive threads), the
// same per-output sequential RN multiply-then-add, and an epilogue that rounds
// alpha*acc, beta*c and their sum separately.
template <bool TA, bool TB>
__global__ void __launch_bounds__(256) k_gemm_onnx(const float *__restrict__ A, const float *__restrict__ B,
                                                  const float *__restrict__ Cm, int c_mode, float alpha, float beta,
                                                  float *__restrict__ Y, int M, int N, int K) {
    pdl_wait();
    pdl_trigger();
    __shared__ float As[SK][SB + 1];
    __shared__ float Bs[SK][SB + 1];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * SB, n0 = blockIdx.x * SB;
    float acc = 0.0f;
    for (int k0 = 0; k0 < K; k0 += SK) {
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int e = tid + 256 * i;
            {
                const int r = TA ? (e & 15) : (e >> 5), c = TA ? (e >> 4) : (e & 31);
                const int m = m0 + r, ka = k0 + c;
                float v = 0.0f;
                if (m < M && ka < K) v = TA ? A[(size_t)ka * M + m] : A[(size_t)m * K + ka];
                As[c][r] = v;
            }
            {
                const int kr = TB ? (e & 31) : (e >> 4), nc = TB ? (e >> 5) : (e & 15);
                const int kb = k0 + kr, n = n0 + nc;
                float v = 0.0f;
                if (kb < K && n < N) v = TB ? B[(size_t)n * K + kb] : B[(size_t)kb * N + n];
                Bs[kr][nc] = v;
            }
        }
        __syncthreads();
        if (K - k0 >= SK) {
#pragma unroll
            for (int kk = 0; kk < SK; kk++) acc = __fadd_rn(acc, __fmul_rn(As[kk][ty], Bs[kk][tx]));
        } else {
            for (int kk = 0; kk < K - k0; kk++) acc = __fadd_rn(acc, __fmul_rn(As[kk][ty], Bs[kk][tx]));
        }
        __syncthreads();
    }
    const int m = m0 + ty, n = n0 + tx;
    if (m < M && n < N) {
        float y = __fmul_rn(alpha, acc);
        if (c_mode) y = __fadd_rn(y, __fmul_rn(beta, c_mode == 1 ? Cm[n] : Cm[(size_t)m * N + n]));
        Y[(size_t)m * N + n] = y;
    }
}

}  // namespace

int launch_gemm_onnx(tpt_cuda_ctx *ctx, const float *a, const float *b, const float *c, int c_mode, float alpha,
                     float beta, float *y, size_t m, size_t k, size_t n, bool ta, bool tb) {
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return TPT_UNSUPPORTED;
    dim3 g((unsigned)((n + SB - 1) / SB), (unsigned)((m + SB - 1) / SB));
    if (g.y > 65535) return TPT_UNSUPPORTED;
#define TPT_ONNX(TA_, TB_)                                                                                     \
    launch_pdl(k_gemm_onnx<TA_, TB_>, g, 256, 0, ctx->stream, a, b, c, c_mode, alpha, beta, y, (int)m, (int)n, (int)k)
    if (ta && tb)
        TPT_ONNX(true, true);
    else if (ta)
        TPT_ONNX(true, false);
    else if (tb)
        TPT_ONNX(false, true);
    else
        TPT_ONNX(false, false);
#undef TPT_ONNX
    return after_launch(ctx, "gemm_onnx");
}

int launch_matmul_f32(tpt_cuda_ctx *ctx, const float *a, const float *b, float *out, size_t m, size_t k,
                      size_t n) {
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return TPT_UNSUPPORTED;
    if (k == 0) {
        cudaError_t e = cudaMemsetAsync(out, 0, m * n * 4, ctx->stream);
        return e == cudaSuccess ? TPT_OK : cuda_fail(ctx, e, "matmul k=0 memset");
    }
    dim3 grid((unsigned)((n + BN - 1) / BN), (unsigned)((m + BM - 1) / BM));
    if ((size_t)grid.x * grid.y < (size_t)ctx->sm_count) {
        dim3 sg((unsigned)((n + SB - 1) / SB), (unsigned)((m + SB - 1) / SB));
        if (sg.y > 65535) return TPT_UNSUPPORTED;
        launch_pdl(k_gemm_f32_small, sg, 256, 0, ctx->stream, a, b, out, (int)m, (int)n, (int)k);
        return after_launch(ctx, "matmul_f32_small");
    }
    if (grid.y > 65535) return TPT_UNSUPPORTED;
    ConvGeom g{};
    launch_pdl(k_gemm_f32<0>, grid, NT, 0, ctx->stream, a, b, out, (int)m, (int)n, (int)k, g, W4Epi{});
    return after_launch(ctx, "matmul_f32");
}

int launch_conv2d_f32(tpt_cuda_ctx *ctx, const float *in, const float *w, float *out, const size_t is[4],
                      const size_t ws[4], size_t oh, size_t ow, size_t sh, size_t sw, size_t ph,
                      size_t pw) {
    size_t M = is[0] * oh * ow, N = ws[0], K = ws[1] * ws[2] * ws[3];
    if (M > INT32_MAX || K > INT32_MAX || is[0] * is[1] * is[2] * is[3] > (size_t)1 << 40)
        return TPT_UNSUPPORTED;
    if (K == 0) {
        cudaError_t e = cudaMemsetAsync(out, 0, M * N * 4, ctx->stream);
        return e == cudaSuccess ? TPT_OK : cuda_fail(ctx, e, "conv k=0 memset");
    }
    ConvGeom g{(int)is[1], (int)is[2], (int)is[3], (int)ws[2], (int)ws[3], (int)oh, (int)ow,
               (int)sh, (int)sw, (int)ph, (int)pw, (int)ws[0]};
    dim3 grid((unsigned)((N + BN - 1) / BN), (unsigned)((M + BM - 1) / BM));
    if (grid.y > 65535) return TPT_UNSUPPORTED;
    launch_pdl(k_gemm_f32<1>, grid, NT, 0, ctx->stream, in, w, out, (int)M, (int)N, (int)K, g, W4Epi{});
    return after_launch(ctx, "conv2d_f32");
}

int launch_w4_simt(tpt_cuda_ctx *ctx, const float *x, const uint8_t *packed, const float *scales, const float *bias,
                   int act, float *y, size_t m, size_t n, size_t k) {
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return TPT_UNSUPPORTED;
    dim3 grid((unsigned)((n + BN - 1) / BN), (unsigned)((m + BM - 1) / BM));
    if (grid.y > 65535) return TPT_UNSUPPORTED;
    ConvGeom g{};
    launch_pdl(k_gemm_f32<2>, grid, NT, 0, ctx->stream, x, reinterpret_cast<const float *>(packed), y, (int)m, (int)n,
                                                (int)k, g, W4Epi{scales, bias, act});
    return after_launch(ctx, "w4_simt");
}

}  // namespace tpt
