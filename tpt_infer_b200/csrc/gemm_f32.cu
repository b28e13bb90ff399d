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
#include "tc_common.cuh"

namespace tpt {

bool make_tmap_2d(CUtensorMap *tm, CUtensorMapDataType dt, const void *base, uint64_t rows, uint64_t cols,
                  uint32_t elem_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz);

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

// Small-output MatMul with all of K resident in shared memory (K <= MK_KMAX),
// and the bias + activation of the plan's MatMul fused into its epilogue.
// Each output is the same sequential chain as above (k ascending, RN multiply
// then RN add), so it is latency-bound: the kernel's job is to have every
// operand in shared memory before its chain needs it. A CTA (128 threads)
// owns 16 rows x 16 columns; thread (ty, tx) computes row ty, columns 2 tx and
// 2 tx + 1 as two interleaved chains. Right after
// the dependency wait every thread issues its cp.async copies of all of K
// (16-byte where rows are 16-byte aligned, else 4-byte), one mbarrier per
// 64-k chunk, so the chains start on chunk 0 while the later chunks land.
// Padding rows / columns / k are zero-filled; the chain stops at K.
constexpr int MK_T = 128;
constexpr int MK_KC = 64;
constexpr int MK_KMAX = 1536;  // A and B tiles: 128 K bytes, 192 KB at most
constexpr int MK_MAXC = MK_KMAX / MK_KC;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void *src, bool valid) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(valid ? 4 : 0) : "memory");
}

// TMA: with 16-byte aligned rows the tiles come in as tensor boxes instead
// (A: 16 rows x 64 floats = 256-byte lines, B: 64 k rows x 16 floats per
// chunk), one thread issuing them: the TMA unit fills shared memory faster
// than per-thread 16-byte copies here. A then sits chunk-major
// ([chunk][16][64]); B keeps the [k][16] layout.
template <bool TMA>
__global__ void __launch_bounds__(MK_T) k_matmul_f32_rows(const __grid_constant__ CUtensorMap tmA,
                                                          const __grid_constant__ CUtensorMap tmB,
                                                          const float *__restrict__ A, const float *__restrict__ B,
                                                          const float *__restrict__ bias, int act,
                                                          float *__restrict__ Cout, int M, int N, int K, int vecA,
                                                          int vecB, unsigned *gflags, float *__restrict__ Ysm) {
    using namespace tc;
    extern __shared__ __align__(16) float mk_smem[];
    __shared__ __align__(8) uint64_t bars[MK_MAXC];
    __shared__ int abort_flag;
    const int nch = (K + MK_KC - 1) / MK_KC, Kp = nch * MK_KC;
    const uint32_t raw = smem_u32(mk_smem), as = (raw + 127u) & ~127u, bs = as + 64u * (uint32_t)Kp;
    float *As = mk_smem + (as - raw) / 4;  // [16][Kp], or [chunk][16][64] with TMA
    float *Bs = As + 16 * Kp;              // [Kp][16]
    const int tid = threadIdx.x, ty = tid >> 3, tx = tid & 7;
    const int m0 = blockIdx.y * 16, n0 = blockIdx.x * 16;
    if (tid == 0) {
        abort_flag = 0;
        for (int c = 0; c < nch; c++) mbar_init(smem_u32(&bars[c]), TMA ? 1 : MK_T);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_wait();  // A and B may be the previous kernel's outputs
    pdl_trigger();
    if constexpr (TMA) {
        if (tid == 0) {
            for (int c = 0; c < nch; c++) {
                const uint32_t bar = smem_u32(&bars[c]);
                mbar_arrive_expect_tx(bar, 2u * 16u * MK_KC * 4u);  // out-of-range rows / columns / k read as 0
                tma_load_2d(as + (uint32_t)c * 16u * MK_KC * 4u, &tmA, bar, c * MK_KC, m0);
                tma_load_2d(bs + (uint32_t)c * MK_KC * 16u * 4u, &tmB, bar, n0, c * MK_KC);
            }
        }
    } else
    for (int c = 0; c < nch; c++) {
        const int kc = c * MK_KC;
        if (vecA) {  // 16 rows x 16 four-float pieces
            for (int e = tid; e < 256; e += MK_T) {
                const int r = e >> 4, k = kc + 4 * (e & 15), m = m0 + r;
                const bool v = m < M && k < K;  // K % 4 == 0
                cp_async16(as + 4u * (uint32_t)(r * Kp + k), v ? A + (size_t)m * K + k : A, v);
            }
        } else {
            for (int e = tid; e < 1024; e += MK_T) {
                const int r = e >> 6, k = kc + (e & 63), m = m0 + r;
                const bool v = m < M && k < K;
                cp_async4(as + 4u * (uint32_t)(r * Kp + k), v ? A + (size_t)m * K + k : A, v);
            }
        }
        if (vecB) {  // 64 k rows x 4 four-float pieces
            for (int e = tid; e < 256; e += MK_T) {
                const int k = kc + (e >> 2), j = 4 * (e & 3), n = n0 + j;
                const bool v = k < K && n < N;  // N % 4 == 0
                cp_async16(bs + 4u * (uint32_t)(k * 16 + j), v ? B + (size_t)k * N + n : B, v);
            }
        } else {
            for (int e = tid; e < 1024; e += MK_T) {
                const int k = kc + (e >> 4), j = e & 15, n = n0 + j;
                const bool v = k < K && n < N;
                cp_async4(bs + 4u * (uint32_t)(k * 16 + j), v ? B + (size_t)k * N + n : B, v);
            }
        }
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&bars[c])) : "memory");
    }
    float acc0 = 0.0f, acc1 = 0.0f;  // columns 2 tx and 2 tx + 1: two independent chains
    volatile int *abort_p = &abort_flag;
    bool ok = true;
    for (int c = 0; c < nch && ok; c++) {
        ok = mbar_wait(smem_u32(&bars[c]), 0u, abort_p, gflags, true);
        if (!ok) break;
        const float *ar = TMA ? As + (c * 16 + ty) * MK_KC : As + ty * Kp + c * MK_KC;
        const float *br = Bs + (size_t)c * MK_KC * 16 + 2 * tx;
        const int kn = min(MK_KC, K - c * MK_KC);
        if (kn == MK_KC) {
            // the whole chunk unrolled: its loads can be issued well ahead of
            // the chains (one warp per SMSP has nothing else to hide them behind)
#pragma unroll
            for (int kk = 0; kk < MK_KC; kk += 4) {
                const float4 a4 = *reinterpret_cast<const float4 *>(ar + kk);
                const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float2 b = *reinterpret_cast<const float2 *>(br + (kk + i) * 16);
                    acc0 = __fadd_rn(acc0, __fmul_rn(av[i], b.x));
                    acc1 = __fadd_rn(acc1, __fmul_rn(av[i], b.y));
                }
            }
        } else {
            for (int kk = 0; kk < kn; kk++) {
                const float2 b = *reinterpret_cast<const float2 *>(br + kk * 16);
                acc0 = __fadd_rn(acc0, __fmul_rn(ar[kk], b.x));
                acc1 = __fadd_rn(acc1, __fmul_rn(ar[kk], b.y));
            }
        }
    }
    if (TMA) {
        if (!ok && tid == 0)  // (after an abort) the boxes in flight land before the CTA exits
            for (int c = 0; c < nch; c++) mbar_wait(smem_u32(&bars[c]), 0u, abort_p, gflags, false);
    } else {
        asm volatile("cp.async.wait_all;" ::: "memory");  // (after an abort) no copy lands after the CTA exits
    }
    __shared__ float zt[16][17];  // the tile's outputs, for a fused softmax
    if (!__syncthreads_and(ok)) return;
    const float v[2] = {acc0, acc1};
    const int m = m0 + ty;
    if (m < M) {
#pragma unroll
        for (int j = 0; j < 2; j++) {
            const int n = n0 + 2 * tx + j;
            if (n >= N) continue;
            float y = v[j];
            if (bias) y = __fadd_rn(y, __ldg(bias + n));
            y = apply_act(y, act);
            Cout[(size_t)m * N + n] = y;
            zt[ty][2 * tx + j] = y;
        }
    }
    if (!Ysm) return;
    // Softmax of each row (N <= 16: one tile holds whole rows), written to
    // Ysm with k_softmax_warp's operations and order (a warp per row, lane j
    // holding element j), so the result is that kernel's, bit for bit
    __syncthreads();
    const int lane = tid & 31, warp = tid >> 5;
    for (int r = warp; r < 16; r += MK_T / 32) {
        const int mr = m0 + r;
        if (mr >= M) break;
        float mx = -INFINITY;
        if (lane < N) mx = fmaxf(mx, zt[r][lane]);
        mx = warp_max(mx);
        float s = 0.0f, e = 0.0f;
        if (lane < N) {
            e = expf(zt[r][lane] - mx);
            s += e;
        }
        s = warp_sum(s);
        if (lane < N) Ysm[(size_t)mr * N + lane] = __fdiv_rn(e, s);
    }
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

// The resident-K small-output kernel when it applies (the 128 x 128 tiling
// would leave SMs idle and 1 <= K <= MK_KMAX); handled = false otherwise.
static int launch_matmul_rows(tpt_cuda_ctx *ctx, const float *a, const float *b, const float *bias, int act,
                              float *out, size_t m, size_t k, size_t n, bool *handled, float *softmax_out = nullptr) {
    *handled = false;
    if (softmax_out && n > 16) return TPT_OK;
    const size_t tiles128 = ((n + BN - 1) / BN) * ((m + BM - 1) / BM);
    if (m == 0 || n == 0 || k == 0 || k > (size_t)MK_KMAX || tiles128 >= (size_t)ctx->sm_count || (m + 15) / 16 > 65535 ||
        m > INT32_MAX || n > INT32_MAX || (((uintptr_t)a | (uintptr_t)b) & 3))
        return TPT_OK;
    static bool attr_done[64] = {};
    const int dev = ctx->device & 63;
    if (!attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(k_matmul_f32_rows<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             128 * MK_KMAX + 128);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_matmul_f32_rows<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     128 * MK_KMAX + 128);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "matmul_f32_rows smem attribute");
        attr_done[dev] = true;
    }
    const size_t kp = (k + MK_KC - 1) / MK_KC * MK_KC;
    const int vec_a = (k % 4 == 0 && ((uintptr_t)a & 15) == 0) ? 1 : 0;
    const int vec_b = (n % 4 == 0 && ((uintptr_t)b & 15) == 0) ? 1 : 0;
    CUtensorMap ta, tb;
    const bool tma = vec_a && vec_b &&
                     make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, a, m, k, 4, MK_KC, 16,
                                  CU_TENSOR_MAP_SWIZZLE_NONE) &&
                     make_tmap_2d(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, b, k, n, 4, 16, MK_KC, CU_TENSOR_MAP_SWIZZLE_NONE);
    dim3 grid((unsigned)((n + 15) / 16), (unsigned)((m + 15) / 16));
    *handled = true;
    if (tma)
        launch_pdl(k_matmul_f32_rows<true>, grid, MK_T, 128 * kp + 128, ctx->stream, ta, tb, a, b, bias, act, out,
                   (int)m, (int)n, (int)k, vec_a, vec_b, ctx->d_flags, softmax_out);
    else
        launch_pdl(k_matmul_f32_rows<false>, grid, MK_T, 128 * kp + 128, ctx->stream, ta, tb, a, b, bias, act, out,
                   (int)m, (int)n, (int)k, vec_a, vec_b, ctx->d_flags, softmax_out);
    return after_launch(ctx, "matmul_f32_rows");
}

// MatMul followed by the plan's bias + activation: one launch where the
// resident-K kernel applies, else the MatMul and then k_bias_act
int launch_matmul_f32_epi(tpt_cuda_ctx *ctx, const float *a, const float *b, const float *bias, int act, float *out,
                          size_t m, size_t k, size_t n) {
    bool handled = false;
    int st = launch_matmul_rows(ctx, a, b, bias, act, out, m, k, n, &handled);
    if (st || handled) return st;
    st = launch_matmul_f32(ctx, a, b, out, m, k, n);
    if (st || (!bias && act == 0)) return st;
    return launch_bias_act(ctx, out, bias, out, m, n, act);
}

// MatMul (+ bias, activation) followed by a Softmax over its rows (n <= 16)
// in one launch, both outputs written; handled = false when the resident-K
// kernel does not apply
int launch_matmul_f32_softmax(tpt_cuda_ctx *ctx, const float *a, const float *b, const float *bias, int act,
                              float *out, float *softmax_out, size_t m, size_t k, size_t n, bool *handled) {
    return launch_matmul_rows(ctx, a, b, bias, act, out, m, k, n, handled, softmax_out);
}

int launch_matmul_f32(tpt_cuda_ctx *ctx, const float *a, const float *b, float *out, size_t m, size_t k,
                      size_t n) {
    {
        bool handled = false;
        int st = launch_matmul_rows(ctx, a, b, nullptr, 0, out, m, k, n, &handled);
        if (st || handled) return st;
    }
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
