// w8a8.cu -- INT8 weight x INT8 activation GEMMs with i32 accumulation and the
// fused per-output-channel dequant epilogue: the per-channel extension of
// quantized_matmul_i8 (crates/tpt-infer-quantize/src/ptq.rs:293-324),
//   y[m,n] = (float)acc[m,n] * (a_scale * w_scale[n]) + bias[n], then act,
// with the scale product formed first, and round-to-nearest multiply and add
// kept separate (no FMA) so the f32 output is bit-exact with the oracle.
//
// Kernels here:
//  - k_w8a8_gemv: M <= 4. One warp per output channel streams the K-contiguous
//    weight row with 128-bit loads (all of a pass in flight) and dp4a.
//  - k_w8a8_simt: general shapes (ragged M/N, K % 16 == 0); dp4a tiles.
//  - 3 <= M <= 32 (uploaded weights, K <= 4096): the TMA-ring mma.sync kernel
//    of w8a8_mma.cu;
//  - the tcgen05 tensor-core kernels: K split over a thread-block cluster
//    for 4 < M <= 64 in w8a8_ck.cu, SM-pair tiles for larger M in w8a8_tc.cu.
// Weight layout in HBM: W^T [n, k] int8 row-major (K-major B operand), which
// is the byte layout quantize_i8_symmetric_per_channel(W^T, rows = n) emits.
#include <string.h>

#include <new>

#include "tc_common.cuh"

namespace tpt {

int launch_w8a8_tc(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, const tpt_cuda_weights *w, float a_scale,
                   const float *bias, int act, float *y, int32_t *acc, bool *handled, Requant rq);
int build_weight_tmap(tpt_cuda_weights *w);
int launch_w8a8_ck(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, const tpt_cuda_weights *w, float a_scale,
                   const float *bias, int act, float *y, int32_t *acc, bool *handled, Requant rq);
int launch_w8a8_mma(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, const tpt_cuda_weights *w, float a_scale,
                    const float *bias, int act, float *y, int32_t *acc, bool *handled, Requant rq);

namespace {

__device__ __forceinline__ float w8a8_epilogue(int32_t acc, float a_scale, float ws, const float *bias, int n,
                                               int act) {
    float y = __fmul_rn((float)acc, __fmul_rn(a_scale, ws));
    if (bias) y = __fadd_rn(y, __ldg(bias + n));
    return apply_act(y, act);
}

__device__ __forceinline__ int dot16(int4 a, int4 b, int acc) {
    acc = __dp4a(a.x, b.x, acc);
    acc = __dp4a(a.y, b.y, acc);
    acc = __dp4a(a.z, b.z, acc);
    acc = __dp4a(a.w, b.w, acc);
    return acc;
}

// One warp per output channel: block b takes the channels [N b / G, N (b + 1) / G)
// (G blocks; two per SM, so every SM streams the same number of rows to within
// one), its warps in turn. Each lane owns 16-byte chunks
// c = lane + 32 j of the row, j < 8, so a warp covers 4 KB of K per pass and
// every load of the pass is issued before the first dp4a: a warp keeps 4 KB in
// flight and the activations stay in registers (A_REG, M <= 2, K <= 4096) or in
// L1 (reloaded per row, the lines are shared by every warp of the SM).
constexpr int GEMV_CH = 8;  // 16-byte chunks per lane per pass

template <int MM, bool A_REG>
__global__ void __launch_bounds__(256, 2) k_w8a8_gemv(const int8_t *__restrict__ A, const int8_t *__restrict__ Wt,
                                                   const float *__restrict__ wscale, const float *__restrict__ bias,
                                                   int M, int N, int K, float a_scale, int act,
                                                   float *__restrict__ Y, int32_t *__restrict__ ACC,
                                                   int8_t *__restrict__ Q, float q_scale) {
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int n_begin = (int)((long long)N * blockIdx.x / gridDim.x) + warp;
    const int n_end = (int)((long long)N * (blockIdx.x + 1) / gridDim.x);
    const int chunks = K >> 4;  // 16-byte chunks per row
    // this warp's weight rows start streaming into L2 while the previous
    // kernel on the stream finishes (the grid is small enough to be resident
    // beside it); the loads below then hit L2
    for (int n = n_begin + lane * nwarps; n < n_end; n += 32 * nwarps)
        for (int c = 0; c < K; c += 32768) prefetch_l2_bulk(Wt + (size_t)n * K + c, (uint32_t)min(K - c, 32768));
    pdl_wait();
    pdl_trigger();
    int4 ar[A_REG ? MM : 1][GEMV_CH];
    if (A_REG) {
#pragma unroll
        for (int i = 0; i < MM; i++)
#pragma unroll
            for (int j = 0; j < GEMV_CH; j++) {
                const int c = lane + 32 * j;
                ar[i][j] = (i < M && c < chunks) ? __ldg(reinterpret_cast<const int4 *>(A + (size_t)i * K) + c)
                                                 : make_int4(0, 0, 0, 0);
            }
    }
    if constexpr (MM == 1 && A_REG) {
        // one row of activations, one pass per row (K <= 4096): a warp's rows are
        // taken two at a time with both rows' loads issued before the first
        // dp4a, so the ~1.7 rows a warp holds at K = N = 4096 stream in one
        // round trip instead of two (8 KB in flight per warp, 128 KB per SM)
        for (int n = n_begin; n < n_end; n += 2 * nwarps) {
            const int n2 = n + nwarps;
            const bool two = n2 < n_end;
            const int4 *w0 = reinterpret_cast<const int4 *>(Wt + (size_t)n * K);
            const int4 *w1 = reinterpret_cast<const int4 *>(Wt + (size_t)(two ? n2 : n) * K);
            int4 wa[GEMV_CH], wb[GEMV_CH];
#pragma unroll
            for (int j = 0; j < GEMV_CH; j++) {
                const int c = lane + 32 * j;
                wa[j] = c < chunks ? __ldcs(w0 + c) : make_int4(0, 0, 0, 0);
                wb[j] = (two && c < chunks) ? __ldcs(w1 + c) : make_int4(0, 0, 0, 0);
            }
            int acc0 = 0, acc1 = 0;
#pragma unroll
            for (int j = 0; j < GEMV_CH; j++) {
                acc0 = dot16(ar[0][j], wa[j], acc0);
                acc1 = dot16(ar[0][j], wb[j], acc1);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                acc0 += __shfl_xor_sync(0xffffffffu, acc0, o);
                acc1 += __shfl_xor_sync(0xffffffffu, acc1, o);
            }
            if (lane == 0) {
                const float ws0 = __ldg(wscale + n);
                if (ACC)
                    ACC[n] = acc0;
                else if (Q)
                    Q[n] = requant_i8(w8a8_epilogue(acc0, a_scale, ws0, bias, n, act), q_scale);
                else
                    Y[n] = w8a8_epilogue(acc0, a_scale, ws0, bias, n, act);
                if (two) {
                    const float ws1 = __ldg(wscale + n2);
                    if (ACC)
                        ACC[n2] = acc1;
                    else if (Q)
                        Q[n2] = requant_i8(w8a8_epilogue(acc1, a_scale, ws1, bias, n2, act), q_scale);
                    else
                        Y[n2] = w8a8_epilogue(acc1, a_scale, ws1, bias, n2, act);
                }
            }
        }
    } else {
    for (int n = n_begin; n < n_end; n += nwarps) {
        const int4 *wrow = reinterpret_cast<const int4 *>(Wt + (size_t)n * K);
        int acc[MM];
#pragma unroll
        for (int i = 0; i < MM; i++) acc[i] = 0;
        for (int c0 = 0; c0 < chunks; c0 += 32 * GEMV_CH) {
            int4 w[GEMV_CH];
#pragma unroll
            for (int j = 0; j < GEMV_CH; j++) {
                const int c = c0 + lane + 32 * j;
                w[j] = c < chunks ? __ldcs(wrow + c) : make_int4(0, 0, 0, 0);
            }
#pragma unroll
            for (int i = 0; i < MM; i++) {
                if (i >= M) break;
                const int4 *arow = reinterpret_cast<const int4 *>(A + (size_t)i * K);
#pragma unroll
                for (int j = 0; j < GEMV_CH; j++) {
                    const int c = c0 + lane + 32 * j;
                    int4 a;
                    if (A_REG)
                        a = ar[i][j];
                    else
                        a = c < chunks ? __ldg(arow + c) : make_int4(0, 0, 0, 0);
                    acc[i] = dot16(a, w[j], acc[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < MM; i++) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
        }
        if (lane == 0) {
            const float ws = __ldg(wscale + n);
#pragma unroll
            for (int i = 0; i < MM; i++) {
                if (i < M) {
                    if (ACC)
                        ACC[(size_t)i * N + n] = acc[i];
                    else if (Q)
                        Q[(size_t)i * N + n] = requant_i8(w8a8_epilogue(acc[i], a_scale, ws, bias, n, act), q_scale);
                    else
                        Y[(size_t)i * N + n] = w8a8_epilogue(acc[i], a_scale, ws, bias, n, act);
                }
            }
        }
    }
    }
}

// Small W8A8 (M <= 64, K <= 1536, K % 16 == 0, few output tiles): all of K
// resident in shared memory, dp4a. A CTA (128 threads) owns 16 activation rows
// x 16 output channels; thread (ty, tx) computes row ty, channels tx and tx + 8.
// Right after the dependency wait every thread issues its 16-byte cp.async
// copies of the 16 activation rows and 16 weight rows (rows padded by 16 bytes
// so that the 8 channel rows a warp reads at one k fall in distinct banks),
// one mbarrier per 64-k chunk, so the sums start on chunk 0 while the later
// chunks land. Padding rows and k are zero-filled (zero products). Integer
// sums are exact, then the same w8a8_epilogue as the other kernels. For the
// short layers (an MLP's 64 x 784 x 512, a 10-way head) where the
// tensor-core kernels' fixed cost (TMEM, clusters, rings) is most of their
// time.
constexpr int WR_T = 128;
constexpr int WR_KC = 64;
constexpr int WR_KMAX = 1536;
constexpr int WR_MAXC = WR_KMAX / WR_KC;

__global__ void __launch_bounds__(WR_T) k_w8a8_rows(const int8_t *__restrict__ A, const int8_t *__restrict__ Wt,
                                                    const float *__restrict__ wscale, const float *__restrict__ bias,
                                                    int M, int N, int K, float a_scale, int act,
                                                    float *__restrict__ Y, int32_t *__restrict__ ACC,
                                                    int8_t *__restrict__ Q, float q_scale, unsigned *gflags) {
    using namespace tc;
    extern __shared__ __align__(16) uint8_t wr_smem[];
    __shared__ __align__(8) uint64_t bars[WR_MAXC];
    __shared__ int abort_flag;
    const int nch = (K + WR_KC - 1) / WR_KC, rs = nch * WR_KC + 16;  // padded row stride
    const int tid = threadIdx.x, ty = tid >> 3, tx = tid & 7;
    const int m0 = blockIdx.y * 16, n0 = blockIdx.x * 16;
    const uint8_t *As = wr_smem, *Ws = wr_smem + 16 * rs;
    if (tid == 0) {
        abort_flag = 0;
        for (int c = 0; c < nch; c++) mbar_init(smem_u32(&bars[c]), WR_T);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_wait();  // the activations are the previous kernel's output
    pdl_trigger();
    const uint32_t base = smem_u32(wr_smem);
    for (int c = 0; c < nch; c++) {
        // 32 rows (16 activation, 16 weight) x 4 sixteen-byte pieces: one per thread
        const int r = tid >> 2, k = c * WR_KC + 16 * (tid & 3);
        const bool is_w = r >= 16;
        const int row = is_w ? n0 + r - 16 : m0 + r;
        const bool v = (is_w ? row < N : row < M) && k < K;
        const int8_t *src = v ? (is_w ? Wt : A) + (size_t)row * K + k : A;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(base + (uint32_t)(r * rs + k)), "l"(src),
                     "r"(v ? 16 : 0)
                     : "memory");
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&bars[c])) : "memory");
    }
    volatile int *abort_p = &abort_flag;
    int acc0 = 0, acc1 = 0;
    bool ok = true;
    const uint8_t *ar = As + ty * rs, *w0 = Ws + tx * rs, *w1 = Ws + (tx + 8) * rs;
    for (int c = 0; c < nch && ok; c++) {
        ok = mbar_wait(smem_u32(&bars[c]), 0u, abort_p, gflags, true);
        if (!ok) break;
#pragma unroll
        for (int q = 0; q < WR_KC / 16; q++) {
            const int k = c * WR_KC + 16 * q;
            const int4 a = *reinterpret_cast<const int4 *>(ar + k);
            acc0 = dot16(a, *reinterpret_cast<const int4 *>(w0 + k), acc0);
            acc1 = dot16(a, *reinterpret_cast<const int4 *>(w1 + k), acc1);
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // (after an abort) no copy lands after the CTA exits
    if (!ok) return;
    const int m = m0 + ty;
    if (m >= M) return;
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const int n = n0 + tx + 8 * j;
        if (n >= N) continue;
        const int acc = j ? acc1 : acc0;
        if (ACC)
            ACC[(size_t)m * N + n] = acc;
        else {
            const float y = w8a8_epilogue(acc, a_scale, __ldg(wscale + n), bias, n, act);
            if (Q)
                Q[(size_t)m * N + n] = requant_i8(y, q_scale);
            else
                Y[(size_t)m * N + n] = y;
        }
    }
}

// General dp4a tile GEMM: 128x128 outputs per CTA, 8x8 per thread, K in
// 32-byte slices (K % 16 == 0; a trailing 16-byte half is zero-filled).
__global__ void __launch_bounds__(256) k_w8a8_simt(const int8_t *__restrict__ A, const int8_t *__restrict__ Wt,
                                                   const float *__restrict__ wscale, const float *__restrict__ bias,
                                                   int M, int N, int K, float a_scale, int act,
                                                   float *__restrict__ Y, int32_t *__restrict__ ACC,
                                                   int8_t *__restrict__ Q, float q_scale) {
    pdl_wait();
    pdl_trigger();
    __shared__ __align__(16) int As[2][8][128 + 4];
    __shared__ __align__(16) int Bs[2][8][128 + 4];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * 128, n0 = blockIdx.x * 128;
    const int lr = tid >> 1, lh = tid & 1;  // loader: row lr, 16-byte half lh
    int4 ra, rb;
    auto load = [&](int k0) {
        int kk = k0 + lh * 16;
        ra = make_int4(0, 0, 0, 0);
        rb = make_int4(0, 0, 0, 0);
        if (m0 + lr < M && kk < K) ra = __ldg(reinterpret_cast<const int4 *>(A + (size_t)(m0 + lr) * K + kk));
        if (n0 + lr < N && kk < K) rb = __ldg(reinterpret_cast<const int4 *>(Wt + (size_t)(n0 + lr) * K + kk));
    };
    auto store = [&](int buf) {
        As[buf][lh * 4 + 0][lr] = ra.x;
        As[buf][lh * 4 + 1][lr] = ra.y;
        As[buf][lh * 4 + 2][lr] = ra.z;
        As[buf][lh * 4 + 3][lr] = ra.w;
        Bs[buf][lh * 4 + 0][lr] = rb.x;
        Bs[buf][lh * 4 + 1][lr] = rb.y;
        Bs[buf][lh * 4 + 2][lr] = rb.z;
        Bs[buf][lh * 4 + 3][lr] = rb.w;
    };
    int acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[i][j] = 0;
    const int kt = (K + 31) / 32;
    load(0);
    store(0);
    __syncthreads();
    for (int t = 0; t < kt; t++) {
        const int buf = t & 1;
        if (t + 1 < kt) load((t + 1) * 32);
#pragma unroll
        for (int w = 0; w < 8; w++) {
            int av[8], bv[8];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                av[i] = As[buf][w][ty * 4 + i];
                av[4 + i] = As[buf][w][64 + ty * 4 + i];
                bv[i] = Bs[buf][w][tx * 4 + i];
                bv[4 + i] = Bs[buf][w][64 + tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 8; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) acc[i][j] = __dp4a(av[i], bv[j], acc[i][j]);
        }
        if (t + 1 < kt) store(buf ^ 1);
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
            if (n >= N) continue;
            if (ACC)
                ACC[(size_t)m * N + n] = acc[i][j];
            else if (Q)
                Q[(size_t)m * N + n] =
                    requant_i8(w8a8_epilogue(acc[i][j], a_scale, __ldg(wscale + n), bias, n, act), q_scale);
            else
                Y[(size_t)m * N + n] = w8a8_epilogue(acc[i][j], a_scale, __ldg(wscale + n), bias, n, act);
        }
    }
}

// [R, C] -> [C, R] byte transpose through 32x32 shared tiles.
__global__ void k_transpose_i8(const int8_t *__restrict__ src, int8_t *__restrict__ dst, int R, int Ccols) {
    __shared__ int8_t tile[32][33];
    int x = blockIdx.x * 32 + threadIdx.x, y = blockIdx.y * 32 + threadIdx.y;
    for (int j = 0; j < 32; j += 8)
        if (x < Ccols && y + j < R) tile[threadIdx.y + j][threadIdx.x] = src[(size_t)(y + j) * Ccols + x];
    __syncthreads();
    x = blockIdx.y * 32 + threadIdx.x;
    y = blockIdx.x * 32 + threadIdx.y;
    for (int j = 0; j < 32; j += 8)
        if (x < R && y + j < Ccols) dst[(size_t)(y + j) * R + x] = tile[threadIdx.x][threadIdx.y + j];
}

__global__ void k_fill_f32(float *p, size_t n, float v) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) p[i] = v;
}

}  // namespace

int launch_w8a8(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, size_t k, const tpt_cuda_weights *w, float a_scale,
                const float *bias, int act, float *y, int32_t *acc, Requant rq) {
    const size_t n = w->n;
    if (m == 0 || n == 0) return TPT_OK;
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return TPT_UNSUPPORTED;
    const int8_t *wt = (const int8_t *)w->data;
    if (m >= 3 && m <= 32) {
        bool handled = false;
        int st = launch_w8a8_mma(ctx, a, m, w, a_scale, bias, act, y, acc, &handled, rq);
        if (st || handled) return st;
    }
    if (m <= 4) {
        // decode-like: SIMT stream of the weight rows (HBM-bound)
        // two 8-warp blocks per SM: the next launch's blocks fit beside them
        // and prefetch their weights while this one runs
        unsigned g = grid_1d(n * 32, 256, (unsigned)ctx->sm_count * 2);
        const bool areg = k <= (size_t)GEMV_CH * 32 * 16;
#define TPT_GEMV(MM, AR) \
    launch_pdl(k_w8a8_gemv<MM, AR>, g, 256, 0, ctx->stream, a, wt, w->scales, bias, (int)m, (int)n, (int)k, a_scale, act, y, acc, \
                                                    rq.q, rq.scale)
        if (m == 1 && areg)
            TPT_GEMV(1, true);
        else if (m == 1)
            TPT_GEMV(1, false);
        else if (m == 2 && areg)
            TPT_GEMV(2, true);
        else
            TPT_GEMV(4, false);
#undef TPT_GEMV
        return after_launch(ctx, "w8a8_gemv");
    }
    if (m <= 64 && k % 16 == 0 && k <= (size_t)WR_KMAX && ((((uintptr_t)a) | ((uintptr_t)wt)) & 15) == 0 &&
        ((n + 15) / 16) * ((m + 15) / 16) <= (size_t)2 * ctx->sm_count) {
        // short layers: the resident-K dp4a kernel
        static bool attr_done[64] = {};
        const int dev = ctx->device & 63;
        if (!attr_done[dev]) {
            cudaError_t e = cudaFuncSetAttribute(k_w8a8_rows, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 32 * (WR_KMAX + 16));
            if (e != cudaSuccess) return cuda_fail(ctx, e, "w8a8_rows smem attribute");
            attr_done[dev] = true;
        }
        const size_t nch = (k + WR_KC - 1) / WR_KC;
        dim3 grid((unsigned)((n + 15) / 16), (unsigned)((m + 15) / 16));
        launch_pdl(k_w8a8_rows, grid, WR_T, 32 * (nch * WR_KC + 16), ctx->stream, a, wt, w->scales, bias, (int)m,
                   (int)n, (int)k, a_scale, act, y, acc, rq.q, rq.scale, ctx->d_flags);
        return after_launch(ctx, "w8a8_rows");
    }
    bool handled = false;
    if (m <= 64) {
        int st = launch_w8a8_ck(ctx, a, m, w, a_scale, bias, act, y, acc, &handled, rq);
        if (st || handled) return st;
    }
    int st = launch_w8a8_tc(ctx, a, m, w, a_scale, bias, act, y, acc, &handled, rq);
    if (st || handled) return st;
    dim3 grid((unsigned)((n + 127) / 128), (unsigned)((m + 127) / 128));
    if (grid.y > 65535) return TPT_UNSUPPORTED;
    launch_pdl(k_w8a8_simt, grid, 256, 0, ctx->stream, a, wt, w->scales, bias, (int)m, (int)n, (int)k, a_scale, act, y, acc,
                                               rq.q, rq.scale);
    return after_launch(ctx, "w8a8_simt");
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

int tpt_cuda_weights_upload_i8(tpt_cuda_ctx *ctx, const int8_t *wt, const float *scales, size_t n, size_t k,
                               tpt_cuda_weights **out) {
    CHECK_CTX(ctx);
    if (!out || !wt || !scales || n == 0 || k == 0 || k % 16 != 0) return TPT_INVALID;
    *out = nullptr;
    size_t bytes;
    if (!checked_mul(n, k, &bytes)) return TPT_INVALID;
    tpt_cuda_weights *w = new (std::nothrow) tpt_cuda_weights();
    if (!w) return TPT_OUT_OF_MEMORY;
    w->ctx = ctx;
    w->device = ctx->device;
    w->kind = 8;
    w->n = n;
    w->k = k;
    w->bytes = bytes;
    cudaError_t e = cudaMalloc(&w->data, bytes);
    if (e == cudaSuccess) e = cudaMalloc(&w->scales, n * sizeof(float));
    if (e == cudaSuccess) e = cudaMemcpy(w->data, wt, bytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(w->scales, scales, n * sizeof(float), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaGetLastError();
        if (w->data) cudaFree(w->data);
        if (w->scales) cudaFree(w->scales);
        delete w;
        return cuda_fail(ctx, e, "weights upload");
    }
    build_weight_tmap(w);
    *out = w;
    return TPT_OK;
}

// Needs only the weight's device (cudaFree waits for work using the memory),
// so a handle may outlive the context it was uploaded through.
int tpt_cuda_weights_free(tpt_cuda_weights *w) {
    if (!w) return TPT_INVALID;
    cudaSetDevice(w->device);
    if (w->data) cudaFree(w->data);
    if (w->scales) cudaFree(w->scales);
    delete w;
    return TPT_OK;
}

int tpt_cuda_weights_shape(const tpt_cuda_weights *w, size_t *n, size_t *k) {
    if (!w) return TPT_INVALID;
    if (n) *n = w->n;
    if (k) *k = w->k;
    return TPT_OK;
}

constexpr int PIPE_CHUNKS = 4;  // row chunks of a pipelined host-buffer call

int tpt_cuda_w8a8_gemm(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, size_t k, float a_scale,
                       const tpt_cuda_weights *w, const float *bias, int act, float *out) {
    CHECK_CTX(ctx);
    if (!w || w->kind != 8) return TPT_INVALID;
    if (k != w->k) return TPT_SHAPE_MISMATCH;
    if (act < 0 || act > 2) return TPT_INVALID;
    size_t an, on;
    if (!checked_mul(m, k, &an) || !checked_mul(m, w->n, &on)) return TPT_INVALID;
    if (on == 0) return TPT_OK;
    Staging st(ctx);
    st.reserve(an);
    st.reserve(on * 4);
    st.reserve(bias ? w->n * 4 : 0);
    TRY(st.commit());
    int8_t *da = st.take<int8_t>(an);
    float *dy = st.take<float>(on);
    float *db = bias ? st.take<float>(w->n) : nullptr;
    if (bias) TRY(h2d(ctx, db, bias, w->n * 4));
    // Large outputs from and to page-locked memory: row chunks pipelined, the
    // H2D of chunk c + 1, the GEMM of chunk c and the D2H of chunk c - 1 in
    // flight together (the two copy engines and the SMs), so the call costs
    // about the larger of the two transfers instead of their sum.
    const size_t rows = ((m + PIPE_CHUNKS - 1) / PIPE_CHUNKS + 127) / 128 * 128;
    if (on * 4 >= ((size_t)16 << 20) && rows < m && !ctx->capturing && is_pinned_host(a) && is_pinned_host(out)) {
        TRY(ensure_copy_streams(ctx));
        cudaEvent_t start = ctx->pipe_ev[2 * PIPE_CHUNKS], fin = ctx->pipe_ev[2 * PIPE_CHUNKS + 1];
        cudaError_t e = cudaEventRecord(start, ctx->stream);  // staging is free: prior work on the stream is done
        if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->copy_in, start, 0);
        for (int c = 0; e == cudaSuccess && (size_t)c * rows < m; c++) {
            const size_t r0 = (size_t)c * rows, rc = m - r0 < rows ? m - r0 : rows;
            cudaEvent_t in_done = ctx->pipe_ev[2 * c], gemm_done = ctx->pipe_ev[2 * c + 1];
            e = cudaMemcpyAsync(da + r0 * k, a + r0 * k, rc * k, cudaMemcpyHostToDevice, ctx->copy_in);
            if (e == cudaSuccess) e = cudaEventRecord(in_done, ctx->copy_in);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->stream, in_done, 0);
            if (e != cudaSuccess) break;
            TRY(launch_w8a8(ctx, da + r0 * k, rc, k, w, a_scale, db, act, dy + r0 * w->n, nullptr, Requant{}));
            e = cudaEventRecord(gemm_done, ctx->stream);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->copy_out, gemm_done, 0);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(out + r0 * w->n, dy + r0 * w->n, rc * w->n * 4, cudaMemcpyDeviceToHost,
                                    ctx->copy_out);
        }
        if (e == cudaSuccess) e = cudaEventRecord(fin, ctx->copy_out);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->stream, fin, 0);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "pipelined w8a8_gemm");
        return sync_and_check(ctx);
    }
    TRY(h2d(ctx, da, a, an));
    TRY(launch_w8a8(ctx, da, m, k, w, a_scale, db, act, dy, nullptr, Requant{}));
    TRY(d2h(ctx, out, dy, on * 4));
    return sync_and_check(ctx);
}

int tpt_cuda_w8a8_gemm_dev(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, float a_scale, const tpt_cuda_weights *w,
                           const float *bias, int act, float *out) {
    CHECK_CTX(ctx);
    if (!w || w->kind != 8 || act < 0 || act > 2) return TPT_INVALID;
    return launch_w8a8(ctx, a, m, w->k, w, a_scale, bias, act, out, nullptr, Requant{});
}

int tpt_cuda_w8a8_gemm_acc_dev(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, const tpt_cuda_weights *w,
                               int32_t *acc) {
    CHECK_CTX(ctx);
    if (!w || w->kind != 8 || !acc) return TPT_INVALID;
    return launch_w8a8(ctx, a, m, w->k, w, 1.0f, nullptr, 0, nullptr, acc, Requant{});
}

// ptq.rs:293-324, the reference contract: B [kb, n], per-tensor b_scales[0].
int tpt_cuda_quantized_matmul_i8(tpt_cuda_ctx *ctx, const int8_t *a, size_t a_len, size_t m, size_t k,
                                 float a_scale, const int8_t *b, size_t b_len, size_t kb, size_t n,
                                 const float *b_scales, size_t n_scales, float *out, size_t out_len) {
    CHECK_CTX(ctx);
    if (k != kb) return TPT_SHAPE_MISMATCH;
    size_t e1, e2, e3;
    if (!checked_mul(m, k, &e1) || !checked_mul(k, n, &e2) || !checked_mul(m, n, &e3)) return TPT_INVALID;
    if (a_len != e1 || b_len != e2 || out_len != e3) return TPT_SIZE_MISMATCH;
    if (e3 == 0) return TPT_OK;
    if (k > INT32_MAX || n > INT32_MAX || m > INT32_MAX) return TPT_UNSUPPORTED;
    const float b_scale = n_scales ? b_scales[0] : 1.0f;
    // K padded to a multiple of 16 with zero bytes (a zero product leaves the
    // i32 sum unchanged).
    const size_t kp = (k + 15) & ~size_t(15);
    Staging st(ctx);
    st.reserve(m * kp);
    st.reserve(k * n);   // B as given, [k, n]
    st.reserve(n * k);   // B^T dense, [n, k]
    st.reserve(n * kp);  // B^T with row pitch kp
    st.reserve(n * 4);
    st.reserve(e3 * 4);
    TRY(st.commit());
    int8_t *da = st.take<int8_t>(m * kp);
    int8_t *db = st.take<int8_t>(k * n);
    int8_t *dbt_dense = st.take<int8_t>(n * k);
    int8_t *dbt = st.take<int8_t>(n * kp);
    float *ds = st.take<float>(n);
    float *dy = st.take<float>(e3);
    cudaError_t ce = cudaSuccess;
    if (kp != k) {
        ce = cudaMemsetAsync(da, 0, m * kp, ctx->stream);
        if (ce == cudaSuccess) ce = cudaMemsetAsync(dbt, 0, n * kp, ctx->stream);
        if (ce == cudaSuccess) ce = cudaMemcpy2DAsync(da, kp, a, k, k, m, cudaMemcpyHostToDevice, ctx->stream);
    } else {
        ce = cudaMemcpyAsync(da, a, m * k, cudaMemcpyHostToDevice, ctx->stream);
    }
    if (ce != cudaSuccess) return cuda_fail(ctx, ce, "quantized_matmul_i8 staging");
    TRY(h2d(ctx, db, b, k * n));
    // transpose [k, n] -> [n, k], then lay the rows out at pitch kp
    dim3 tgrid((unsigned)((n + 31) / 32), (unsigned)((k + 31) / 32));
    if (tgrid.y > 65535) return TPT_UNSUPPORTED;
    k_transpose_i8<<<tgrid, dim3(32, 8), 0, ctx->stream>>>(db, kp == k ? dbt : dbt_dense, (int)k, (int)n);
    TRY(after_launch(ctx, "transpose_i8"));
    if (kp != k) {
        ce = cudaMemcpy2DAsync(dbt, kp, dbt_dense, k, k, n, cudaMemcpyDeviceToDevice, ctx->stream);
        if (ce != cudaSuccess) return cuda_fail(ctx, ce, "quantized_matmul_i8 repitch");
    }
    k_fill_f32<<<grid_1d(n, 256), 256, 0, ctx->stream>>>(ds, n, b_scale);
    TRY(after_launch(ctx, "fill"));
    tpt_cuda_weights w;
    w.ctx = ctx;
    w.kind = 8;
    w.n = n;
    w.k = kp;
    w.data = dbt;
    w.scales = ds;
    w.tmap_ok = false;  // transient weights: no tensor-map path
    // out = (float)acc * (a_scale * b_scale): the per-channel epilogue with every
    // channel scale equal to b_scale and no bias.
    TRY(launch_w8a8(ctx, da, m, kp, &w, a_scale, nullptr, 0, dy, nullptr, Requant{}));
    TRY(d2h(ctx, out, dy, e3 * 4));
    return sync_and_check(ctx);
}

// ------------------------------------------------------------------ quantize entry points
int tpt_cuda_quantize_i8_symmetric(tpt_cuda_ctx *ctx, const float *x, size_t n, int8_t *q, float *scale) {
    CHECK_CTX(ctx);
    if (!scale) return TPT_INVALID;
    if (n == 0) {
        *scale = 1.0f;  // max_abs of an empty slice is 0 -> scale 1.0
        return TPT_OK;
    }
    Staging st(ctx);
    st.reserve(n * 4);
    st.reserve(n);
    st.reserve(4);
    TRY(st.commit());
    float *dx = st.take<float>(n);
    int8_t *dq = st.take<int8_t>(n);
    float *ds = st.take<float>(1);
    TRY(h2d(ctx, dx, x, n * 4));
    TRY(launch_quant_i8_sym(ctx, dx, n, dq, ds, ctx->d_reduce));
    TRY(d2h(ctx, q, dq, n));
    TRY(d2h(ctx, scale, ds, 4));
    return sync_and_check(ctx);
}

int tpt_cuda_quantize_i8_symmetric_dev(tpt_cuda_ctx *ctx, const float *x, size_t n, int8_t *q, float *scale_dev) {
    CHECK_CTX(ctx);
    if (n == 0) return TPT_OK;
    return launch_quant_i8_sym(ctx, x, n, q, scale_dev, ctx->d_reduce);
}

int tpt_cuda_quantize_i8_static_dev(tpt_cuda_ctx *ctx, const float *x, size_t n, float scale, int8_t *q) {
    CHECK_CTX(ctx);
    if (n == 0) return TPT_OK;
    return launch_quant_i8_static(ctx, x, n, scale, q);
}

int tpt_cuda_quantize_i8_symmetric_per_channel(tpt_cuda_ctx *ctx, const float *x, size_t len, size_t rows,
                                               int8_t *q, float *scales) {
    CHECK_CTX(ctx);
    if (rows == 0 || len % rows != 0) return TPT_INVALID;  // quant.rs:96 assert
    if (len == 0) {
        for (size_t r = 0; r < rows; r++) scales[r] = 1.0f;
        return TPT_OK;
    }
    const size_t cols = len / rows;
    Staging st(ctx);
    st.reserve(len * 4);
    st.reserve(len);
    st.reserve(rows * 4);
    TRY(st.commit());
    float *dx = st.take<float>(len);
    int8_t *dq = st.take<int8_t>(len);
    float *ds = st.take<float>(rows);
    TRY(h2d(ctx, dx, x, len * 4));
    TRY(launch_quant_i8_rows(ctx, dx, rows, cols, dq, ds));
    TRY(d2h(ctx, q, dq, len));
    TRY(d2h(ctx, scales, ds, rows * 4));
    return sync_and_check(ctx);
}

int tpt_cuda_quantize_i8_asymmetric(tpt_cuda_ctx *ctx, const float *x, size_t n, int8_t *q, float *scale,
                                    int32_t *zero_point) {
    CHECK_CTX(ctx);
    if (!scale || !zero_point) return TPT_INVALID;
    if (n == 0) {
        // min/max fold over nothing -> (inf, -inf) -> (0, 0) -> scale 1, zp 0
        *scale = 1.0f;
        *zero_point = 0;
        return TPT_OK;
    }
    Staging st(ctx);
    st.reserve(n * 4);
    st.reserve(n);
    st.reserve(4);
    st.reserve(4);
    TRY(st.commit());
    float *dx = st.take<float>(n);
    int8_t *dq = st.take<int8_t>(n);
    float *ds = st.take<float>(1);
    int32_t *dz = st.take<int32_t>(1);
    TRY(h2d(ctx, dx, x, n * 4));
    TRY(launch_quant_i8_asym(ctx, dx, n, dq, ds, dz, ctx->d_reduce));
    TRY(d2h(ctx, q, dq, n));
    TRY(d2h(ctx, scale, ds, 4));
    TRY(d2h(ctx, zero_point, dz, 4));
    return sync_and_check(ctx);
}

int tpt_cuda_pack_i4(tpt_cuda_ctx *ctx, const int8_t *values, size_t n, uint8_t *out) {
    CHECK_CTX(ctx);
    if (n == 0) return TPT_OK;
    const size_t nb = (n + 1) / 2;
    Staging st(ctx);
    st.reserve(n);
    st.reserve(nb);
    TRY(st.commit());
    int8_t *dv = st.take<int8_t>(n);
    uint8_t *dp = st.take<uint8_t>(nb);
    TRY(h2d(ctx, dv, values, n));
    TRY(launch_pack_i4(ctx, dv, n, dp, ctx->d_reduce));
    unsigned bad = 0;
    TRY(d2h(ctx, &bad, ctx->d_reduce, 4));
    TRY(sync_and_check(ctx));
    if (bad) return TPT_INVALID;  // the reference panics: "i4 out of range"
    TRY(d2h(ctx, out, dp, nb));
    return sync_and_check(ctx);
}

int tpt_cuda_unpack_i4(tpt_cuda_ctx *ctx, const uint8_t *packed, size_t packed_len, size_t n, int8_t *out,
                       size_t *written) {
    CHECK_CTX(ctx);
    const size_t count = n < 2 * packed_len ? n : 2 * packed_len;
    if (written) *written = count;
    if (count == 0) return TPT_OK;
    const size_t nb = (count + 1) / 2;
    Staging st(ctx);
    st.reserve(nb);
    st.reserve(count);
    TRY(st.commit());
    uint8_t *dp = st.take<uint8_t>(nb);
    int8_t *dv = st.take<int8_t>(count);
    TRY(h2d(ctx, dp, packed, nb));
    TRY(launch_unpack_i4(ctx, dp, count, dv));
    TRY(d2h(ctx, out, dv, count));
    return sync_and_check(ctx);
}

static int quant_i4_host(tpt_cuda_ctx *ctx, const float *x, size_t len, size_t rows, uint8_t *packed,
                         float *scales) {
    const size_t cols = len / rows, rb = (cols + 1) / 2;
    Staging st(ctx);
    st.reserve(len * 4);
    st.reserve(rows * rb);
    st.reserve(rows * 4);
    TRY(st.commit());
    float *dx = st.take<float>(len);
    uint8_t *dp = st.take<uint8_t>(rows * rb);
    float *ds = st.take<float>(rows);
    TRY(h2d(ctx, dx, x, len * 4));
    TRY(launch_quant_i4_rows(ctx, dx, rows, cols, dp, ds));
    TRY(d2h(ctx, packed, dp, rows * rb));
    TRY(d2h(ctx, scales, ds, rows * 4));
    return sync_and_check(ctx);
}

int tpt_cuda_quantize_i4_symmetric(tpt_cuda_ctx *ctx, const float *x, size_t n, uint8_t *packed, float *scale) {
    CHECK_CTX(ctx);
    if (!scale) return TPT_INVALID;
    if (n == 0) {
        *scale = 1.0f;
        return TPT_OK;
    }
    return quant_i4_host(ctx, x, n, 1, packed, scale);
}

int tpt_cuda_quantize_i4_symmetric_per_channel(tpt_cuda_ctx *ctx, const float *x, size_t len, size_t rows,
                                               uint8_t *packed, float *scales) {
    CHECK_CTX(ctx);
    if (rows == 0 || len % rows != 0) return TPT_INVALID;  // quant.rs:193 assert
    if (len == 0) {
        for (size_t r = 0; r < rows; r++) scales[r] = 1.0f;
        return TPT_OK;
    }
    return quant_i4_host(ctx, x, len, rows, packed, scales);
}

int tpt_cuda_dequantize_i8_symmetric(tpt_cuda_ctx *ctx, const int8_t *q, size_t n, float scale, float *out) {
    return tpt_cuda_dequantize_i8_symmetric_per_channel(ctx, q, n, &scale, 1, out);
}

int tpt_cuda_dequantize_i8_symmetric_per_channel(tpt_cuda_ctx *ctx, const int8_t *q, size_t n, const float *scales,
                                                 size_t n_scales, float *out) {
    CHECK_CTX(ctx);
    if (n_scales == 0 || n % n_scales != 0) return TPT_INVALID;  // dequant.rs:27-28 asserts
    if (n == 0) return TPT_OK;
    Staging st(ctx);
    st.reserve(n);
    st.reserve(n_scales * 4);
    st.reserve(n * 4);
    TRY(st.commit());
    int8_t *dq = st.take<int8_t>(n);
    float *ds = st.take<float>(n_scales);
    float *dy = st.take<float>(n);
    TRY(h2d(ctx, dq, q, n));
    TRY(h2d(ctx, ds, scales, n_scales * 4));
    TRY(launch_dequant_i8_rows(ctx, dq, n_scales, n / n_scales, ds, dy));
    TRY(d2h(ctx, out, dy, n * 4));
    return sync_and_check(ctx);
}

int tpt_cuda_dequantize_i8_asymmetric(tpt_cuda_ctx *ctx, const int8_t *q, size_t n, float scale, int32_t zero_point,
                                      float *out) {
    CHECK_CTX(ctx);
    if (n == 0) return TPT_OK;
    if (!q || !out) return TPT_INVALID;
    Staging st(ctx);
    st.reserve(n);
    st.reserve(n * 4);
    TRY(st.commit());
    int8_t *dq = st.take<int8_t>(n);
    float *dy = st.take<float>(n);
    TRY(h2d(ctx, dq, q, n));
    TRY(launch_dequant_i8_asym(ctx, dq, n, scale, zero_point, dy));
    TRY(d2h(ctx, out, dy, n * 4));
    return sync_and_check(ctx);
}

// dequantize_i4_symmetric (dequant.rs:45-50) = unpack_i4(packed, n) (quant.rs:143-157: min(n, 2 * packed_len)
// values) scaled: one row of n values with a single scale.
int tpt_cuda_dequantize_i4_symmetric(tpt_cuda_ctx *ctx, const uint8_t *packed, size_t packed_len, size_t n,
                                     float scale, float *out, size_t *written) {
    CHECK_CTX(ctx);
    const size_t cnt = n < 2 * packed_len ? n : 2 * packed_len;
    if (written) *written = cnt;
    if (cnt == 0) return TPT_OK;
    if (!packed || !out) return TPT_INVALID;
    const size_t pb = (cnt + 1) / 2;  // the bytes holding the cnt values
    Staging st(ctx);
    st.reserve(pb);
    st.reserve(4);
    st.reserve(cnt * 4);
    TRY(st.commit());
    uint8_t *dp = st.take<uint8_t>(pb);
    float *ds = st.take<float>(1);
    float *dy = st.take<float>(cnt);
    TRY(h2d(ctx, dp, packed, pb));
    TRY(h2d(ctx, ds, &scale, 4));
    TRY(launch_dequant_i4_rows(ctx, dp, 1, cnt, pb, ds, dy));
    TRY(d2h(ctx, out, dy, cnt * 4));
    return sync_and_check(ctx);
}

int tpt_cuda_dequantize_i4_symmetric_per_channel(tpt_cuda_ctx *ctx, const uint8_t *packed, size_t packed_len,
                                                 size_t row_elems, const float *scales, size_t n_scales,
                                                 float *out) {
    CHECK_CTX(ctx);
    if (n_scales == 0) return TPT_INVALID;  // dequant.rs:61 assert
    const size_t n = row_elems * n_scales;
    if (n == 0) return TPT_OK;
    Staging st(ctx);
    st.reserve(packed_len ? packed_len : 1);
    st.reserve(n_scales * 4);
    st.reserve(n * 4);
    TRY(st.commit());
    uint8_t *dp = st.take<uint8_t>(packed_len ? packed_len : 1);
    float *ds = st.take<float>(n_scales);
    float *dy = st.take<float>(n);
    TRY(h2d(ctx, dp, packed, packed_len));
    TRY(h2d(ctx, ds, scales, n_scales * 4));
    // values whose byte lies past packed_len are absent in the reference; the
    // caller's buffer keeps its contents there: copy it in first
    TRY(h2d(ctx, dy, out, n * 4));
    TRY(launch_dequant_i4_rows(ctx, dp, n_scales, row_elems, packed_len, ds, dy));
    TRY(d2h(ctx, out, dy, n * 4));
    return sync_and_check(ctx);
}

}  // extern "C"
