// w8a8_mma.cu -- W8A8 GEMM for small batches (3 <= M <= 32): the int8 weight
// rows stream through the TMA ring of ring.cuh and meet the int8 activations
// in register-fragment MMAs.
//
// Reference semantics: quantized_matmul_i8 (crates/tpt-infer-quantize/src/
// ptq.rs:293-324) with the per-output-channel scale and bias epilogue:
// acc = sum_k a[m,k] w[n,k] in i32, y = (float)acc * (a_scale * w_scale[n])
// + bias[n], then act (and, with a requantizing output, q = clamp(roundf(y / s))).
// The integer sums are exact, so the result is bit-identical to the reference.
//
// Layout. A CTA takes a contiguous run of 16-row weight groups (one 3-D TMA
// load of 16 rows x K bytes each, 128B-swizzled). Consumer warp w owns k slice
// [32 CH w, 32 CH (w + 1)) of every row and holds the activation fragments of
// that slice in registers for the whole kernel (activation rows on the MMA's N
// side, MT tiles of 8); per stage it runs CH k-steps of mma.sync m16n8k32
// s8 x s8 -> s32 (A = the 16 weight rows straight from the ring, no decode),
// and stores its i32 slice sums; the flush adds the slices (exact) and applies
// the epilogue. tcgen05 is not used here: at N = 8-32 its per-instruction
// cost, not the arithmetic, would bound this HBM-speed stream. Only weights
// with a tensor map (host uploads) take this path, so the first stages are
// requested before the dependency wait.
#include "ring.cuh"

namespace tpt {

namespace {
using namespace tc;
using namespace ring;

constexpr int WM_MAX_KW = 16;  // consumer warps
constexpr int WM_THREADS = 32 * (WM_MAX_KW + 1);
constexpr int WM_PART_BUDGET = 48 * 1024;
constexpr int WM_SMEM_MAX = 200 * 1024;

__device__ __forceinline__ void mma_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// MT activation tiles of 8 rows (M <= 8 MT); CH k-steps of 32 per consumer warp.
template <int MT, int CH>
__global__ void __launch_bounds__(WM_THREADS, 1)
    k_w8a8_mma(const __grid_constant__ CUtensorMap tmW, const int8_t *__restrict__ A, int M, int N, int K,
               float a_scale, const float *__restrict__ wscale, const float *__restrict__ bias, int act,
               float *__restrict__ Y, int32_t *__restrict__ ACC, int8_t *__restrict__ Q, float q_scale, int S, int P,
               unsigned *gflags) {
    constexpr int SL = 32 * CH, MP = 8 * MT;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int abort_flag;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int KW = (K + SL - 1) / SL;  // consumer warps; warp KW is the producer
    const uint32_t stage_bytes = (uint32_t)K * WG_ROWS;
    const int groups = (N + WG_ROWS - 1) / WG_ROWS;
    const int g0 = (int)((long long)blockIdx.x * groups / gridDim.x);
    const int g1 = (int)((long long)(blockIdx.x + 1) * groups / gridDim.x);
    const uint32_t raw = smem_u32(smem), ring = (raw + 1023u) & ~1023u;  // 128B swizzle: 1 KB aligned
    int32_t *part = reinterpret_cast<int32_t *>(smem + (ring - raw) + (size_t)S * stage_bytes);  // [P][MP][KW][16]
    const uint32_t bars = smem_u32(part + P * MP * KW * WG_ROWS);
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (S + s); };

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), (uint32_t)KW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    }
    __syncthreads();
    volatile int *abort_p = &abort_flag;
    if (warp == KW) {
        if (lane == 0) produce(tmW, ring, stage_bytes, bars, S, g0, g1, abort_p, gflags);
        return;
    }
    if (warp > KW) return;
    pdl_wait();  // A (the previous kernel's output) is complete from here on
    pdl_trigger();

    const int ncons = KW * 32;
    const int gq = lane >> 2, tq = lane & 3;
    const int kslice = warp * SL;
    const int ksteps = min(SL, K - kslice) / 32;
    // The MMA's k positions 4 tq..4 tq+3 and 16+4 tq..16+4 tq+3 of k-step j are
    // given the 8 consecutive k [32 j + 8 tq, +8) of the slice, identically in
    // both operands (the sum over k is unchanged), so each fragment pair is one
    // 8-byte load. Fragment row g is weight row pr = 2 (g & 3) + (g >> 2) (and
    // pr + 8): the 4 rows of a half-warp then differ in swizzle bits 1-2 and
    // its 8-byte loads hit 16 distinct banks pairs.
    const int pr = ((gq & 3) << 1) | (gq >> 2);
    // activation fragments: tile tt, column gq = activation row 8 tt + gq
    uint32_t bf[MT][CH][2];
#pragma unroll
    for (int tt = 0; tt < MT; tt++) {
        const int m = 8 * tt + gq;
        const int8_t *arow = A + (size_t)m * K + kslice + 8 * tq;
#pragma unroll
        for (int j = 0; j < CH; j++) {
            const uint2 v = (m < M && j < ksteps) ? __ldg(reinterpret_cast<const uint2 *>(arow + 32 * j))
                                                  : make_uint2(0u, 0u);
            bf[tt][j][0] = v.x;
            bf[tt][j][1] = v.y;
        }
    }

    // When one flush covers the CTA's run and every output has a thread, each
    // thread's channel scale and bias are loaded now, off the flush's path.
    const bool one_flush = P >= g1 - g0 && (g1 - g0) * WG_ROWS * M <= ncons;
    float my_sc = 0.0f, my_bi = 0.0f;
    if (one_flush && !ACC) {
        const int idx = (int)threadIdx.x, n = (g0 + idx / (WG_ROWS * M)) * WG_ROWS + idx % WG_ROWS;
        if (idx < (g1 - g0) * WG_ROWS * M && n < N) {
            my_sc = __ldg(wscale + n);
            if (bias) my_bi = __ldg(bias + n);
        }
    }

    int s = 0, gl = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int g = g0; g < g1; g++) {
        if (ok) ok = mbar_wait(full_bar(s), ph, abort_p, gflags, true);
        int d[MT][4] = {};
        const uint32_t base = ring + (uint32_t)s * stage_bytes;
        // plain loads (ordered after the barrier wait by its memory clobber)
        const uint2 *stg2 = reinterpret_cast<const uint2 *>(smem + (base - raw));
        if (ok) {
#pragma unroll
            for (int j = 0; j < CH; j++) {
                if (j < ksteps) {
                    const uint32_t o = stage_off(pr, (uint32_t)kslice + 32u * j + 8u * tq) >> 3;
                    const uint2 r0 = stg2[o], r1 = stg2[o + 128u];  // weight rows pr, pr + 8
                    const uint32_t a[4] = {r0.x, r1.x, r0.y, r1.y};
#pragma unroll
                    for (int tt = 0; tt < MT; tt++) mma_s8(d[tt], a, bf[tt][j][0], bf[tt][j][1]);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(empty_bar(s));
        // d[tt]: weight rows pr (0, 1) and pr + 8 (2, 3), activation rows 8 tt + 2 tq (+1)
#pragma unroll
        for (int tt = 0; tt < MT; tt++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int m = 8 * tt + 2 * tq + (e & 1), r = pr + 8 * (e >> 1);
                part[((gl * MP + m) * KW + warp) * WG_ROWS + r] = d[tt][e];
            }
        if (++s == S) {
            s = 0;
            ph ^= 1u;
        }
        if (++gl == P || g + 1 == g1) {  // flush: add the slices, apply the epilogue
            ok = bar_and(1, ncons, ok);
            if (ok) {
                const int gb = g + 1 - gl;
                for (int idx = (int)threadIdx.x; idx < gl * WG_ROWS * M; idx += ncons) {
                    const int r = idx % WG_ROWS, m = (idx / WG_ROWS) % M, gi = idx / (WG_ROWS * M);
                    const int n = (gb + gi) * WG_ROWS + r;
                    if (n >= N) continue;
                    int acc = 0;
                    for (int sl = 0; sl < KW; sl++) acc += part[((gi * MP + m) * KW + sl) * WG_ROWS + r];
                    const size_t o = (size_t)m * N + n;
                    if (ACC) {
                        ACC[o] = acc;
                    } else {
                        const float sc = one_flush ? my_sc : __ldg(wscale + n);
                        float y = __fmul_rn(__int2float_rn(acc), __fmul_rn(a_scale, sc));
                        if (bias) y = __fadd_rn(y, one_flush ? my_bi : __ldg(bias + n));
                        y = apply_act(y, act);
                        if (Q)
                            Q[o] = requant_i8(y, q_scale);
                        else
                            Y[o] = y;
                    }
                }
            }
            bar_sync(1, ncons);  // part is free again
            gl = 0;
        }
    }
}

template <int MT, int CH>
int launch_mt(tpt_cuda_ctx *ctx, const CUtensorMap &tw, const int8_t *a, int m, int n, int k, float a_scale,
              const float *ws, const float *bias, int act, float *y, int32_t *acc, Requant rq, int S, int P,
              size_t smem) {
    static bool attr_done[64] = {};
    auto kfn = k_w8a8_mma<MT, CH>;
    const int dev = ctx->device & 63;
    if (!attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, WM_SMEM_MAX + 1024);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "w8a8_mma smem attribute");
        attr_done[dev] = true;
    }
    const int kw = (k + 32 * CH - 1) / (32 * CH), groups = (n + WG_ROWS - 1) / WG_ROWS;
    const unsigned grid = (unsigned)(groups < ctx->sm_count ? groups : ctx->sm_count);  // one CTA per SM
    launch_pdl(kfn, grid, 32 * (kw + 1), smem, ctx->stream, tw, a, m, n, k, a_scale, ws, bias, act, y, acc, rq.q,
               rq.scale, S, P, ctx->d_flags);
    return after_launch(ctx, "w8a8_mma");
}

}  // namespace

// 3 <= M <= 32, K % 128 == 0, K <= 4096, uploaded weights (with a tensor map),
// A 16-byte aligned; returns handled = false otherwise.
int launch_w8a8_mma(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, const tpt_cuda_weights *w, float a_scale,
                    const float *bias, int act, float *y, int32_t *acc, bool *handled, Requant rq) {
    *handled = false;
    const size_t n = w->n, k = w->k;
    if (!w->tmap_ok || m < 3 || m > 32 || k % 128 != 0 || k > (size_t)WM_MAX_KW * 256 || n > INT32_MAX) return TPT_OK;
    if (((uintptr_t)a & 15) != 0) return TPT_OK;
    CUtensorMap tw;
    if (!make_tmap_rows3d(&tw, w->data, n, k)) return TPT_OK;
    const int kw = (int)((k + 255) / 256);
    const int MT = m <= 8 ? 1 : m <= 16 ? 2 : 4;
    const size_t stage = WG_ROWS * k;
    const size_t per_group = (size_t)8 * MT * kw * WG_ROWS * 4;
    const size_t groups = (n + WG_ROWS - 1) / WG_ROWS;
    const size_t ctas = groups < (size_t)ctx->sm_count ? groups : (size_t)ctx->sm_count;
    const size_t run = (groups + ctas - 1) / ctas;
    const size_t pmax = WM_PART_BUDGET / per_group;
    const int P = (int)(run < pmax ? run : pmax);
    if (P < 1) return TPT_OK;
    const size_t budget = WM_SMEM_MAX - (size_t)P * per_group - 1024 - 128;
    const int S = (int)(budget / stage < 4 ? budget / stage : 4);
    if (S < 2) return TPT_OK;
    const size_t smem = 1024 + (size_t)S * stage + (size_t)P * per_group + (size_t)2 * S * 8;
    *handled = true;
    const int M = (int)m, N = (int)n, K = (int)k;
    if (MT == 1) return launch_mt<1, 8>(ctx, tw, a, M, N, K, a_scale, w->scales, bias, act, y, acc, rq, S, P, smem);
    if (MT == 2) return launch_mt<2, 8>(ctx, tw, a, M, N, K, a_scale, w->scales, bias, act, y, acc, rq, S, P, smem);
    return launch_mt<4, 8>(ctx, tw, a, M, N, K, a_scale, w->scales, bias, act, y, acc, rq, S, P, smem);
}

}  // namespace tpt
