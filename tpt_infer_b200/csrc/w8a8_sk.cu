// w8a8_sk.cu -- small-M W8A8 GEMM (M <= 64) on the tcgen05 tensor cores,
// stream-K over the weight bytes.
//
// Same arithmetic as the large-M kernels (the per-channel extension of
// quantized_matmul_i8, crates/tpt-infer-quantize/src/ptq.rs:293-324):
//   acc[m,n] = sum_k A[m,k] * Wt[n,k]  (exact i32)
//   y[m,n]   = (float)acc * (a_scale * w_scale[n]) + bias[n], then act
//
// Orientation. A decode-like GEMM is a weight stream: M activation rows are
// tiny next to the N x K weight bytes. The MMA's M side therefore holds 128
// WEIGHT rows (output channels) and its N side the BN = 16/32/64 activation
// rows, so each weight byte is read from HBM once and feeds full-height MMAs.
//
// Stream-K. N = 4096 gives only 32 weight tiles, far fewer than 148 SMs, so the
// (tile, 128-byte k-block) units are split into one equal contiguous range per
// CTA. A CTA whose range covers a whole tile writes the output directly.
// Otherwise it stores its partial i32 tile into its own slot of the tile in an
// L2-resident workspace (plain coalesced stores: the contributors of a tile
// are consecutive CTAs, slot = CTA - first contributor) and counts itself in
// the tile's counter; the CTA that completes the count adds the slots in slot
// order, applies the epilogue and resets the counter. Integer sums are exact,
// so the output is bit-identical for any split. Nothing waits on another CTA.
//
// Roles (192 threads, one CTA per SM):
//   warp 0      TMA: weight tile [128 rows x 128 B] + activation tile
//               [BN rows x 128 B] per k-block, 128B-swizzled, 8-stage ring
//   warp 1      TMEM allocation; one lane issues tcgen05.mma kind::i8
//               (M=128, N=BN, K=32) and the commits
//   warps 2..5  epilogue, thread = weight row (TMEM lane), double-buffered
//               accumulators so segment i's epilogue overlaps segment i+1
// All waits are bounded (1 s); a timeout raises the CTA's abort, records the
// device timeout flag and the context clears the tile counters before next use.
#include "tc_common.cuh"

namespace tpt {

bool make_tmap_2d(CUtensorMap *tm, CUtensorMapDataType dt, const void *base, uint64_t rows, uint64_t cols,
                  uint32_t elem_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz);

namespace {
using namespace tc;

constexpr int SK_TM = 128;       // weight rows per tile (MMA M)
constexpr int SK_BK = 128;       // k bytes per stage
constexpr int SK_THREADS = 192;  // 6 warps
constexpr int SK_EPI = 128;      // epilogue threads (warps 2..5)

template <int BN>
struct SkCfg {
    static constexpr int W_BYTES = SK_TM * SK_BK;
    static constexpr int A_BYTES = BN * SK_BK;
    static constexpr int STAGE_BYTES = W_BYTES + A_BYTES;  // multiple of 1024
    static constexpr int STAGES = 8;
    static constexpr int ACC_COLS = BN < 32 ? 32 : BN;     // column stride of the two accumulators
    static constexpr int TMEM_COLS = 2 * ACC_COLS;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + (2 * STAGES + 5) * 8 + 1024;
    static_assert(BN == 16 || BN == 32 || BN == 64, "activation tile");
    static_assert(SMEM_BYTES <= 232448, "shared memory");
};

template <int BN>
__host__ __device__ constexpr uint32_t sk_idesc() {
    return (2u << 4)            // D format: s32
           | (1u << 7)          // A format: signed 8-bit
           | (1u << 10)         // B format: signed 8-bit
           | ((uint32_t)(BN >> 3) << 17)
           | ((uint32_t)(SK_TM >> 4) << 24);
}

// BN accumulator columns of this thread's TMEM lane -> v[0..BN)
template <int BN>
__device__ __forceinline__ void load_acc(uint32_t taddr, uint32_t (&v)[BN]) {
    if constexpr (BN == 16) {
        tmem_ld16(taddr, v);
    } else {
#pragma unroll
        for (int c = 0; c < BN / 32; c++) tmem_ld32(taddr + 32u * c, *reinterpret_cast<uint32_t(*)[32]>(v + 32 * c));
    }
    tmem_wait_ld();
}

template <int BN, bool ACC_OUT>
__global__ void __launch_bounds__(SK_THREADS, 1)
    k_w8a8_sk(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA, int M, int N, int K,
              float a_scale, const float *__restrict__ wscale, const float *__restrict__ bias, int act,
              float *__restrict__ Y, int32_t *__restrict__ ACC, int32_t *__restrict__ part,
              int *__restrict__ cnt, unsigned *gflags, int8_t *__restrict__ Q, float q_scale) {
    using Cfg = SkCfg<BN>;
    constexpr int S = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    __shared__ int abort_flag;
    __shared__ int last_flag;
    __shared__ int fin_slot[TPT_SK_MAX_CTAS];  // the finishing CTA's table of contributor slots
    __shared__ uint32_t tmem_slot;

    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t ring = (raw + 1023u) & ~1023u;
    const uint32_t bars = ring + S * Cfg::STAGE_BYTES;
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (S + s); };
    auto tfull_bar = [&](int b) { return bars + 8u * (2 * S + b); };
    auto tempty_bar = [&](int b) { return bars + 8u * (2 * S + 2 + b); };
    const uint32_t drain_bar = bars + 8u * (2 * S + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_w = (N + SK_TM - 1) / SK_TM, tiles_x = (M + BN - 1) / BN;
    const int kblocks = (K + SK_BK - 1) / SK_BK;
    const long long units = (long long)tiles_w * tiles_x * kblocks;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), SK_EPI);
        }
        mbar_init(drain_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"((uint32_t)Cfg::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    volatile int *abort_p = &abort_flag;
    SkRange range(units, kblocks, blockIdx.x, gridDim.x);
    int tile, kb0, kb1;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int stage = 0;
            uint32_t phase = 0, issued_mask = 0, last_phase = 0;
            bool ok = true;
            while (ok && range.next(tile, kb0, kb1)) {
                const int xt = tile / tiles_w, wt = tile - xt * tiles_w;
                for (int kb = kb0; kb < kb1; kb++) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_p, gflags, true)) {
                        ok = false;
                        break;
                    }
                    const uint32_t dst = ring + stage * Cfg::STAGE_BYTES;
                    mbar_arrive_expect_tx(full_bar(stage), Cfg::STAGE_BYTES);
                    tma_load_2d(dst, &tmW, full_bar(stage), kb * SK_BK, wt * SK_TM);
                    tma_load_2d(dst + Cfg::W_BYTES, &tmA, full_bar(stage), kb * SK_BK, xt * BN);
                    issued_mask |= 1u << stage;
                    last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // our own copies in flight must land before the CTA can exit
            for (int s = 0; s < S; s++)
                if (issued_mask & (1u << s)) mbar_wait(full_bar(s), (last_phase >> s) & 1u, abort_p, gflags, false);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = sk_idesc<BN>();
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = true;
            while (ok && range.next(tile, kb0, kb1)) {
                if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_p, gflags, true)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)(acc * Cfg::ACC_COLS);
                for (int kb = kb0; kb < kb1; kb++) {
                    if (!mbar_wait(full_bar(stage), phase, abort_p, gflags, true)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t w_addr = ring + stage * Cfg::STAGE_BYTES;
                    const uint32_t a_addr = w_addr + Cfg::W_BYTES;
#pragma unroll
                    for (int kk = 0; kk < SK_BK / 32; kk++)
                        tc_mma_i8(d_tmem, sw128_desc(w_addr + 32 * kk), sw128_desc(a_addr + 32 * kk), idesc,
                                  (kb != kb0 || kk != 0) ? 1u : 0u);
                    tc_commit(empty_bar(stage));
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(tfull_bar(acc));
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            // every MMA this thread issued completes before TMEM is freed
            tc_commit(drain_bar);
            mbar_wait(drain_bar, 0, abort_p, gflags, false);
        }
    } else {
        // ---------------- epilogue (warps 2..5): thread = weight row ----------------
        // Every epilogue thread walks the same segments and reaches the same
        // named barriers; an abort is agreed on with bar.red.and so no thread
        // can leave the others waiting.
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int r = q * 32 + lane;
        const int epi_tid = threadIdx.x - 64;
        int acc = 0;
        uint32_t acc_phase = 0;
        while (range.next(tile, kb0, kb1)) {
            const int xt = tile / tiles_w, wt = tile - xt * tiles_w;
            bool okw = mbar_wait(tfull_bar(acc), acc_phase, abort_p, gflags, true);
            if (!bar_and(1, SK_EPI, okw)) break;
            tc_fence_after();
            uint32_t v[BN];
            load_acc<BN>(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * Cfg::ACC_COLS), v);
            tc_fence_before();
            mbar_arrive(tempty_bar(acc));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }

            const int n = wt * SK_TM + r;
            const bool nv = n < N;
            const int m0 = xt * BN;
            float sc = 0.0f, bi = 0.0f;
            if (!ACC_OUT && nv) {
                sc = __fmul_rn(a_scale, __ldg(wscale + n));
                if (bias) bi = __ldg(bias + n);
            }
            auto emit = [&](int j, int32_t a) {
                const size_t o = (size_t)(m0 + j) * N + n;
                if (ACC_OUT) {
                    ACC[o] = a;
                } else {
                    float y = __fmul_rn(__int2float_rn(a), sc);
                    if (bias) y = __fadd_rn(y, bi);
                    y = apply_act(y, act);
                    if (Q)
                        Q[o] = requant_i8(y, q_scale);
                    else
                        Y[o] = y;
                }
            };
            if (kb0 == 0 && kb1 == kblocks) {
                // the whole k range: straight to the output
#pragma unroll
                for (int j = 0; j < BN; j++)
                    if (nv && m0 + j < M) emit(j, (int32_t)v[j]);
                continue;
            }
            // partial tile: this CTA's slot of [tile][slot][BN][128]
            const long long ub = (long long)tile * kblocks;
            const int c_first = sk_cta_of_unit(ub, units, gridDim.x);
            const int nslots = sk_cta_of_unit(ub + kblocks - 1, units, gridDim.x) - c_first + 1;
            constexpr size_t SLOT = (size_t)BN * SK_TM;
            int32_t *mine = part + (size_t)sk_slot(blockIdx.x, tile, units, kblocks, gridDim.x) * SLOT + r;
#pragma unroll
            for (int j = 0; j < BN; j++)
                if (nv && m0 + j < M) mine[(size_t)j * SK_TM] = (int32_t)v[j];
            __threadfence();
            bar_sync(1, SK_EPI);
            if (epi_tid == 0) last_flag = (atomicAdd(cnt + c_first, 1) + 1 == nslots) ? 1 : 0;
            bar_sync(1, SK_EPI);
            if (last_flag) {
                __threadfence();
                for (int i = epi_tid; i < nslots; i += SK_EPI)
                    fin_slot[i] = sk_slot(c_first + i, tile, units, kblocks, gridDim.x);
                bar_sync(1, SK_EPI);
                // every load of a group of (8 slots x JG columns) is in flight
                // at once; the sum still runs in slot order
                constexpr int JG = BN < 16 ? BN : 16, SG = 8;
#pragma unroll 1
                for (int j0 = 0; j0 < BN; j0 += JG) {
                    int32_t a[JG];
#pragma unroll
                    for (int jj = 0; jj < JG; jj++) a[jj] = 0;
#pragma unroll 1
                    for (int s0 = 0; s0 < nslots; s0 += SG) {
                        int32_t b[SG][JG];
#pragma unroll
                        for (int sl = 0; sl < SG; sl++)
#pragma unroll
                            for (int jj = 0; jj < JG; jj++)
                                b[sl][jj] = (s0 + sl < nslots && nv && m0 + j0 + jj < M)
                                                ? __ldcg(part + (size_t)fin_slot[s0 + sl] * SLOT + r + (size_t)(j0 + jj) * SK_TM)
                                                : 0;
#pragma unroll
                        for (int sl = 0; sl < SG; sl++)
#pragma unroll
                            for (int jj = 0; jj < JG; jj++) a[jj] += b[sl][jj];
                    }
#pragma unroll
                    for (int jj = 0; jj < JG; jj++)
                        if (nv && m0 + j0 + jj < M) emit(j0 + jj, a[jj]);
                }
                if (epi_tid == 0) cnt[c_first] = 0;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"((uint32_t)Cfg::TMEM_COLS)
                     : "memory");
    }
}

template <int BN, bool ACC_OUT>
int launch_sk(tpt_cuda_ctx *ctx, const CUtensorMap &tw, const CUtensorMap &ta, int M, int N, int K, float a_scale,
              const float *ws, const float *bias, int act, float *y, int32_t *acc, Requant rq) {
    using Cfg = SkCfg<BN>;
    static bool attr_done[64] = {};
    auto kfn = k_w8a8_sk<BN, ACC_OUT>;
    const int dev = ctx->device & 63;
    if (!attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "w8a8_sk smem attribute");
        attr_done[dev] = true;
    }
    const int tiles = ((N + SK_TM - 1) / SK_TM) * ((M + BN - 1) / BN);
    const long long units = (long long)tiles * ((K + SK_BK - 1) / SK_BK);
    const int ctas = ctx->sm_count < tc::TPT_SK_MAX_CTAS ? ctx->sm_count : tc::TPT_SK_MAX_CTAS;
    // fewer than two units per SM: whole tiles per CTA, no cross-CTA reduction
    const int grid = units < 2LL * ctas ? (tiles < ctas ? tiles : ctas) : ctas;
    int st = ensure_sk(ctx, (size_t)2 * grid * BN * SK_TM * sizeof(int32_t));
    if (st) return st;
    int *cnt = reinterpret_cast<int *>(ctx->sk);
    int32_t *part = reinterpret_cast<int32_t *>(ctx->sk + TPT_SK_SLOTS_OFFSET);
    kfn<<<grid, SK_THREADS, Cfg::SMEM_BYTES, ctx->stream>>>(tw, ta, M, N, K, a_scale, ws, bias, act, y, acc, part, cnt,
                                                            ctx->d_flags, rq.q, rq.scale);
    return after_launch(ctx, "w8a8_sk");
}

}  // namespace

// M <= 64 with the weight's tensor maps available and A 16-byte aligned;
// returns handled = false otherwise (the caller falls back to the GEMV).
int launch_w8a8_sk(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, const tpt_cuda_weights *w, float a_scale,
                   const float *bias, int act, float *y, int32_t *acc, bool *handled, Requant rq) {
    *handled = false;
    if (!w->tmap_ok || m == 0 || m > 64 || w->k == 0) return TPT_OK;
    const int BN = m <= 16 ? 16 : m <= 32 ? 32 : 64;
    CUtensorMap ta;
    if (!make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, m, w->k, 1, SK_BK, (uint32_t)BN,
                      CU_TENSOR_MAP_SWIZZLE_128B))
        return TPT_OK;
    *handled = true;
    const CUtensorMap &tw = *reinterpret_cast<const CUtensorMap *>(w->tmaps[0]);  // 128-row box
    const int M = (int)m, N = (int)w->n, K = (int)w->k;
#define TPT_SK(BNV)                                                                                         \
    return acc ? launch_sk<BNV, true>(ctx, tw, ta, M, N, K, a_scale, w->scales, bias, act, y, acc, rq)      \
               : launch_sk<BNV, false>(ctx, tw, ta, M, N, K, a_scale, w->scales, bias, act, y, acc, rq)
    if (BN == 16) TPT_SK(16);
    if (BN == 32) TPT_SK(32);
    TPT_SK(64);
#undef TPT_SK
}

}  // namespace tpt
