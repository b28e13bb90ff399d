// w8a8_ck.cu -- small-M W8A8 GEMM (4 < M <= 64) on the tcgen05 tensor cores,
// split along K over a thread-block cluster.
//
// Same arithmetic as the large-M kernel (the per-channel extension of
// quantized_matmul_i8, crates/tpt-infer-quantize/src/ptq.rs:293-324):
//   acc[m,n] = sum_k A[m,k] * Wt[n,k]  (exact i32)
//   y[m,n]   = (float)acc * (a_scale * w_scale[n]) + bias[n], then act
//
// Orientation. A decode-like GEMM is a weight stream: the MMA's M side holds
// 128 WEIGHT rows (output channels) and its N side the BN = 16/32/64
// activation rows, so each weight byte is read from HBM once and feeds
// full-height MMAs.
//
// Split. N = 4096 gives only 32 weight tiles, far fewer than 148 SMs, so each
// tile is handled by a cluster of KS CTAs (KS = 1, 2, 4 or 8), CTA r of the
// cluster taking the r-th of KS equal k ranges. Its loads are all in flight
// at once (the ring holds the whole range at the sizes this path serves).
// The KS partial accumulators meet in distributed shared memory: CTA r owns
// rows [r*128/KS, (r+1)*128/KS) of the tile, every CTA sends each row of its
// partial to the row's owner with st.async (counted on the owner's mbarrier),
// and each owner adds the KS partials of its rows and writes the output.
// Integer sums are exact, so the result does not depend on KS. Nothing goes
// through global memory between CTAs and no CTA waits on a global flag.
//
// Roles (192 threads, one CTA per SM):
//   warp 0      TMA: weight tile [128 rows x 128 B] + activation tile
//               [BN rows x 128 B] per k-block, 128B-swizzled, 8-stage ring
//   warp 1      TMEM allocation; one lane issues tcgen05.mma kind::i8
//               (M=128, N=BN, K=32) and the commits
//   warps 2..5  epilogue: thread = weight row (TMEM lane) for the exchange,
//               then (row, activation) outputs of the rows this CTA owns
// Every wait is bounded (about 1 s). A CTA that stops early still waits
// (bounded) for what the others send it, and the cluster meets once more
// before exiting, so no CTA's shared memory goes away while it is written.
#include "tc_common.cuh"

namespace tpt {

bool make_tmap_2d(CUtensorMap *tm, CUtensorMapDataType dt, const void *base, uint64_t rows, uint64_t cols,
                  uint32_t elem_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz);

namespace {
using namespace tc;

constexpr int CK_TM = 128;       // weight rows per tile (MMA M)
constexpr int CK_BK = 128;       // k bytes per stage
constexpr int CK_THREADS = 192;  // 6 warps
constexpr int CK_EPI = 128;      // epilogue threads (warps 2..5)

template <int BN>
struct CkCfg {
    static constexpr int W_BYTES = CK_TM * CK_BK;
    static constexpr int A_BYTES = BN * CK_BK;
    static constexpr int STAGE_BYTES = W_BYTES + A_BYTES;  // multiple of 1024
    // BN <= 32: small enough for two CTAs per SM, so the next launch's CTAs
    // are resident early and pull their weights into L2 during this one
    static constexpr int STAGES = BN == 16 ? 5 : BN == 32 ? 4 : 8;
    static constexpr int RECV_BYTES = CK_TM * BN * 4;      // KS partials of 128/KS rows each
    static constexpr int TMEM_COLS = BN < 32 ? 32 : BN;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + RECV_BYTES + (2 * STAGES + 3) * 8 + 1024;
    static_assert(BN == 16 || BN == 32 || BN == 64, "activation tile");
    static_assert(SMEM_BYTES <= 232448, "shared memory");
};

template <int BN>
__host__ __device__ constexpr uint32_t ck_idesc() {
    return (2u << 4)            // D format: s32
           | (1u << 7)          // A format: signed 8-bit
           | (1u << 10)         // B format: signed 8-bit
           | ((uint32_t)(BN >> 3) << 17)
           | ((uint32_t)(CK_TM >> 4) << 24);
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
__global__ void __launch_bounds__(CK_THREADS, 1)
    k_w8a8_ck(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA, int M, int N, int K,
              float a_scale, const float *__restrict__ wscale, const float *__restrict__ bias, int act,
              float *__restrict__ Y, int32_t *__restrict__ ACC, unsigned *gflags, int8_t *__restrict__ Q,
              float q_scale) {
    using Cfg = CkCfg<BN>;
    constexpr int S = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    __shared__ int abort_flag;
    __shared__ uint32_t tmem_slot;

    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t ring = (raw + 1023u) & ~1023u;
    const uint32_t recv = ring + S * Cfg::STAGE_BYTES;  // [KS][BN][128/KS] i32, 16-byte aligned
    const uint32_t bars = recv + Cfg::RECV_BYTES;
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (S + s); };
    const uint32_t tfull_bar = bars + 8u * (2 * S);
    const uint32_t recv_bar = bars + 8u * (2 * S + 1);
    const uint32_t drain_bar = bars + 8u * (2 * S + 2);
    const int32_t *recv_g = reinterpret_cast<const int32_t *>(smem_raw + (recv - raw));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint32_t ks_u;
    asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(ks_u));
    const int ks = (int)ks_u;
    const int rank = (int)cluster_rank();
    const int rows_per = CK_TM / ks;
    const int tile = blockIdx.x / ks;
    const int tiles_w = (N + CK_TM - 1) / CK_TM;
    const int xt = tile / tiles_w, wt = tile - xt * tiles_w;
    const int kblocks = (K + CK_BK - 1) / CK_BK;
    const int kb0 = rank * kblocks / ks, kb1 = (rank + 1) * kblocks / ks;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(tfull_bar, 1);
        mbar_init(recv_bar, 1);
        mbar_init(drain_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        // this CTA's weight boxes start streaming into L2 while the previous
        // kernel finishes; the ring's loads below then come from L2
        for (int kb = kb0; kb < kb1; kb++) tma_prefetch_l2_2d(&tmW, kb * CK_BK, wt * CK_TM);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"((uint32_t)Cfg::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync();  // every CTA's barriers exist before any partial is sent
    tc_fence_after();
    pdl_wait();  // the previous kernel's output (A) is complete from here on
    pdl_trigger();
    const uint32_t tmem = tmem_slot;
    volatile int *abort_p = &abort_flag;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int stage = 0;
            uint32_t phase = 0, issued_mask = 0, last_phase = 0;
            for (int kb = kb0; kb < kb1; kb++) {
                if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_p, gflags, true)) break;
                const uint32_t dst = ring + stage * Cfg::STAGE_BYTES;
                mbar_arrive_expect_tx(full_bar(stage), Cfg::STAGE_BYTES);
                tma_load_2d(dst, &tmW, full_bar(stage), kb * CK_BK, wt * CK_TM);
                tma_load_2d(dst + Cfg::W_BYTES, &tmA, full_bar(stage), kb * CK_BK, xt * BN);
                issued_mask |= 1u << stage;
                last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
                if (++stage == S) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            // our own copies in flight must land before the CTA can exit
            for (int s = 0; s < S; s++)
                if (issued_mask & (1u << s)) mbar_wait(full_bar(s), (last_phase >> s) & 1u, abort_p, gflags, false);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = ck_idesc<BN>();
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int kb = kb0; kb < kb1 && ok; kb++) {
                if (!mbar_wait(full_bar(stage), phase, abort_p, gflags, true)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t w_addr = ring + stage * Cfg::STAGE_BYTES;
                const uint32_t a_addr = w_addr + Cfg::W_BYTES;
#pragma unroll
                for (int kk = 0; kk < CK_BK / 32; kk++)
                    tc_mma_i8(tmem, sw128_desc(w_addr + 32 * kk), sw128_desc(a_addr + 32 * kk), idesc,
                              (kb != kb0 || kk != 0) ? 1u : 0u);
                tc_commit(empty_bar(stage));
                if (++stage == S) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (ok) tc_commit(tfull_bar);
            // every MMA this thread issued completes before TMEM is freed
            tc_commit(drain_bar);
            mbar_wait(drain_bar, 0, abort_p, gflags, false);
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int r = q * 32 + lane;  // weight row of the tile
        const int et = threadIdx.x - 64;
        // every partial row of every CTA of the cluster lands here
        if (et == 0) mbar_arrive_expect_tx(recv_bar, (uint32_t)Cfg::RECV_BYTES);
        bool okw = mbar_wait(tfull_bar, 0, abort_p, gflags, true);
        const bool ok = bar_and(1, CK_EPI, okw);
        if (ok) {
            tc_fence_after();
            uint32_t v[BN];
            load_acc<BN>(tmem + ((uint32_t)(q * 32) << 16), v);
            // row r goes to its owner: recv[rank][j][r % rows_per]
            const int owner = r / rows_per, lr = r - owner * rows_per;
            const uint32_t dst = map_to_rank(recv + (uint32_t)((rank * BN * rows_per + lr) * 4), (uint32_t)owner);
            const uint32_t bar = map_to_rank(recv_bar, (uint32_t)owner);
#pragma unroll
            for (int j = 0; j < BN; j++) st_async_b32(dst + (uint32_t)(j * rows_per * 4), v[j], bar);
        }
        // the rows this CTA owns, once every CTA of the cluster has sent them
        // (not cut short by an abort: the others may still be sending)
        const bool okr = bar_and(1, CK_EPI, mbar_wait(recv_bar, 0, abort_p, gflags, false) && ok);
        if (okr) {
            const int n_base = wt * CK_TM + rank * rows_per, m_base = xt * BN;
            const int per = rows_per * BN;
            for (int idx = et; idx < per; idx += CK_EPI) {
                const int j = idx / rows_per, lr = idx - j * rows_per;
                int32_t sum = 0;
                for (int p = 0; p < ks; p++) sum += recv_g[(p * BN + j) * rows_per + lr];
                const int n = n_base + lr, m = m_base + j;
                if (n >= N || m >= M) continue;
                const size_t o = (size_t)m * N + n;
                if (ACC_OUT) {
                    ACC[o] = sum;
                } else {
                    float y = __fmul_rn(__int2float_rn(sum), __fmul_rn(a_scale, __ldg(wscale + n)));
                    if (bias) y = __fadd_rn(y, __ldg(bias + n));
                    y = apply_act(y, act);
                    if (Q)
                        Q[o] = requant_i8(y, q_scale);
                    else
                        Y[o] = y;
                }
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
    cluster_sync();  // no CTA leaves while another may still address its shared memory
}

template <int BN, bool ACC_OUT>
int launch_ck(tpt_cuda_ctx *ctx, const CUtensorMap &tw, const CUtensorMap &ta, int M, int N, int K, float a_scale,
              const float *ws, const float *bias, int act, float *y, int32_t *acc, Requant rq) {
    using Cfg = CkCfg<BN>;
    static bool attr_done[64] = {};
    static int max_clusters[64][4] = {};  // per KS = 1, 2, 4, 8
    auto kfn = k_w8a8_ck<BN, ACC_OUT>;
    const int dev = ctx->device & 63;
    if (!attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "w8a8_ck smem attribute");
        for (int i = 0; i < 4; i++) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)(1 << i) * 16, 1, 1);
            cfg.blockDim = dim3(CK_THREADS, 1, 1);
            cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = 1u << i;
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = 1;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess) {
                cudaGetLastError();
                n = 0;
            }
            max_clusters[dev][i] = n;
        }
        attr_done[dev] = true;
    }
    const int tiles = ((N + CK_TM - 1) / CK_TM) * ((M + BN - 1) / BN);
    const int kblocks = (K + CK_BK - 1) / CK_BK;
    // the widest split whose CTAs all fit on the GPU at once, with at least
    // two k-blocks per CTA
    int li = 0;
    for (int i = 3; i >= 1; i--) {
        const int ks = 1 << i;
        if (2 * ks <= kblocks && (long long)tiles * ks <= ctx->sm_count && max_clusters[dev][i] >= tiles) {
            li = i;
            break;
        }
    }
    const int ks = 1 << li;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(tiles * ks), 1, 1);
    cfg.blockDim = dim3(CK_THREADS, 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = (unsigned)ks;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see pdl_wait
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, tw, ta, M, N, K, a_scale, ws, bias, act, y, acc, ctx->d_flags, rq.q,
                                       rq.scale);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "w8a8_ck launch");
    return after_launch(ctx, "w8a8_ck");
}

}  // namespace

// 4 < M <= 64 with the weight's tensor maps available and A 16-byte aligned;
// returns handled = false otherwise (the caller falls back to the GEMV).
int launch_w8a8_ck(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, const tpt_cuda_weights *w, float a_scale,
                   const float *bias, int act, float *y, int32_t *acc, bool *handled, Requant rq) {
    *handled = false;
    if (!w->tmap_ok || m == 0 || m > 64 || w->k == 0 || w->n > 0x7fffffff || w->k > 0x7fffffff) return TPT_OK;
    const int BN = m <= 16 ? 16 : m <= 32 ? 32 : 64;
    CUtensorMap ta;
    if (!make_tmap_2d(&ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, a, m, w->k, 1, CK_BK, (uint32_t)BN,
                      CU_TENSOR_MAP_SWIZZLE_128B))
        return TPT_OK;
    *handled = true;
    const CUtensorMap &tw = *reinterpret_cast<const CUtensorMap *>(w->tmaps[0]);  // 128-row box
    const int M = (int)m, N = (int)w->n, K = (int)w->k;
#define TPT_CK(BNV)                                                                                         \
    return acc ? launch_ck<BNV, true>(ctx, tw, ta, M, N, K, a_scale, w->scales, bias, act, y, acc, rq)      \
               : launch_ck<BNV, false>(ctx, tw, ta, M, N, K, a_scale, w->scales, bias, act, y, acc, rq)
    if (BN == 16) TPT_CK(16);
    if (BN == 32) TPT_CK(32);
    TPT_CK(64);
#undef TPT_CK
}

}  // namespace tpt
