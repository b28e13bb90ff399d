// w8a8_tc.cu -- the W8A8 GEMM for M > 64 on Blackwell's 5th-generation tensor
// cores (tcgen05.mma kind::i8, i32 accumulators in tensor memory), one output
// tile per pair of SMs (cta_group::2).
//
// Computes the per-channel extension of quantized_matmul_i8
// (crates/tpt-infer-quantize/src/ptq.rs:293-324):
//   acc[m,n] = sum_k A[m,k] * Wt[n,k]           (int8 x int8 -> i32, exact)
//   y[m,n]   = (float)acc * (a_scale * w_scale[n]) + bias[n], then act
// The epilogue rounds exactly like the oracle (separate RN multiply/add), so
// the f32 output is bit-exact.
//
// Every mbarrier wait is bounded (TPT_WAIT_CYCLES of the SM clock, about 1 s).
// A wait that runs out records TPT_FLAG_TIMEOUT in the context's device flag
// words, raises a CTA-wide abort so every role leaves its loop, the producer
// waits (bounded) for its own TMA copies still in flight, the MMA issuer waits
// (bounded) for its MMAs, tensor memory is freed and the kernel returns.
// No multicast loads are used anywhere.
#include "tc_common.cuh"

namespace tpt {

// cuTensorMapEncodeTiled through the runtime's driver entry point (null when
// the driver does not provide it)
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

namespace {
using namespace tc;

constexpr int TC_BK = 128;       // k bytes per stage (one 128B swizzle row)

// ---------------------------------------------------------------------------
// SM-pair kernel: tcgen05.mma.cta_group::2, 256 x 256 output tiles per
// cluster of two CTAs on two SMs. Each CTA loads its 128 rows of A and its 128
// rows of B (its half of the tile's N) per k-block; the leader CTA (cluster
// rank 0) issues the M=256 MMA, which reads both CTAs' shared memory, and
// each CTA's tensor memory receives its own 128 x 256 accumulator. Per SM the
// operand traffic is 8 KB per MMA instruction instead of 12 KB for the
// one-SM 128 x 256 form, which is what lets the tensor pipe run at its rate.
//   full[s]   (leader)  : completed by both CTAs' TMA bytes (2-SM loads)
//   empty[s]  (each)    : leader's MMA commit, multicast to both CTAs
//   tfull[b]  (each)    : leader's MMA commit, multicast to both CTAs
//   tempty[b] (leader)  : one arrival per epilogue warp of both CTAs
// 8 epilogue warps per CTA: two per TMEM lane quarter, each taking half of
// the 256 accumulator columns.
// ---------------------------------------------------------------------------
constexpr int P_BM = 256;                 // tile M (MMA M over the pair)
constexpr int P_EPI_WARPS = 8;
constexpr int P_THREADS = (2 + P_EPI_WARPS) * 32;
constexpr int P_A_BYTES = 128 * TC_BK;    // this CTA's 128 rows of A
constexpr int P_OUT_BYTES = P_EPI_WARPS * 2 * 4096;

// Tile N (the MMA's N) is a template parameter: 64, 128, 192 or 256. Each CTA holds
// BN/2 rows of B per stage; the ring is sized to ~160 KB.
template <int BN>
struct PairCfg {
    static constexpr int B_BYTES = (BN / 2) * TC_BK;
    static constexpr int STAGE_BYTES = P_A_BYTES + B_BYTES;
    static constexpr int STAGES_RAW = 163840 / STAGE_BYTES;
    static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
    // two accumulators of BN columns, rounded up to a power of two (the allocation unit)
    static constexpr int TMEM_COLS = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + P_OUT_BYTES + (2 * STAGES + 5) * 8 + 16 + 1024;
    static_assert(SMEM_BYTES <= 232448, "dynamic shared memory per CTA");
    static_assert(BN == 64 || BN == 128 || BN == 192 || BN == 256, "tile N");
};

// 2-SM TMA load: data into this CTA's shared memory, transaction bytes
// counted on the barrier at `bar_cluster` (the leader's).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *tm, uint32_t bar_cluster, int x,
                                                 int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar_cluster), "r"(x), "r"(y)
        : "memory");
}
__device__ __forceinline__ void tc2_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// commit the leader's MMAs to the barrier at `bar` in both CTAs of the pair
__device__ __forceinline__ void tc2_commit_both(uint32_t bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"((uint16_t)3)
        : "memory");
}

// ACT: the activation, a compile-time choice so that each instantiation's
// epilogue holds only its own code
template <int BN, bool ACC_OUT, int ACT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(P_THREADS, 1)
    k_w8a8_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmY, int tma_store, int M, int N, int K, float a_scale,
               const float *__restrict__ wscale, const float *__restrict__ bias, float *__restrict__ Y,
               int32_t *__restrict__ ACC, unsigned *gflags, int8_t *__restrict__ Q, float q_scale) {
    using Cfg = PairCfg<BN>;
    constexpr int S = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    __shared__ int abort_flag;
    __shared__ uint32_t tmem_slot;

    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t ring = (raw + 1023u) & ~1023u;
    const uint32_t staging = ring + S * Cfg::STAGE_BYTES;
    const uint32_t bars = staging + P_OUT_BYTES;
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (S + s); };
    auto tfull_bar = [&](int b) { return bars + 8u * (2 * S + b); };
    auto tempty_bar = [&](int b) { return bars + 8u * (2 * S + 2 + b); };
    const uint32_t drain_bar = bars + 8u * (2 * S + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
    const int tiles_m = (M + P_BM - 1) / P_BM, tiles_n = (N + BN - 1) / BN;
    const int ntiles = tiles_m * tiles_n;
    const int kblocks = (K + TC_BK - 1) / TC_BK;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), 2 * P_EPI_WARPS);
        }
        mbar_init(drain_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"((uint32_t)Cfg::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
    tc_fence_after();
    pdl_wait();  // the previous kernel's output (A) is complete from here on
    pdl_trigger();
    const uint32_t tmem = tmem_slot;
    volatile int *abort_p = &abort_flag;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs) ----------------
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = cluster; t < ntiles && ok; t += nclusters) {
                const int mt = t / tiles_n, nt = t - mt * tiles_n;
                const int arow = mt * P_BM + (int)rank * 128, brow = nt * BN + (int)rank * (BN / 2);
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_p, gflags, true)) {
                        ok = false;
                        break;
                    }
                    const uint32_t a_dst = ring + stage * Cfg::STAGE_BYTES;
                    const uint32_t fb = map_to_rank(full_bar(stage), 0);
                    if (leader) mbar_arrive_expect_tx(full_bar(stage), 2 * Cfg::STAGE_BYTES);
                    tma_load_2d_pair(a_dst, &tmA, fb, kb * TC_BK, arow);
                    tma_load_2d_pair(a_dst + P_A_BYTES, &tmB, fb, kb * TC_BK, brow);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            // ---------------- MMA issuer (leader CTA only) ----------------
            constexpr uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                       ((uint32_t)(P_BM >> 4) << 24);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = cluster; t < ntiles && ok; t += nclusters) {
                if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_p, gflags, true)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)(acc * BN);
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait(full_bar(stage), phase, abort_p, gflags, true)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = ring + stage * Cfg::STAGE_BYTES;
                    const uint32_t b_addr = a_addr + P_A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 32; kk++)
                        tc2_mma_i8(d_tmem, sw128_desc(a_addr + 32 * kk), sw128_desc(b_addr + 32 * kk), idesc,
                                   (kb | kk) != 0 ? 1u : 0u);
                    tc2_commit_both(empty_bar(stage));
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                tc2_commit_both(tfull_bar(acc));
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            // drain: every MMA issued completes before TMEM is freed
            asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                             drain_bar)
                         : "memory");
            mbar_wait(drain_bar, 0, abort_p, gflags, false);
        }
    } else {
        // ---------------- epilogue (warps 2..9 of both CTAs) ----------------
        const int e = warp - 2;        // 0..7
        const int q = warp & 3;        // TMEM lane quarter this warp may access
        const int half = e >> 2;       // which half of the BN accumulator columns
        const uint32_t stage_s = staging + (uint32_t)(e * 8192);
        uint8_t *stage_g = smem_raw + (stage_s - raw);
        const uint32_t tempty_leader0 = map_to_rank(tempty_bar(0), 0);
        const uint32_t tempty_leader1 = map_to_rank(tempty_bar(1), 0);
        int buf = 0;
        int acc = 0;
        uint32_t acc_phase = 0;
        // The channel scales and biases of the next chunk are loaded as soon as
        // the current chunk's arithmetic is done, so their latency (an L2 round
        // trip behind the operand traffic) overlaps the current chunk's stores
        float sc[32], bi[32];
        const uint64_t nz2 = opaque_nz2((uint32_t)M >> 31);  // M >= 0
        auto chunk_n0 = [&](int tt, int c) {
            return (tt - (tt / tiles_n) * tiles_n) * BN + half * (BN / 2) + c * 32;
        };
        if (!ACC_OUT && cluster < ntiles) w8a8_load_consts(chunk_n0(cluster, 0), N, wscale, bias, sc, bi);
        for (int t = cluster; t < ntiles; t += nclusters) {
            int okw = 0;
            if (lane == 0) okw = mbar_wait(tfull_bar(acc), acc_phase, abort_p, gflags, true) ? 1 : 0;
            okw = __shfl_sync(0xffffffffu, okw, 0);
            if (!okw) break;
            tc_fence_after();
            const int mt = t / tiles_n, nt = t - mt * tiles_n;
            const int mrow0 = mt * P_BM + (int)rank * 128 + q * 32;  // first row of this warp's block
            const int m = mrow0 + lane;
            const uint32_t t_base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + half * (BN / 2));
#pragma unroll 1
            for (int c = 0; c < BN / 64; c++) {
                uint32_t v[32];
                tmem_ld32(t_base + (uint32_t)(c * 32), v);
                tmem_wait_ld();
                const int n0 = nt * BN + half * (BN / 2) + c * 32;
                if (!ACC_OUT) {
                    w8a8_apply32_x2<ACT>(v, a_scale, sc, bi, bias != nullptr, nz2);
                    const bool last = c + 1 == BN / 64;
                    if (!last || t + nclusters < ntiles)
                        w8a8_load_consts(chunk_n0(last ? t + nclusters : t, last ? 0 : c + 1), N, wscale, bias, sc, bi);
                }
                if (!ACC_OUT && Q) {
                    // int8 output requantized with the next point's scale: this
                    // lane's row gets 32 consecutive bytes
                    if (m < M) {
                        uint32_t b[8];
                        requant_pack32_x2(v, q_scale, __frcp_rn(q_scale), requant_fast_ok(q_scale), nz2, b);
                        int8_t *dst = Q + (size_t)m * N + n0;
                        if (n0 + 32 <= N && (N & 15) == 0) {
                            reinterpret_cast<uint4 *>(dst)[0] = make_uint4(b[0], b[1], b[2], b[3]);
                            reinterpret_cast<uint4 *>(dst)[1] = make_uint4(b[4], b[5], b[6], b[7]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; j++)
                                if (n0 + j < N) dst[j] = (int8_t)(b[j / 4] >> (8 * (j % 4)));
                        }
                    }
                } else if (tma_store) {
                    if (mrow0 < M) {  // a block entirely below the last row is not stored
                        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                        __syncwarp();
                        uint8_t *sb = stage_g + buf * 4096 + lane * 128;
#pragma unroll
                        for (int cc = 0; cc < 8; cc++)
                            *reinterpret_cast<uint4 *>(sb + ((cc ^ (lane & 7)) << 4)) =
                                make_uint4(v[4 * cc], v[4 * cc + 1], v[4 * cc + 2], v[4 * cc + 3]);
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&tmY, stage_s + (uint32_t)(buf * 4096), n0, mrow0);
                            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                        }
                        buf ^= 1;
                    }
                } else if (m < M) {
                    uint32_t *dst = ACC_OUT ? reinterpret_cast<uint32_t *>(ACC) + (size_t)m * N + n0
                                            : reinterpret_cast<uint32_t *>(Y) + (size_t)m * N + n0;
                    if (n0 + 32 <= N && (N & 3) == 0) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4)
                            *reinterpret_cast<uint4 *>(dst + j) = make_uint4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (n0 + j < N) dst[j] = v[j];
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            // CTA-scope release: the arrival publishes only that this warp's
            // tensor-memory reads are complete (tcgen05.wait::ld, then the
            // fence above); its global stores need no order against the MMA,
            // and a cluster-scope release would wait for them to reach L2
            if (lane == 0) mbar_arrive_remote(acc == 0 ? tempty_leader0 : tempty_leader1);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        if (tma_store && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }

    // Both CTAs stay resident until neither needs the other: the leader's MMAs
    // read the peer's shared memory, the peer's epilogue arrives on the
    // leader's barriers, and both CTAs' TMA loads signal the leader.
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)Cfg::TMEM_COLS)
                     : "memory");
    }
}

// 2-D 4-byte tensor [rows, cols] (f32 or i32, cols contiguous), box 32 x 32,
// 128B swizzle: the epilogue's store map (stores are clipped to the tensor).
bool make_tmap_out(CUtensorMap *tm, const void *base, uint64_t rows, uint64_t cols, bool is_int) {
    auto fn = encode_fn();
    if (!fn) return false;
    if (((uintptr_t)base & 15) || (cols & 3)) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 4};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(tm, is_int ? CU_TENSOR_MAP_DATA_TYPE_INT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                    const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 2-D uint8 tensor [rows, k] (k contiguous), box [box_rows, 128 B], 128B swizzle,
// out-of-range elements read as zero.
bool make_tmap_i8(CUtensorMap *tm, const void *base, uint64_t rows, uint64_t k, uint32_t box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    if (((uintptr_t)base & 15) || (k & 15)) return false;
    cuuint64_t dims[2] = {k, rows};
    cuuint64_t strides[1] = {k};
    cuuint32_t box[2] = {(cuuint32_t)TC_BK, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int BN, bool ACC_OUT, int ACT>
int launch_tc2_act(tpt_cuda_ctx *ctx, const CUtensorMap &ta, const CUtensorMap &tb, int M, int N, int K,
                   float a_scale, const float *ws, const float *bias, float *y, int32_t *acc, Requant rq) {
    using Cfg = PairCfg<BN>;
    constexpr int P_SMEM_BYTES = Cfg::SMEM_BYTES;
    static bool attr_done[64] = {};
    static int max_clusters[64] = {};
    auto kfn = k_w8a8_tc2<BN, ACC_OUT, ACT>;
    const int dev = ctx->device & 63;
    if (!attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, P_SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "w8a8_tc2 smem attribute");
        // how many SM pairs can hold one cluster each at the same time (the
        // persistent tile loop assumes every launched cluster is resident)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (ctx->sm_count / 2), 1, 1);
        cfg.blockDim = dim3(P_THREADS, 1, 1);
        cfg.dynamicSmemBytes = P_SMEM_BYTES;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 2;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kfn, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = ctx->sm_count / 2;
        }
        max_clusters[dev] = n;
        attr_done[dev] = true;
    }
    const int ntiles = ((M + P_BM - 1) / P_BM) * ((N + BN - 1) / BN);
    const int pairs = max_clusters[dev];
    const int clusters = ntiles < pairs ? ntiles : pairs;
    CUtensorMap ty;
    const bool tma_store = !rq.q && make_tmap_out(&ty, ACC_OUT ? (const void *)acc : (const void *)y, (uint64_t)M,
                                                  (uint64_t)N, ACC_OUT);
    launch_pdl(kfn, 2 * clusters, P_THREADS, P_SMEM_BYTES, ctx->stream, ta, tb, tma_store ? ty : ta, tma_store ? 1 : 0,
               M, N, K, a_scale, ws, bias, y, acc, ctx->d_flags, rq.q, rq.scale);
    return after_launch(ctx, "w8a8_tc2");
}

template <int BN, bool ACC_OUT>
int launch_tc2(tpt_cuda_ctx *ctx, const CUtensorMap &ta, const CUtensorMap &tb, int M, int N, int K, float a_scale,
               const float *ws, const float *bias, int act, float *y, int32_t *acc, Requant rq) {
    if (ACC_OUT || act == TPT_ACT_NONE)  // raw accumulators take no epilogue
        return launch_tc2_act<BN, ACC_OUT, TPT_ACT_NONE>(ctx, ta, tb, M, N, K, a_scale, ws, bias, y, acc, rq);
    if (act == TPT_ACT_RELU)
        return launch_tc2_act<BN, false, TPT_ACT_RELU>(ctx, ta, tb, M, N, K, a_scale, ws, bias, y, acc, rq);
    return launch_tc2_act<BN, false, TPT_ACT_GELU>(ctx, ta, tb, M, N, K, a_scale, ws, bias, y, acc, rq);
}

}  // namespace

// Generic 2-D tiled tensor map (row-major [rows, cols] of elem_bytes-byte
// elements, box box_cols x box_rows); false if the driver entry point is
// missing or the layout breaks TMA's alignment rules.
bool make_tmap_2d(CUtensorMap *tm, CUtensorMapDataType dt, const void *base, uint64_t rows, uint64_t cols,
                  uint32_t elem_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz) {
    auto fn = encode_fn();
    if (!fn) return false;
    if (((uintptr_t)base & 15) || ((cols * elem_bytes) & 15)) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * elem_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(tm, dt, 2, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int build_weight_tmap(tpt_cuda_weights *w) {
    bool ok = w->kind == 8 && w->n <= 0x7fffffff && w->k <= 0x7fffffff;
    const uint32_t rows[4] = {128, 64, 32, 96};
    for (int i = 0; i < 4 && ok; i++)
        ok = make_tmap_i8(reinterpret_cast<CUtensorMap *>(w->tmaps[i]), w->data, w->n, w->k, rows[i]);
    w->tmap_ok = ok;
    return TPT_OK;
}

// Large-M shapes go to the tensor-core kernel: M >= 128, weights with a tensor
// map (K % 16 == 0, 16-byte aligned), A 16-byte aligned.
// M > 64 with the weight's tensor maps available and A 16-byte aligned.
// Tile N (256 / 128 / 64) minimises rounds of tiles over the SM pairs x tile
// width x a per-width cost factor: a narrower tile's lower shared-memory
// efficiency (an M=256 x N=64 MMA reads 5 KB of operands per 64 tensor-core
// cycles per SM against 4 KB at N=256), scaled down for short K, where the
// epilogue's per-output work dominates.
int launch_w8a8_tc(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, const tpt_cuda_weights *w, float a_scale,
                   const float *bias, int act, float *y, int32_t *acc, bool *handled, Requant rq) {
    *handled = false;
    if (!w->tmap_ok || m <= 64 || m > 0x7fffffff) return TPT_OK;
    CUtensorMap ta;
    if (!make_tmap_i8(&ta, a, m, w->k, 128)) return TPT_OK;
    *handled = true;
    const int M = (int)m, N = (int)w->n, K = (int)w->k;
    const long long pairs = ctx->sm_count / 2 > 0 ? ctx->sm_count / 2 : 1;
    const long long mt = (M + P_BM - 1) / P_BM;
    const int widths[4] = {256, 192, 128, 64};
    // per-column cost of a round at long K, from the operand bytes per MMA
    // (measured for 192: 12.8 us per round against 14.6 for 256 at 4096^3)
    const double cost[4] = {1.0, 1.17, 1.6, 2.6};
    // the narrow-tile penalty is an operand-bandwidth cost of the k loop: it
    // fades for short K, where the epilogue (per output, any width) dominates
    const double kw = K < 4096 ? (double)K / 4096.0 : 1.0;
    int bn = 256;
    double best = 0.0;
    for (int i = 0; i < 4; i++) {
        const long long tiles = mt * ((N + widths[i] - 1) / widths[i]);
        const double t = (double)((tiles + pairs - 1) / pairs) * widths[i] * (1.0 + (cost[i] - 1.0) * kw);
        if (i == 0 || t < best) {
            best = t;
            bn = widths[i];
        }
    }
    // each CTA's B box holds BN/2 rows: tmaps[0..3] are the 128 / 64 / 32 / 96-row boxes
    const CUtensorMap *maps = reinterpret_cast<const CUtensorMap *>(w->tmaps);
    if (bn == 192)
        return acc ? launch_tc2<192, true>(ctx, ta, maps[3], M, N, K, a_scale, w->scales, bias, act, y, acc, rq)
                   : launch_tc2<192, false>(ctx, ta, maps[3], M, N, K, a_scale, w->scales, bias, act, y, acc, rq);
    if (bn == 64)
        return acc ? launch_tc2<64, true>(ctx, ta, maps[2], M, N, K, a_scale, w->scales, bias, act, y, acc, rq)
                   : launch_tc2<64, false>(ctx, ta, maps[2], M, N, K, a_scale, w->scales, bias, act, y, acc, rq);
    if (bn == 128)
        return acc ? launch_tc2<128, true>(ctx, ta, maps[1], M, N, K, a_scale, w->scales, bias, act, y, acc, rq)
                   : launch_tc2<128, false>(ctx, ta, maps[1], M, N, K, a_scale, w->scales, bias, act, y, acc, rq);
    return acc ? launch_tc2<256, true>(ctx, ta, maps[0], M, N, K, a_scale, w->scales, bias, act, y, acc, rq)
               : launch_tc2<256, false>(ctx, ta, maps[0], M, N, K, a_scale, w->scales, bias, act, y, acc, rq);
}

}  // namespace tpt
