// conv_tc.cu -- INT8 convolution of an NHWC tensor as an implicit GEMM on the
// tcgen05 tensor cores (kind::i8, i32 accumulators in tensor memory).
//
// The same arithmetic as im2col followed by the W8A8 GEMM (the reference's
// Conv2d, crates/tpt-infer-ops/src/naive.rs:36-83, on quantized operands, with
// the per-channel epilogue of quantized_matmul_i8, crates/tpt-infer-quantize/
// src/ptq.rs:293-324): GEMM row m = output pixel (n, oy, ox), column k =
// (ky, kx, c) of the tap-major, channel-minor weight rows Wt [OC, Kw],
//   acc[m, oc] = sum_k x[n, oy*sh - ph + ky, ox*sw - pw + kx, c] * Wt[oc, k]
// with taps outside the image (and k >= KH*KW*C) contributing zero, then
//   y = (float)acc * (a_scale * w_scale[oc]) + bias[oc], act, and optionally
// the int8 requantization of the next quantization point, and optionally a
// residual added after the activation with a second activation (the plan's
// ADD_ACT folded in: out = act2(y + r)). The rows of the
// im2col matrix are gathered straight from the activation tensor into shared
// memory instead of being written to and read back from HBM.
//
// Tile: 128 output pixels (MMA M) x BN = 64/128/256 output channels (MMA N).
// Two ways to fill the activation operand:
//  - TMA im2col (C % 64 == 0, input >= 128 KB): the tensor unit walks the 128
//    output pixels' windows itself (cp.async.bulk.tensor.4d ... .im2col: the
//    window starts of the tile's first pixel, the tap as the im2col offset,
//    padding read as zeros from outside the tensor's bounding box). A k-block
//    is one tap x KB channels, KB = 128 (128B swizzle) or 64 (C == 64, 64B
//    swizzle, two MMA k-steps).
//  - gather (otherwise, e.g. the 4-channel stem): 128-byte k-blocks (two taps
//    of 64 channels, ..., 32 taps of 4), VB-byte cp.async chunks, VB = 16 when
//    C % 16 == 0 and 4 when C % 4 == 0, so a chunk never straddles two taps.
// Roles (one CTA per SM, persistent over tiles):
//   warp 0      TMA: weight tile [BN rows x KB B] (and the im2col tile)
//   warp 1      TMEM allocation; one lane issues tcgen05.mma (M=128, N=BN,
//               K=32) and the commits
//   warps 2..    epilogue, thread = output pixel (TMEM lane): 4 warps, or 8
//               for 128-wide tiles with TMA operands (two per TMEM lane quarter,
//               alternate 32-column chunks). f32 and int8 rows leave through
//               swizzled staging tiles and bulk-tensor stores; a residual
//               (a folded ADD_ACT) arrives by TMA two chunks ahead; the int8
//               requantization has no division (requant_i8_fast)
//   last 4 warps (gather mode) at each tile the 128 rows' first input pixel goes to a
//               shared table; lane = (chunk of the k-block, pixel row);
//               cp.async with zero fill for padding taps, S - 2 k-blocks in
//               flight per thread; a warp arrives on the stage's barrier
//               after its copies landed and were fenced for the tensor core
// Every wait is bounded (about 1 s); a timeout raises the CTA abort and the
// device timeout flag.
#include "tc_common.cuh"

namespace tpt {

bool make_tmap_2d(CUtensorMap *tm, CUtensorMapDataType dt, const void *base, uint64_t rows, uint64_t cols,
                  uint32_t elem_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz);

namespace {
using namespace tc;

constexpr int CV_BM = 128;                  // output pixels per tile (MMA M)
constexpr int CV_WARP_OUT = 3 * 4096 + 2 * 1024;  // epilogue staging per warp: 3 f32 + 2 int8 32 x 32 tiles
// activation operand modes: gather with 16- or 4-byte chunks (128-byte
// k-blocks), TMA im2col with 128- or 64-byte k-blocks
enum { CV_GATHER16 = 0, CV_GATHER4 = 1, CV_IM2COL128 = 2, CV_IM2COL64 = 3 };
__host__ __device__ constexpr bool cv_tma(int mode) { return mode >= CV_IM2COL128; }
__host__ __device__ constexpr int cv_kb(int mode) { return mode == CV_IM2COL64 ? 64 : 128; }
// epilogue warps: two per TMEM lane quarter (each takes every other 32-column
// chunk) for 128-wide tiles with TMA operands, else one (64-wide tiles have two
// chunks per tile, and 256-wide ones lack the shared memory for the staging)
__host__ __device__ constexpr int cv_epi_warps(int mode, int bn) { return cv_tma(mode) && bn == 128 ? 8 : 4; }
// warp 0 TMA, warp 1 MMA, then the epilogue warps, then (gather modes) 4 gather warps
__host__ __device__ constexpr int cv_threads(int mode, int bn) {
    return 64 + 32 * cv_epi_warps(mode, bn) + (cv_tma(mode) ? 0 : 128);
}

struct ConvShape {
    int N, H, W, C, KH, KW, sh, sw, ph, pw, OH, OW;
    int K;  // KH*KW*C: columns past it are zero
    int Kw; // the weight rows' length (>= K)
};

// RB: the weights of the (single) output-channel tile stay resident in shared
// memory for the whole launch (up to RES_MAX bytes), so a ring stage carries
// only the activation rows: the tensor unit moves a third fewer box lines per
// k-block (128 instead of 128 + BN), which bounds the 64-channel convs
constexpr int CV_RES_MAX = 40 * 1024;
template <int BN, int MODE, bool RB = false>
struct ConvCfg {
    static constexpr int KB = cv_kb(MODE);  // k bytes per stage
    static constexpr int A_BYTES = CV_BM * KB;
    static constexpr int B_BYTES = BN * KB;
    static constexpr int RES_BYTES = RB ? CV_RES_MAX : 0;
    static constexpr int STAGE_BYTES = A_BYTES + (RB ? 0 : B_BYTES);
    static constexpr int EPI = cv_epi_warps(MODE, BN);
    static constexpr int OUT_BYTES = EPI * CV_WARP_OUT;
    static constexpr int STAGES_FIT = (232448 - OUT_BYTES - RES_BYTES - 2048 - 3 * CV_BM * 4) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
    static constexpr int TMEM_COLS = 2 * BN;
    static constexpr int SMEM_BYTES =
        STAGES * STAGE_BYTES + RES_BYTES + OUT_BYTES + (2 * STAGES + 6 + 3 * EPI) * 8 + 1024;
    static_assert(SMEM_BYTES + 3 * CV_BM * 4 + 16 <= 232448, "shared memory (dynamic + the static gather table)");
    static_assert(BN == 64 || BN == 128 || BN == 256, "tile N");
    static_assert(STAGES >= 3, "stages");
};

// Shared-memory matrix descriptor of a K-major operand tile with 64-byte
// rows, 64B swizzle (8-row groups 512 B apart)
__device__ __forceinline__ uint64_t sw64_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(512 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)4 << 61;  // swizzle mode: 64B
    return d;
}
template <int KB>
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr) {
    if constexpr (KB == 64)
        return sw64_desc(saddr);
    else
        return sw128_desc(saddr);
}

// 4-D im2col load: 128 window positions starting at {c, w, h, n} (input
// coordinates of the first output pixel's window), tap offsets {ow, oh}
__device__ __forceinline__ void tma_load_im2col_4d(uint32_t dst, const CUtensorMap *tm, uint32_t bar, int c, int w,
                                                   int h, int n, uint16_t ow, uint16_t oh) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c), "r"(w), "r"(h), "r"(n), "h"(ow), "h"(oh)
        : "memory");
}

template <int VB>
__device__ __forceinline__ void cp_async_zfill(uint32_t dst, const void *src, bool valid) {
    if constexpr (VB == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                     : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(valid ? 4 : 0)
                     : "memory");
}
// waits until at most n (0..7) of this thread's cp.async groups are pending
__device__ __forceinline__ void cp_async_wait_upto(int n) {
    switch (n) {
        case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
        case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
        case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
        case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
        case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
        case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
        case 6: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
        default: asm volatile("cp.async.wait_group 7;" ::: "memory"); break;
    }
}

template <int BN, int MODE, bool RB>
__global__ void __launch_bounds__(cv_threads(MODE, BN), 1)
    k_conv_w8a8(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                const __grid_constant__ CUtensorMap tmY, const __grid_constant__ CUtensorMap tmQ,
                const __grid_constant__ CUtensorMap tmR, int tma_store, int tma_q, int tma_r,
                const int8_t *__restrict__ X, ConvShape cs, int OC, float a_scale, const float *__restrict__ wscale,
                const float *__restrict__ bias, int act, float *__restrict__ Y, int8_t *__restrict__ Q,
                float q_scale, const float *__restrict__ R, int ract, unsigned *gflags) {
    using Cfg = ConvCfg<BN, MODE, RB>;
    constexpr int S = Cfg::STAGES;
    constexpr bool TMA_A = cv_tma(MODE);
    constexpr int KB = Cfg::KB;
    constexpr int VB = MODE == CV_GATHER4 ? 4 : 16;
    constexpr int INFLIGHT = S - 2;  // k-blocks a gather thread keeps in flight
    constexpr int EPI = Cfg::EPI;
    constexpr int GATHER0 = 2 + EPI;  // first gather warp
    extern __shared__ uint8_t smem_raw[];
    __shared__ int abort_flag;
    __shared__ uint32_t tmem_slot;
    // gather table of the tile: image offset, first input row / column of each pixel
    __shared__ int row_base[CV_BM], row_iy[CV_BM], row_ix[CV_BM];

    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t ring = (raw + 1023u) & ~1023u;
    const uint32_t resw = ring + S * Cfg::STAGE_BYTES;  // resident weights (RB), 1 KB aligned
    const uint32_t staging = resw + Cfg::RES_BYTES;
    const uint32_t bars = staging + Cfg::OUT_BYTES;
    auto a_s = [&](int s) { return ring + (uint32_t)(s * Cfg::STAGE_BYTES); };
    // the weight tile of stage s (k-block kb): in the stage, or resident
    auto b_s = [&](int s) { return a_s(s) + (uint32_t)Cfg::A_BYTES; };
    auto b_at = [&](int s, int kb) { return RB ? resw + (uint32_t)(kb * Cfg::B_BYTES) : b_s(s); };
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (S + s); };
    auto tfull_bar = [&](int b) { return bars + 8u * (2 * S + b); };
    auto tempty_bar = [&](int b) { return bars + 8u * (2 * S + 2 + b); };
    const uint32_t drain_bar = bars + 8u * (2 * S + 4);
    const uint32_t wres_bar = bars + 8u * (2 * S + 5 + 3 * EPI);  // the resident weights (RB)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int M = cs.N * cs.OH * cs.OW;
    const int tiles_n = (OC + BN - 1) / BN;
    const int ntiles = ((M + CV_BM - 1) / CV_BM) * tiles_n;
    const int kblocks = (cs.Kw + KB - 1) / KB;
    const int HWo = cs.OH * cs.OW;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; s++) {
            mbar_init(full_bar(s), TMA_A ? 1 : 1 + 4);  // the TMA producer (+ the 4 gather warps)
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), EPI);
        }
        mbar_init(drain_bar, 1);
        for (int b = 0; b < 3 * EPI; b++) mbar_init(bars + 8u * (2 * S + 5 + b), 1);  // residual tiles, 3 per epilogue warp
        mbar_init(wres_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
        if (TMA_A) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
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
    pdl_wait();  // the previous kernel's output (the input tensor) is complete from here on
    pdl_trigger();
    const uint32_t tmem = tmem_slot;
    volatile int *abort_p = &abort_flag;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA: weight tile (and the im2col activation tile) ----------------
            int stage = 0;
            uint32_t phase = 0, issued_mask = 0, last_phase = 0;
            bool ok = true;
            const int cblocks = TMA_A ? cs.C / KB : 1;  // k-blocks per tap
            if (RB) {  // every k-block's weight tile once (one output-channel tile)
                mbar_arrive_expect_tx(wres_bar, (uint32_t)(kblocks * Cfg::B_BYTES));
                for (int kb = 0; kb < kblocks; kb++) tma_load_2d(b_at(0, kb), &tmW, wres_bar, kb * KB, 0);
            }
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const int nt = t % tiles_n, m0 = (t / tiles_n) * CV_BM;
                const int n0 = m0 / HWo, r0 = m0 - n0 * HWo, oy0 = r0 / cs.OW, ox0 = r0 - oy0 * cs.OW;
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_p, gflags, true)) {
                        ok = false;
                        break;
                    }
                    if (TMA_A) {
                        const int tap = kb / cblocks, c0 = (kb - tap * cblocks) * KB;
                        const int ky = tap / cs.KW, kx = tap - ky * cs.KW;
                        mbar_arrive_expect_tx(full_bar(stage), Cfg::A_BYTES + (RB ? 0 : Cfg::B_BYTES));
                        tma_load_im2col_4d(a_s(stage), &tmX, full_bar(stage), c0, ox0 * cs.sw - cs.pw,
                                           oy0 * cs.sh - cs.ph, n0, (uint16_t)kx, (uint16_t)ky);
                    } else {
                        mbar_arrive_expect_tx(full_bar(stage), Cfg::B_BYTES);
                    }
                    if (!RB) tma_load_2d(b_s(stage), &tmW, full_bar(stage), kb * KB, nt * BN);
                    issued_mask |= 1u << stage;
                    last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // our own copies in flight land before the CTA can exit (the
            // stage's barrier also waits for the gather warps)
            if (RB) mbar_wait(wres_bar, 0, abort_p, gflags, false);
            for (int s = 0; s < S; s++)
                if (issued_mask & (1u << s)) mbar_wait(full_bar(s), (last_phase >> s) & 1u, abort_p, gflags, false);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                       ((uint32_t)(CV_BM >> 4) << 24);
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = !RB || mbar_wait(wres_bar, 0, abort_p, gflags, true);
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_p, gflags, true)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + (uint32_t)(acc * BN);
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait(full_bar(stage), phase, abort_p, gflags, true)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < KB / 32; kk++)
                        tc_mma_i8(d_tmem, kmajor_desc<KB>(a_s(stage) + 32 * kk), kmajor_desc<KB>(b_at(stage, kb) + 32 * kk),
                                  idesc, (kb | kk) != 0 ? 1u : 0u);
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
            tc_commit(drain_bar);
            mbar_wait(drain_bar, 0, abort_p, gflags, false);
        }
    } else if (!TMA_A && warp >= GATHER0) {
        // ---------------- gather ----------------
        // VB = 16: lane = (chunk j of 8, row r of a 4-row group), 8 rows per thread;
        // VB = 4:  lane = chunk j of 32, one row per warp step, 32 rows per thread
        constexpr int CPR = 128 / VB;                 // chunks per row
        constexpr int RPW = 32 / CPR;                 // rows a warp covers per step
        constexpr int STEPS = CV_BM / (4 * RPW);      // steps per k-block
        const int gt = threadIdx.x - GATHER0 * 32, gw = gt >> 5, j = lane % CPR, rr = lane / CPR;
        int stage = 0;
        uint32_t phase = 0;
        int pend_stage[S] = {};  // stages whose copies are in flight, oldest first
        int npend = 0;
        bool ok = true;
        auto retire = [&](int keep) {
            // this thread's copies of the oldest stage landed: fence them for the
            // tensor core, and the warp arrives once for the stage
            cp_async_wait_upto(keep);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(full_bar(pend_stage[0]));
            for (int i = 0; i < npend - 1; i++) pend_stage[i] = pend_stage[i + 1];
            npend--;
        };
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
            const int mt = t / tiles_n;
            // the 4 gather warps stop together (they share the named barriers), and
            // every gather thread is done reading the previous tile's table
            if (!bar_and(1, 128, ok)) break;
            {
                const int m = mt * CV_BM + gt;
                if (m < M) {
                    const int n = m / HWo, rem = m - n * HWo, oy = rem / cs.OW, ox = rem - oy * cs.OW;
                    row_base[gt] = n * cs.H * cs.W * cs.C;
                    row_iy[gt] = oy * cs.sh - cs.ph;
                    row_ix[gt] = ox * cs.sw - cs.pw;
                } else {
                    row_base[gt] = 0;
                    row_iy[gt] = -(1 << 28);  // every tap outside: zeros
                    row_ix[gt] = 0;
                }
            }
            bar_sync(1, 128);
            for (int kb = 0; kb < kblocks; kb++) {
                if (!ok) continue;  // stopped: issue nothing more, meet the others at the next tile
                int okw = 1;
                if (lane == 0) okw = mbar_wait(empty_bar(stage), phase ^ 1u, abort_p, gflags, true) ? 1 : 0;
                okw = __shfl_sync(0xffffffffu, okw, 0);
                if (!okw) {
                    ok = false;
                    continue;
                }
                const int k = kb * 128 + j * VB;
                const bool kin = k < cs.K;
                const int tap = kin ? k / cs.C : 0, c = kin ? k - tap * cs.C : 0;
                const int ky = tap / cs.KW, kx = tap - ky * cs.KW;
                const uint32_t chunk_off = (uint32_t)(((j * VB) >> 4) << 4), in16 = (uint32_t)((j * VB) & 15);
#pragma unroll 8
                for (int i = 0; i < STEPS; i++) {
                    const int ml = (i * 4 + gw) * RPW + rr;
                    const int iy = row_iy[ml] + ky, ix = row_ix[ml] + kx;
                    const bool v = kin && iy >= 0 && iy < cs.H && ix >= 0 && ix < cs.W;
                    const int8_t *src = v ? X + row_base[ml] + (iy * cs.W + ix) * cs.C + c : X;
                    cp_async_zfill<VB>(a_s(stage) + (uint32_t)(ml * 128) + ((chunk_off ^ ((ml & 7) << 4))) + in16,
                                       src, v);
                }
                asm volatile("cp.async.commit_group;" ::: "memory");
                pend_stage[npend++] = stage;
                if (npend > INFLIGHT) retire(INFLIGHT);
                if (++stage == S) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        while (npend > 0) retire(npend - 1);
    } else {
        // ---------------- epilogue (warps 2 .. 2 + EPI): thread = output pixel ----------------
        // Per warp: a ring of three 32 x 32 f32 tiles (128B swizzle) and two
        // 32 x 32 int8 tiles (32B swizzle). A chunk's residual block arrives in
        // its f32 tile by TMA two chunks ahead; the result is written back in
        // place and leaves, with its int8 copy, as one bulk store group. With 8
        // epilogue warps, the two warps of a lane quarter take alternate chunks.
        constexpr int CSTEP = EPI / 4;
        const int q = warp & 3;  // TMEM lane quarter
        const int e = warp - 2;
        const int c0 = e >> 2;   // this warp's first chunk of a tile
        const uint32_t ys = staging + (uint32_t)(e * CV_WARP_OUT), qs = ys + 3u * 4096u;
        uint8_t *yg = smem_raw + (ys - raw);
        auto rbar = [&](int b) { return bars + 8u * (2 * S + 5 + 3 * e + b); };
        const bool bulk = (Y && tma_store) || (Q && tma_q);
        const float q_rs = __frcp_rn(q_scale);
        const bool q_fast = requant_fast_ok(q_scale);
        const uint64_t nz2 = opaque_nz2((uint32_t)OC >> 31);  // OC > 0
        int acc = 0, k = 0;
        uint32_t acc_phase = 0, rphase = 0, rpend = 0;
        int pt = blockIdx.x, pcc = c0, pk = 0;  // residual prefetch cursor: tile, chunk, sequence number
        auto issue_r = [&]() {
            while (pt < ntiles && (pt % tiles_n) * BN + pcc * 32 >= OC) {  // no chunk of this warp left in the tile
                pcc = c0;
                pt += gridDim.x;
            }
            if (pt >= ntiles) return;
            const int mt = pt / tiles_n, nt = pt - mt * tiles_n, mrow0 = mt * CV_BM + q * 32, b = pk % 3;
            if (mrow0 < M) {  // blocks entirely below the last row are neither loaded nor stored
                rpend |= 1u << b;
                if (lane == 0) {
                    mbar_arrive_expect_tx(rbar(b), 4096);
                    tma_load_2d(ys + (uint32_t)(b * 4096), &tmR, rbar(b), nt * BN + pcc * 32, mrow0);
                }
            }
            pk++;
            pcc += CSTEP;
            if (pcc >= BN / 32) {
                pcc = c0;
                pt += gridDim.x;
            }
        };
        if (tma_r) {
            issue_r();
            issue_r();
        }
        bool ok = true;
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
            int okw = 0;
            if (lane == 0) okw = mbar_wait(tfull_bar(acc), acc_phase, abort_p, gflags, true) ? 1 : 0;
            okw = __shfl_sync(0xffffffffu, okw, 0);
            if (!okw) break;
            tc_fence_after();
            const int mt = t / tiles_n, nt = t - mt * tiles_n;
            const int mrow0 = mt * CV_BM + q * 32, m = mrow0 + lane;
            const bool live = mrow0 < M;
            const uint32_t t_base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
            for (int cc = c0; cc < BN / 32; cc += CSTEP, k++) {
                const int n0 = nt * BN + cc * 32;
                if (n0 >= OC) break;
                const int b = k % 3;
                uint8_t *sb = yg + b * 4096 + lane * 128;
                uint32_t v[32];
                tmem_ld32(t_base + (uint32_t)(cc * 32), v);
                tmem_wait_ld();
                {
                    float sc[32], bi[32];
                    w8a8_load_consts(n0, OC, wscale, bias, sc, bi);
                    w8a8_apply32_x2<TPT_ACT_NONE>(v, a_scale, sc, bi, bias != nullptr, nz2);
                }
                act32(v, act);
                if (R && tma_r) {  // residual: y = ract(conv + r), the ADD_ACT op's f32 add
                    if (live) {
                        int okr = 0;
                        if (lane == 0) okr = mbar_wait(rbar(b), (rphase >> b) & 1u, abort_p, gflags, true) ? 1 : 0;
                        okr = __shfl_sync(0xffffffffu, okr, 0);
                        __syncwarp();  // lane 0's completed wait orders the tile's bytes for the warp
                        if (!okr) {
                            ok = false;
                            break;
                        }
                        rphase ^= 1u << b;
                        rpend &= ~(1u << b);
#pragma unroll
                        for (int c4 = 0; c4 < 8; c4++) {
                            const float4 r = *reinterpret_cast<const float4 *>(sb + ((c4 ^ (lane & 7)) << 4));
                            float y0, y1, y2, y3;
                            f2unpack(add2(f2pack(__uint_as_float(v[4 * c4]), __uint_as_float(v[4 * c4 + 1])),
                                          f2pack(r.x, r.y)),
                                     y0, y1);
                            f2unpack(add2(f2pack(__uint_as_float(v[4 * c4 + 2]), __uint_as_float(v[4 * c4 + 3])),
                                          f2pack(r.z, r.w)),
                                     y2, y3);
                            v[4 * c4] = __float_as_uint(y0);
                            v[4 * c4 + 1] = __float_as_uint(y1);
                            v[4 * c4 + 2] = __float_as_uint(y2);
                            v[4 * c4 + 3] = __float_as_uint(y3);
                        }
                        act32(v, ract);
                    }
                } else if (R && m < M) {
                    const float *src = R + (size_t)m * OC + n0;
#pragma unroll
                    for (int jj = 0; jj < 32; jj++)
                        if (n0 + jj < OC) v[jj] = __float_as_uint(__fadd_rn(__uint_as_float(v[jj]), src[jj]));
                    act32(v, ract);
                }
                if (Q && live) {
                    uint32_t qb[8];
                    requant_pack32_x2(v, q_scale, q_rs, q_fast, nz2, qb);
                    if (tma_q) {  // 32B swizzle: half h of row `lane` sits at h ^ bit 2 of the row
                        uint8_t *qrow = yg + 3 * 4096 + (k & 1) * 1024 + lane * 32;
                        const int sw = (lane >> 2) & 1;
                        *reinterpret_cast<uint4 *>(qrow + (sw << 4)) = make_uint4(qb[0], qb[1], qb[2], qb[3]);
                        *reinterpret_cast<uint4 *>(qrow + ((sw ^ 1) << 4)) = make_uint4(qb[4], qb[5], qb[6], qb[7]);
                    } else if (m < M) {
                        int8_t *dst = Q + (size_t)m * OC + n0;
                        if (n0 + 32 <= OC && (OC & 15) == 0) {
                            reinterpret_cast<uint4 *>(dst)[0] = make_uint4(qb[0], qb[1], qb[2], qb[3]);
                            reinterpret_cast<uint4 *>(dst)[1] = make_uint4(qb[4], qb[5], qb[6], qb[7]);
                        } else {
                            for (int jj = 0; jj < 32; jj++)
                                if (n0 + jj < OC) dst[jj] = (int8_t)(qb[jj / 4] >> (8 * (jj % 4)));
                        }
                    }
                }
                if (Y && tma_store) {
                    if (live) {
#pragma unroll
                        for (int c4 = 0; c4 < 8; c4++)
                            *reinterpret_cast<uint4 *>(sb + ((c4 ^ (lane & 7)) << 4)) =
                                make_uint4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
                    }
                } else if (Y && m < M) {
                    float *dst = Y + (size_t)m * OC + n0;
                    for (int jj = 0; jj < 32; jj++)
                        if (n0 + jj < OC) dst[jj] = __uint_as_float(v[jj]);
                }
                if (bulk) {
                    if (live) {
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        __syncwarp();
                        if (lane == 0) {
                            if (Y && tma_store) tma_store_2d(&tmY, ys + (uint32_t)(b * 4096), n0, mrow0);
                            if (Q && tma_q) tma_store_2d(&tmQ, qs + (uint32_t)((k & 1) * 1024), n0, mrow0);
                        }
                    }
                    // one group per chunk; after the wait only this chunk's stores may
                    // still read their tiles, so the next chunks' tiles are free
                    if (lane == 0) {
                        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                        asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                    }
                    __syncwarp();
                }
                if (tma_r) {  // two chunks ahead, into the tile of chunk k - 1 (read by every lane by now)
                    __syncwarp();
                    issue_r();
                }
            }
            if (!ok) break;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(acc));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        // residual loads still in flight (an abort) land before the CTA exits
        if (lane == 0)
            for (int b = 0; b < 3; b++)
                if (rpend & (1u << b)) mbar_wait(rbar(b), (rphase >> b) & 1u, abort_p, gflags, false);
        if (bulk && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)Cfg::TMEM_COLS)
                     : "memory");
    }
}

PFN_cuTensorMapEncodeIm2col_v12000 im2col_encode_fn() {
    static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(p);
        else
            cudaGetLastError();
    }
    return fn;
}

// im2col tensor map of the NHWC int8 input [N, H, W, C]: the bounding box of
// window starts runs from -pad to (extent + pad - kernel) per spatial
// dimension with the conv stride as the traversal stride; 128 window
// positions per load, KB channels each, swizzled like the MMA operand.
bool make_tmap_im2col(CUtensorMap *tm, const int8_t *x, const ConvShape &cs, int kb) {
    auto fn = im2col_encode_fn();
    if (!fn) return false;
    cuuint64_t dims[4] = {(cuuint64_t)cs.C, (cuuint64_t)cs.W, (cuuint64_t)cs.H, (cuuint64_t)cs.N};
    cuuint64_t strides[3] = {(cuuint64_t)cs.C, (cuuint64_t)cs.W * cs.C, (cuuint64_t)cs.H * cs.W * cs.C};
    int lower[2] = {-cs.pw, -cs.ph};
    int upper[2] = {cs.pw - (cs.KW - 1), cs.ph - (cs.KH - 1)};
    cuuint32_t estr[4] = {1, (cuuint32_t)cs.sw, (cuuint32_t)cs.sh, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t *>(x), dims, strides, lower, upper,
                    (cuuint32_t)kb, CV_BM, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    kb == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int BN, int MODE, bool RB = false>
int launch_conv(tpt_cuda_ctx *ctx, const int8_t *x, const ConvShape &cs, const CUtensorMap *tx,
                const tpt_cuda_weights *w, float a_scale, const float *bias, int act, float *y, Requant rq,
                const Residual &res) {
    using Cfg = ConvCfg<BN, MODE, RB>;
    static bool attr_done[64] = {};
    auto kfn = k_conv_w8a8<BN, MODE, RB>;
    const int dev = ctx->device & 63;
    if (!attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "conv smem attribute");
        attr_done[dev] = true;
    }
    const int OC = (int)w->n;
    CUtensorMap tw, ty, tq, tr;
    if (!make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->data, w->n, w->k, 1, Cfg::KB, BN,
                      Cfg::KB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
        return TPT_UNSUPPORTED;
    const long long M = (long long)cs.N * cs.OH * cs.OW;
    const bool tma_store = y && make_tmap_2d(&ty, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, y, (uint64_t)M, (uint64_t)OC, 4,
                                                 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    // int8 output rows of 32 bytes (32B swizzle) and residual rows like the f32 output
    const bool tma_q = rq.q && make_tmap_2d(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT8, rq.q, (uint64_t)M, (uint64_t)OC, 1,
                                            32, 32, CU_TENSOR_MAP_SWIZZLE_32B);
    const bool tma_r = res.r && make_tmap_2d(&tr, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, res.r, (uint64_t)M, (uint64_t)OC,
                                             4, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B);
    const long long ntiles = ((M + CV_BM - 1) / CV_BM) * ((OC + BN - 1) / BN);
    const int grid = (int)(ntiles < ctx->sm_count ? ntiles : ctx->sm_count);
    launch_pdl(kfn, grid, cv_threads(MODE, BN), Cfg::SMEM_BYTES, ctx->stream, tw, tx ? *tx : tw, tma_store ? ty : tw,
               tma_q ? tq : tw, tma_r ? tr : tw, tma_store ? 1 : 0, tma_q ? 1 : 0, tma_r ? 1 : 0, x, cs, OC, a_scale,
               w->scales, bias, act, y, rq.q, rq.scale, res.r, res.act, ctx->d_flags);
    return after_launch(ctx, "conv_w8a8");
}

template <int MODE>
int launch_conv_bn(tpt_cuda_ctx *ctx, const int8_t *x, const ConvShape &cs, const CUtensorMap *tx,
                   const tpt_cuda_weights *w, float a_scale, const float *bias, int act, float *y, Requant rq,
                   const Residual &res) {
    // tile N: the widest tile up to the channel count, unless a narrower one
    // fills more SMs: rounds of tiles over the SMs x width x a per-width cost
    // (the narrow tile's operand-bandwidth penalty, fading for short K)
    const long long mt = ((long long)cs.N * cs.OH * cs.OW + CV_BM - 1) / CV_BM;
    const long long sms = ctx->sm_count > 0 ? ctx->sm_count : 1;
    const double kw = w->k < 4096 ? (double)w->k / 4096.0 : 1.0;
    const int widths[3] = {256, 128, 64};
    const double cost[3] = {1.0, 1.6, 2.6};
    int bn = 64;
    double best = 0.0;
    bool first = true;
    for (int i = 0; i < 3; i++) {
        if (i < 2 && w->n <= (size_t)widths[i + 1]) continue;  // wider than the channels need
        const long long tiles = mt * (((long long)w->n + widths[i] - 1) / widths[i]);
        const double t = (double)((tiles + sms - 1) / sms) * widths[i] * (1.0 + (cost[i] - 1.0) * kw);
        if (first || t < best) {
            best = t;
            bn = widths[i];
            first = false;
        }
    }
    // one output-channel tile whose weights fit in shared memory: resident weights
    if (cv_tma(MODE) && bn == 64 && w->n <= 64 && ((w->k + cv_kb(MODE) - 1) / cv_kb(MODE)) * 64 * cv_kb(MODE) <= CV_RES_MAX)
        return launch_conv<64, MODE, true>(ctx, x, cs, tx, w, a_scale, bias, act, y, rq, res);
    if (bn == 64) return launch_conv<64, MODE>(ctx, x, cs, tx, w, a_scale, bias, act, y, rq, res);
    if (bn == 128) return launch_conv<128, MODE>(ctx, x, cs, tx, w, a_scale, bias, act, y, rq, res);
    return launch_conv<256, MODE>(ctx, x, cs, tx, w, a_scale, bias, act, y, rq, res);
}

}  // namespace

// INT8 NHWC convolution as an implicit GEMM. Needs C % 4 == 0, a 16-byte
// aligned input, int8 weights [OC, Kw] with Kw >= KH*KW*C and a tensor map
// (Kw % 16 == 0); returns *handled = false otherwise (the caller runs im2col +
// GEMM instead).
int launch_conv_w8a8(tpt_cuda_ctx *ctx, const int8_t *x, int N, int H, int W, int C, int KH, int KW, int sh, int sw,
                     int ph, int pw, int OH, int OW, const tpt_cuda_weights *w, float a_scale, const float *bias,
                     int act, float *y, bool *handled, Requant rq, Residual res) {
    *handled = false;
    if (w->kind != 8 || !w->tmap_ok || C % 4 != 0 || ((uintptr_t)x & 15) || w->k < (size_t)KH * KW * C ||
        w->n > 0x7fffffff || w->k > 0x7fffffff || (!y && !rq.q) || ((uintptr_t)y & 15))
        return TPT_OK;
    const long long M = (long long)N * OH * OW, xin = (long long)N * H * W * C;
    if (M <= 0 || M > 0x7fffffffLL || xin > 0x7fffffffLL) return TPT_OK;  // 32-bit pixel offsets
    ConvShape cs{N, H, W, C, KH, KW, sh, sw, ph, pw, OH, OW, KH * KW * C, (int)w->k};
    *handled = true;
    // TMA im2col needs channel blocks of 64 or 128 bytes and k-blocks that are
    // whole taps (Kw == K); inputs under 128 KB take the gather instead (the
    // im2col descriptor of a tensor that small is not used on this driver)
    if (C % 64 == 0 && (size_t)KH * KW * C == w->k && xin >= 131072) {
        CUtensorMap tx;
        const int kb = C % 128 == 0 ? 128 : 64;
        if (make_tmap_im2col(&tx, x, cs, kb))
            return kb == 128 ? launch_conv_bn<CV_IM2COL128>(ctx, x, cs, &tx, w, a_scale, bias, act, y, rq, res)
                             : launch_conv_bn<CV_IM2COL64>(ctx, x, cs, &tx, w, a_scale, bias, act, y, rq, res);
    }
    if (C % 16 == 0) return launch_conv_bn<CV_GATHER16>(ctx, x, cs, nullptr, w, a_scale, bias, act, y, rq, res);
    return launch_conv_bn<CV_GATHER4>(ctx, x, cs, nullptr, w, a_scale, bias, act, y, rq, res);
}

}  // namespace tpt
