// w4_tc.cu -- INT4-weight x f32-activation GEMM on the tcgen05 tensor cores
// (kind::f16, f32 accumulators in tensor memory), stream-K over the weight
// bytes.
//
// Reference semantics: dequantize_i4_symmetric_per_channel then the f32 matmul
// (crates/tpt-infer-quantize/src/dequant.rs:56-71, crates/tpt-infer-ops/src/
// avx512.rs:55-78): y[m,n] = sum_k x[m,k] * (q[n,k] * s[n]) + bias[n], then act.
//
// Numerics. q in [-8, 7] is exact in fp16. Each activation is split once into
// fp16 hi = rn(x) and lo = rn(x - hi) (x ~ hi + lo to ~2^-22 relative), and both
// products accumulate in f32. x_hi and x_lo of a BN-row activation tile are
// stacked along the MMA's N side (2 x BN rows in one 128B-swizzled tile), so one
// MMA per 16-k step yields both sum_k q*hi and sum_k q*lo in separate TMEM
// columns and reads the weight tile once. The tensor core's f32 accumulation
// loses a little at every accumulate step, so consecutive k-blocks of a segment
// go to SUBS separate accumulators (block i -> sub i % SUBS); the epilogue adds
// subs and halves in IEEE f32 and applies y = acc * s[n] + bias[n]. The result
// stays inside the strict W4 tolerance (1e-3 x max|y| / 127), which a single
// fp16 or bf16 pass would not meet.
//
// Orientation. The MMA's M side is 128 WEIGHT rows (output channels) and its N
// side BN = 16/32/64/128 activation rows, so a decode-like M still runs
// full-height MMAs and each weight byte is unpacked once per BN activation rows.
//
// Stream-K. The (tile, 128-k block) units are split into one equal contiguous
// range per CTA, so all SMs share the nibble stream and the unpacking. A CTA
// covering a whole tile writes the output directly; otherwise it stores its
// f32 partial tile in its own slot of the tile (plain coalesced stores; slot =
// CTA - first contributor) and counts itself; the CTA completing the count sums
// the slots in slot order (deterministic for a given launch shape) and applies
// the epilogue. Nothing waits on another CTA.
//
// Roles (480 threads, one CTA per SM):
//   warp 0       TMA: nibbles [128 rows x 64 B] (128 k) into a ring (HBM)
//   warp 14      TMA: x_hi, x_lo [BN rows x 64 fp16] x 2 sub-tiles into their own ring
//                (L2 hits; freed by the MMA commit, so they run ahead of it)
//   warps 6..13  unpack: thread = (weight row, half of the 32 B), 8 nibbles per
//                32-bit word -> 8 fp16 with one LOP3 and one fp16 subtract per
//                pair, written into a short ring of 128B-swizzled K-major fp16
//                weight tiles
//   warp 1       tcgen05.mma (M=128, N=2 x BN, K=16) per k-step
//   warps 2..5   epilogue, thread = weight row (TMEM lane)
// K order inside each group of 8 is permuted identically in the weights (the
// unpacker's natural order) and the activations (the split kernel), which
// leaves the sum of products unchanged. All waits are bounded (1 s).
#include <cuda_fp16.h>

#include "tc_common.cuh"

namespace tpt {

bool make_tmap_2d(CUtensorMap *tm, CUtensorMapDataType dt, const void *base, uint64_t rows, uint64_t cols,
                  uint32_t elem_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz);

namespace {
using namespace tc;

constexpr int W4_TM = 128;                      // weight rows per tile (MMA M)
constexpr int W4_KB = 128;                      // k per block (two 64-k sub-tiles)
constexpr int W4_SUBK = 64;                     // k of one 128B-swizzled fp16 sub-tile
constexpr int NIB_BYTES = W4_TM * (W4_KB / 2);  // 8 KB of nibbles per block
constexpr int W16_SUB = W4_TM * W4_SUBK * 2;    // 16 KB: one fp16 weight sub-tile
constexpr int W16_BYTES = 2 * W16_SUB;          // 32 KB fp16 weight tile per block
constexpr int W4_UNPACK_WARPS = 8;
constexpr int W4_THREADS = 15 * 32;
constexpr int W4_EPI = 128;

template <int BN>
struct W4Cfg {
    static constexpr int X_BYTES = BN * W4_SUBK * 2;  // one of x_hi / x_lo for one 64-k sub-tile
    // activation stage: [x_hi; x_lo] of sub-tile 0, then of sub-tile 1 (each pair
    // is the MMA's 2 x BN-row B operand), multiple of 1024
    static constexpr int XSTG_BYTES = 4 * X_BYTES;
    static constexpr int NS = BN == 16 ? 8 : BN == 128 ? 4 : 6;  // nibble stages (HBM latency)
    static constexpr int XS = BN == 16 ? 4 : BN == 32 ? 4 : 2;   // activation stages (L2 latency)
    static constexpr int WS = BN == 128 ? 2 : 3;                 // fp16 weight stages (unpack -> MMA)
    static constexpr int SUBS = BN <= 32 ? 4 : BN == 64 ? 2 : 1;
    static constexpr int ACC_STRIDE = 2 * BN;             // columns of one sub-accumulator (hi | lo)
    static constexpr int TMEM_COLS = 2 * SUBS * ACC_STRIDE;  // double-buffered
    static constexpr int NBARS = 2 * NS + 2 * XS + 2 * WS + 5;
    static constexpr int SMEM_BYTES = WS * W16_BYTES + XS * XSTG_BYTES + NS * NIB_BYTES + NBARS * 8 + 1024;
    static_assert(BN == 16 || BN == 32 || BN == 64 || BN == 128, "activation tile");
    static_assert(SMEM_BYTES <= 232448, "shared memory");
    static_assert(TMEM_COLS <= 512, "tensor memory");
};

// 8 signed nibbles (low nibble first) -> 4 half2: (n0,n4) (n1,n5) (n2,n6) (n3,n7).
// (u ^ 8) = v + 8 in [0, 15]; as the low mantissa bits of 1024.0 it gives
// 1024 + v + 8 exactly; subtracting 1032 leaves v.
__device__ __forceinline__ uint4 unpack8(uint32_t w) {
    const uint32_t mask = 0x000F000Fu, magic_flip = 0x64086408u;  // (u & mask) ^ 0x0008 | 0x6400
    const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
    uint32_t t[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint32_t u = ((w >> (4 * i)) & mask) ^ magic_flip;
        __half2 h = __hsub2(*reinterpret_cast<__half2 *>(&u), bias);
        t[i] = *reinterpret_cast<uint32_t *>(&h);
    }
    return make_uint4(t[0], t[1], t[2], t[3]);
}

__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// C columns (16 or 32) of this thread's TMEM lane: for each of `nsubs`
// accumulators spaced `stride` columns apart, the hi column plus the lo column
// `lo_off` further, added in sub order.
template <int C>
__device__ __forceinline__ void load_sum(uint32_t taddr, int nsubs, uint32_t stride, uint32_t lo_off, float (&a)[C]) {
    uint32_t v[C], w[C];
#pragma unroll
    for (int j = 0; j < C; j++) a[j] = 0.0f;
    for (int s = 0; s < nsubs; s++) {
        if constexpr (C == 16) {
            tmem_ld16(taddr + s * stride, v);
            tmem_ld16(taddr + s * stride + lo_off, w);
        } else {
            tmem_ld32(taddr + s * stride, v);
            tmem_ld32(taddr + s * stride + lo_off, w);
        }
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < C; j++) a[j] += __uint_as_float(v[j]) + __uint_as_float(w[j]);
    }
}

template <int BN>
__global__ void __launch_bounds__(W4_THREADS, 1)
    k_w4_tc(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmXh,
            const __grid_constant__ CUtensorMap tmXl, int M, int N, int K, const float *__restrict__ wscale,
            const float *__restrict__ bias, int act, float *__restrict__ Y, float *__restrict__ part,
            int *__restrict__ cnt, unsigned *gflags) {
    using Cfg = W4Cfg<BN>;
    constexpr int NS = Cfg::NS, XS = Cfg::XS, WS = Cfg::WS, SUBS = Cfg::SUBS, AS = Cfg::ACC_STRIDE;
    constexpr int CW = BN < 32 ? BN : 32;  // epilogue column chunk
    extern __shared__ uint8_t smem_raw[];
    __shared__ int abort_flag;
    __shared__ int last_flag;
    __shared__ int fin_slot[TPT_SK_MAX_CTAS];  // the finishing CTA's table of contributor slots
    __shared__ uint32_t tmem_slot;

    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t w16 = (raw + 1023u) & ~1023u;  // WS fp16 weight tiles (1 KB aligned)
    const uint32_t xst = w16 + WS * W16_BYTES;    // XS activation stages
    const uint32_t nib = xst + XS * Cfg::XSTG_BYTES;
    const uint32_t bars = nib + NS * NIB_BYTES;
    auto w16_s = [&](int s) { return w16 + (uint32_t)(s * W16_BYTES); };
    // x_hi / x_lo of 64-k sub-tile j of activation stage s
    auto xh_s = [&](int s, int j) { return xst + (uint32_t)(s * Cfg::XSTG_BYTES + j * 2 * Cfg::X_BYTES); };
    auto xl_s = [&](int s, int j) { return xh_s(s, j) + Cfg::X_BYTES; };
    auto nib_s = [&](int s) { return nib + (uint32_t)(s * NIB_BYTES); };
    auto full_nib = [&](int s) { return bars + 8u * s; };
    auto empty_nib = [&](int s) { return bars + 8u * (NS + s); };
    auto full_x = [&](int s) { return bars + 8u * (2 * NS + s); };
    auto empty_x = [&](int s) { return bars + 8u * (2 * NS + XS + s); };
    auto wready = [&](int s) { return bars + 8u * (2 * NS + 2 * XS + s); };
    auto empty_w16 = [&](int s) { return bars + 8u * (2 * NS + 2 * XS + WS + s); };
    auto tfull_bar = [&](int b) { return bars + 8u * (2 * NS + 2 * XS + 2 * WS + b); };
    auto tempty_bar = [&](int b) { return bars + 8u * (2 * NS + 2 * XS + 2 * WS + 2 + b); };
    const uint32_t drain_bar = bars + 8u * (2 * NS + 2 * XS + 2 * WS + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_w = (N + W4_TM - 1) / W4_TM, tiles_x = (M + BN - 1) / BN;
    const int kblocks = K / W4_KB;
    const long long units = (long long)tiles_w * tiles_x * kblocks;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < NS; s++) {
            mbar_init(full_nib(s), 1);
            mbar_init(empty_nib(s), W4_UNPACK_WARPS);
        }
        for (int s = 0; s < XS; s++) {
            mbar_init(full_x(s), 1);
            mbar_init(empty_x(s), 1);
        }
        for (int s = 0; s < WS; s++) {
            mbar_init(wready(s), W4_UNPACK_WARPS);
            mbar_init(empty_w16(s), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), W4_EPI);
        }
        mbar_init(drain_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmXh)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmXl)) : "memory");
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
    pdl_wait();  // the previous kernel's output (x_hi / x_lo) is complete from here on
    pdl_trigger();
    const uint32_t tmem = tmem_slot;
    volatile int *abort_p = &abort_flag;
    SkRange range(units, kblocks, blockIdx.x, gridDim.x);
    int tile, kb0, kb1;

    if (warp == 0 || warp == 14) {
        if (lane == 0) {
            // ---------------- TMA producers: nibbles (warp 0), activations (warp 14) ----------------
            const bool is_nib = warp == 0;
            const int S = is_nib ? NS : XS;
            int stage = 0;
            uint32_t phase = 0, issued_mask = 0, last_phase = 0;
            bool ok = true;
            while (ok && range.next(tile, kb0, kb1)) {
                const int xt = tile / tiles_w, wt = tile - xt * tiles_w;
                for (int kb = kb0; kb < kb1; kb++) {
                    const uint32_t fb = is_nib ? full_nib(stage) : full_x(stage);
                    if (!mbar_wait(is_nib ? empty_nib(stage) : empty_x(stage), phase ^ 1u, abort_p, gflags, true)) {
                        ok = false;
                        break;
                    }
                    if (is_nib) {
                        mbar_arrive_expect_tx(fb, NIB_BYTES);
                        tma_load_2d(nib_s(stage), &tmW, fb, kb * (W4_KB / 2), wt * W4_TM);
                    } else {
                        mbar_arrive_expect_tx(fb, Cfg::XSTG_BYTES);
#pragma unroll
                        for (int j = 0; j < 2; j++) {
                            tma_load_2d(xh_s(stage, j), &tmXh, fb, kb * W4_KB + j * W4_SUBK, xt * BN);
                            tma_load_2d(xl_s(stage, j), &tmXl, fb, kb * W4_KB + j * W4_SUBK, xt * BN);
                        }
                    }
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
                if (issued_mask & (1u << s))
                    mbar_wait(is_nib ? full_nib(s) : full_x(s), (last_phase >> s) & 1u, abort_p, gflags, false);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = (1u << 4)  // D: f32
                                       | (0u << 7) | (0u << 10)  // A, B: f16
                                       | ((uint32_t)((2 * BN) >> 3) << 17) | ((uint32_t)(W4_TM >> 4) << 24);
            int xs = 0, ws = 0, acc = 0;
            uint32_t xph = 0, wph = 0, acc_phase = 0;
            bool ok = true;
            while (ok && range.next(tile, kb0, kb1)) {
                if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_p, gflags, true)) break;
                tc_fence_after();
                const uint32_t d_base = tmem + (uint32_t)(acc * SUBS * AS);
                for (int kb = kb0; kb < kb1; kb++) {
                    const int i = kb - kb0;
                    const uint32_t d_tmem = d_base + (uint32_t)((i % SUBS) * AS);
                    if (!mbar_wait(full_x(xs), xph, abort_p, gflags, true) ||
                        !mbar_wait(wready(ws), wph, abort_p, gflags, true)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < W4_KB / 16; kk++) {  // B = [x_hi; x_lo], 2 x BN rows
                        const int j = kk / (W4_SUBK / 16), k16 = kk % (W4_SUBK / 16);
                        tc_mma_f16(d_tmem, sw128_desc(w16_s(ws) + j * W16_SUB + 32 * k16),
                                   sw128_desc(xh_s(xs, j) + 32 * k16), idesc, (i >= SUBS || kk != 0) ? 1u : 0u);
                    }
                    tc_commit(empty_x(xs));
                    tc_commit(empty_w16(ws));
                    if (++xs == XS) {
                        xs = 0;
                        xph ^= 1u;
                    }
                    if (++ws == WS) {
                        ws = 0;
                        wph ^= 1u;
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
    } else if (warp >= 6) {
        // ---------------- nibble unpack (warps 6..13) ----------------
        const int u = threadIdx.x - 6 * 32;  // 0..255
        const int r = u & (W4_TM - 1), half = u >> 7;
        int ns = 0, ws = 0;
        uint32_t nph = 0, wph = 0;
        bool ok = true;
        while (ok && range.next(tile, kb0, kb1)) {
            for (int kb = kb0; kb < kb1; kb++) {
                // the fp16 tile is free (MMA done with it) and the nibbles landed
                if (!mbar_wait(empty_w16(ws), wph ^ 1u, abort_p, gflags, true) ||
                    !mbar_wait(full_nib(ns), nph, abort_p, gflags, true)) {
                    ok = false;
                    break;
                }
                // this thread: row r, k-half `half` (= fp16 sub-tile) of the block's 64 nibble bytes
                const uint8_t *src = smem_raw + (nib_s(ns) - raw) + r * 64 + half * 32;
                const uint4 p0 = *reinterpret_cast<const uint4 *>(src);
                const uint4 p1 = *reinterpret_cast<const uint4 *>(src + 16);
                __syncwarp();
                if (lane == 0) mbar_arrive(empty_nib(ns));
                uint8_t *dst = smem_raw + (w16_s(ws) - raw) + half * W16_SUB + r * 128;
                const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
                for (int c = 0; c < 8; c++)  // 16-byte chunk c of the sub-tile's 128-byte fp16 row
                    *reinterpret_cast<uint4 *>(dst + ((c ^ (r & 7)) << 4)) = unpack8(words[c]);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(wready(ws));
                if (++ns == NS) {
                    ns = 0;
                    nph ^= 1u;
                }
                if (++ws == WS) {
                    ws = 0;
                    wph ^= 1u;
                }
            }
        }
    } else {
        // ---------------- epilogue (warps 2..5): thread = weight row ----------------
        const int q = warp & 3;
        const int r = q * 32 + lane;
        const int epi_tid = threadIdx.x - 64;
        int acc = 0;
        uint32_t acc_phase = 0;
        while (range.next(tile, kb0, kb1)) {
            const int xt = tile / tiles_w, wt = tile - xt * tiles_w;
            const bool okw = mbar_wait(tfull_bar(acc), acc_phase, abort_p, gflags, true);
            if (!bar_and(1, W4_EPI, okw)) break;
            tc_fence_after();
            const int n = wt * W4_TM + r;
            const bool nv = n < N;
            const float sc = nv ? __ldg(wscale + n) : 0.0f;
            const float bi = (nv && bias) ? __ldg(bias + n) : 0.0f;
            const int m0 = xt * BN;
            const bool full = kb0 == 0 && kb1 == kblocks;
            const int nsubs = kb1 - kb0 < SUBS ? kb1 - kb0 : SUBS;
            const uint32_t t_base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * SUBS * AS);
            auto emit = [&](int j, float a) {
                float y = a * sc;
                if (bias) y += bi;
                Y[(size_t)(m0 + j) * N + n] = apply_act(y, act);
            };
            const long long ub = (long long)tile * kblocks;
            const int c_first = full ? 0 : sk_cta_of_unit(ub, units, gridDim.x);
            const int nslots = full ? 1 : sk_cta_of_unit(ub + kblocks - 1, units, gridDim.x) - c_first + 1;
            constexpr size_t SLOT = (size_t)BN * W4_TM;
            float *mine = part + (size_t)(full ? 0 : sk_slot(blockIdx.x, tile, units, kblocks, gridDim.x)) * SLOT + r;
#pragma unroll 1
            for (int c = 0; c < BN / CW; c++) {
                float a[CW];
                load_sum<CW>(t_base + (uint32_t)(c * CW), nsubs, (uint32_t)AS, (uint32_t)BN, a);
#pragma unroll
                for (int j = 0; j < CW; j++) {
                    const int jj = c * CW + j;
                    if (nv && m0 + jj < M) {
                        if (full)
                            emit(jj, a[j]);
                        else
                            mine[(size_t)jj * W4_TM] = a[j];
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(tempty_bar(acc));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
            if (full) continue;
            __threadfence();
            bar_sync(1, W4_EPI);
            if (epi_tid == 0) last_flag = (atomicAdd(cnt + c_first, 1) + 1 == nslots) ? 1 : 0;
            bar_sync(1, W4_EPI);
            if (last_flag) {
                __threadfence();
                for (int i = epi_tid; i < nslots; i += W4_EPI)
                    fin_slot[i] = sk_slot(c_first + i, tile, units, kblocks, gridDim.x);
                bar_sync(1, W4_EPI);
                constexpr int JG = BN < 8 ? BN : 8, SG = 4;
#pragma unroll 1
                for (int j0 = 0; j0 < BN; j0 += JG) {
                    float a[JG];
#pragma unroll
                    for (int jj = 0; jj < JG; jj++) a[jj] = 0.0f;
#pragma unroll 1
                    for (int s0 = 0; s0 < nslots; s0 += SG) {
                        float b[SG][JG];
#pragma unroll
                        for (int sl = 0; sl < SG; sl++)
#pragma unroll
                            for (int jj = 0; jj < JG; jj++)
                                b[sl][jj] = (s0 + sl < nslots && nv && m0 + j0 + jj < M)
                                                ? __ldcg(part + (size_t)fin_slot[s0 + sl] * SLOT + r + (size_t)(j0 + jj) * W4_TM)
                                                : 0.0f;
#pragma unroll
                        for (int sl = 0; sl < SG; sl++)
#pragma unroll
                            for (int jj = 0; jj < JG; jj++)
                                if (s0 + sl < nslots) a[jj] += b[sl][jj];
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

// x f32 [M, K] -> hi, lo fp16 [M, K]; inside each group of 8 the k order is
// (0, 4, 1, 5, 2, 6, 3, 7), the order the unpacker produces for the weights.
__global__ void k_split_f16(const float *__restrict__ x, __half *__restrict__ hi, __half *__restrict__ lo, size_t groups) {
    pdl_wait();
    pdl_trigger();
    for (size_t g = blockIdx.x * (size_t)blockDim.x + threadIdx.x; g < groups; g += (size_t)gridDim.x * blockDim.x) {
        const float4 a = __ldg(reinterpret_cast<const float4 *>(x) + 2 * g);
        const float4 b = __ldg(reinterpret_cast<const float4 *>(x) + 2 * g + 1);
        const float v[8] = {a.x, b.x, a.y, b.y, a.z, b.z, a.w, b.w};  // k = 0,4,1,5,2,6,3,7
        __half h[8], l[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            h[i] = __float2half_rn(v[i]);
            l[i] = __float2half_rn(v[i] - __half2float(h[i]));
        }
        *reinterpret_cast<uint4 *>(hi + 8 * g) = *reinterpret_cast<uint4 *>(h);
        *reinterpret_cast<uint4 *>(lo + 8 * g) = *reinterpret_cast<uint4 *>(l);
    }
}

template <int BN>
int launch_w4_tc_bn(tpt_cuda_ctx *ctx, const CUtensorMap &tw, const CUtensorMap &th, const CUtensorMap &tl, int M,
                    int N, int K, const float *ws, const float *bias, int act, float *y) {
    using Cfg = W4Cfg<BN>;
    static bool attr[64] = {};
    if (!attr[ctx->device & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_w4_tc<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "w4_tc smem attribute");
        attr[ctx->device & 63] = true;
    }
    const int tiles = ((N + W4_TM - 1) / W4_TM) * ((M + BN - 1) / BN);
    const int kblocks = K / W4_KB;
    const long long units = (long long)tiles * kblocks;
    const int ctas = ctx->sm_count < tc::TPT_SK_MAX_CTAS ? ctx->sm_count : tc::TPT_SK_MAX_CTAS;
    // fewer than two units per SM: whole tiles per CTA, no cross-CTA reduction
    const int grid = units < 2LL * ctas ? (tiles < ctas ? tiles : ctas) : ctas;
    int st = ensure_sk(ctx, (size_t)2 * grid * BN * W4_TM * sizeof(float));
    if (st) return st;
    int *cnt = reinterpret_cast<int *>(ctx->sk);
    float *part = reinterpret_cast<float *>(ctx->sk + TPT_SK_SLOTS_OFFSET);
    k_w4_tc<BN><<<grid, W4_THREADS, Cfg::SMEM_BYTES, ctx->stream>>>(tw, th, tl, M, N, K, ws, bias, act, y, part, cnt,
                                                                    ctx->d_flags);
    return after_launch(ctx, "w4_tc");
}

}  // namespace

// Tensor-core W4 for K % 128 == 0 and a 16-byte aligned x; returns handled =
// false otherwise (the caller falls back to the SIMT kernel).
int launch_w4_tc(tpt_cuda_ctx *ctx, const float *x, size_t m, const tpt_cuda_weights *w, const float *bias, int act,
                 float *y, bool *handled) {
    *handled = false;
    const size_t n = w->n, k = w->k;
    if (m == 0 || k == 0 || k % W4_KB || m > 0x7fffffff || n > 0x7fffffff || ((uintptr_t)x & 15)) return TPT_OK;
    int st = ensure_ws(ctx, 2 * m * k * sizeof(__half) + 256);
    if (st) return st;
    __half *hi = reinterpret_cast<__half *>(ctx->ws);
    __half *lo = hi + m * k;
    CUtensorMap tw, th, tl;
    const int BN = m <= 16 ? 16 : m <= 32 ? 32 : m <= 64 ? 64 : 128;
    if (!make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->data, n, k / 2, 1, W4_KB / 2, W4_TM,
                      CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_tmap_2d(&th, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, hi, m, k, 2, W4_SUBK, BN, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_2d(&tl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, lo, m, k, 2, W4_SUBK, BN, CU_TENSOR_MAP_SWIZZLE_128B))
        return TPT_OK;
    *handled = true;
    const size_t groups = m * k / 8;
    k_split_f16<<<grid_1d(groups, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream>>>(x, hi, lo, groups);
    st = after_launch(ctx, "w4_split");
    if (st) return st;
    const int M = (int)m, N = (int)n, K = (int)k;
    if (BN == 16) return launch_w4_tc_bn<16>(ctx, tw, th, tl, M, N, K, w->scales, bias, act, y);
    if (BN == 32) return launch_w4_tc_bn<32>(ctx, tw, th, tl, M, N, K, w->scales, bias, act, y);
    if (BN == 64) return launch_w4_tc_bn<64>(ctx, tw, th, tl, M, N, K, w->scales, bias, act, y);
    return launch_w4_tc_bn<128>(ctx, tw, th, tl, M, N, K, w->scales, bias, act, y);
}

}  // namespace tpt
