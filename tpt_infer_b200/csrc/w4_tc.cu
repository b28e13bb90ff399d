// w4_tc.cu -- INT4-weight x f32-activation GEMM on the tcgen05 tensor cores
// (kind::f16, f32 accumulators in tensor memory) for M >= 3.
//
// Reference semantics: dequantize_i4_symmetric_per_channel then the f32 matmul
// (crates/tpt-infer-quantize/src/dequant.rs:56-71, crates/tpt-infer-ops/src/
// avx512.rs:55-78): y[m,n] = sum_k x[m,k] * (q[n,k] * s[n]) + bias[n], then act.
//
// Numerics. q in [-8, 7] is exact in fp16. Each activation is split once into
// fp16 hi = rn(x) and lo = rn(x - hi) (x ~ hi + lo to ~2^-22 relative), and both
// products accumulate in f32: acc[n,m] = sum_k q*hi + q*lo. The epilogue applies
// y = acc * s[n] + bias[n]. The tensor core's f32 accumulation loses a little at
// every accumulate step, so consecutive k-blocks go to W4_SUBS separate TMEM
// accumulators (k-block kb -> sub kb % W4_SUBS), each seeing 1/W4_SUBS of the
// steps, and the epilogue adds the subs in IEEE f32. The result stays inside the
// strict W4 tolerance (1e-3 x max|y| / 127), which a single fp16 or bf16 pass
// would not meet.
//
// Orientation. The MMA's M side is 128 WEIGHT rows (output channels) and its N
// side is BN activation rows, so a decode-like M = 8 still runs full-height
// MMAs and streams each weight byte from HBM once per BN activation rows.
//
// Pipeline per CTA (persistent over (weight tile, activation tile) units):
//   warp 0      TMA: nibbles [128 rows x 32 B] (64 k) into a staging buffer,
//               x_hi and x_lo [BN rows x 64 fp16] into 128B-swizzled buffers
//   warps 2..5  unpack: one weight row per thread, 8 nibbles per 32-bit word
//               -> 8 fp16 with two LOP3s and one fp16 subtract per pair,
//               written into the 128B-swizzled K-major fp16 weight tile
//   warp 1      tcgen05.mma (M=128, N=BN, K=16) x {hi, lo} per k-step
//   warps 6..9  epilogue: tcgen05.ld, thread = weight row, so the per-channel
//               scale and bias live in registers and each store instruction
//               writes 32 consecutive output channels of one activation row.
// K order inside each group of 8 is permuted identically in the weights (the
// unpacker's natural order) and the activations (the split kernel), which
// leaves the sum of products unchanged.
#include <cuda_fp16.h>

#include "tc_common.cuh"

namespace tpt {

bool make_tmap_2d(CUtensorMap *tm, CUtensorMapDataType dt, const void *base, uint64_t rows, uint64_t cols,
                  uint32_t elem_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz);
int launch_w4_simt(tpt_cuda_ctx *ctx, const float *x, const uint8_t *packed, const float *scales, const float *bias,
                   int act, float *y, size_t m, size_t n, size_t k);

namespace {
using namespace tc;

constexpr int W4_TM = 128;   // weight rows per tile (MMA M)
constexpr int W4_SUBS = 4;   // TMEM sub-accumulators per tile
constexpr int W4_KB = 64;    // k per stage (one 128-byte fp16 row)
constexpr int W4_THREADS = 320;
constexpr int NIB_BYTES = W4_TM * (W4_KB / 2);  // 4 KB
constexpr int W16_BYTES = W4_TM * W4_KB * 2;    // 16 KB

template <int BN>
struct W4Cfg {
    static constexpr int X_BYTES = BN * W4_KB * 2;
    static constexpr int STAGE_BYTES = NIB_BYTES + W16_BYTES + 2 * X_BYTES;
    static constexpr int STAGES_RAW = 204800 / STAGE_BYTES;
    static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
    static constexpr int TMEM_COLS = 2 * W4_SUBS * BN;  // double-buffered, W4_SUBS subs
    static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + (3 * STAGES + 5) * 8 + 16 + 1024;
    static_assert(SMEM_BYTES <= 232448, "shared memory");
    static_assert(BN == 32 || BN == 64, "activation tile");
    static_assert(TMEM_COLS <= 512, "tensor memory");
};

// 8 signed nibbles (low nibble first) -> 4 half2: (n0,n4) (n1,n5) (n2,n6) (n3,n7).
// (u ^ 8) = v + 8 in [0, 15]; as the low mantissa bits of 1024.0 it gives
// 1024 + v + 8 exactly; subtracting 1032 leaves v.
__device__ __forceinline__ uint4 unpack8(uint32_t w) {
    const uint32_t magic = 0x64006400u, mask = 0x000F000Fu, flip = 0x00080008u;
    const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1032
    uint32_t t[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        uint32_t u = ((w >> (4 * i)) & mask) ^ flip;
        u |= magic;
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

template <int BN>
__global__ void __launch_bounds__(W4_THREADS, 1)
    k_w4_tc(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmXh,
            const __grid_constant__ CUtensorMap tmXl, int M, int N, int K, const float *__restrict__ wscale,
            const float *__restrict__ bias, int act, float *__restrict__ Y, unsigned *gflags) {
    using Cfg = W4Cfg<BN>;
    constexpr int S = Cfg::STAGES;
    extern __shared__ uint8_t smem_raw[];
    __shared__ int abort_flag;
    __shared__ uint32_t tmem_slot;

    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t ring = (raw + 1023u) & ~1023u;
    auto nib_s = [&](int s) { return ring + (uint32_t)(s * Cfg::STAGE_BYTES); };
    auto w16_s = [&](int s) { return nib_s(s) + NIB_BYTES; };
    auto xh_s = [&](int s) { return w16_s(s) + W16_BYTES; };
    auto xl_s = [&](int s) { return xh_s(s) + Cfg::X_BYTES; };
    const uint32_t bars = ring + S * Cfg::STAGE_BYTES;
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto wready_bar = [&](int s) { return bars + 8u * (S + s); };
    auto empty_bar = [&](int s) { return bars + 8u * (2 * S + s); };
    auto tfull_bar = [&](int b) { return bars + 8u * (3 * S + b); };
    auto tempty_bar = [&](int b) { return bars + 8u * (3 * S + 2 + b); };
    const uint32_t drain_bar = bars + 8u * (3 * S + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_w = (N + W4_TM - 1) / W4_TM, tiles_x = (M + BN - 1) / BN;
    const int ntiles = tiles_w * tiles_x;
    const int kblocks = K / W4_KB;

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(wready_bar(s), 4 * 32);
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), 4);
        }
        mbar_init(drain_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
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
    // unit t -> (weight tile, activation tile); consecutive CTAs take different
    // weight tiles of the same activation tile
    auto unit = [&](int t, int &wt, int &xt) {
        xt = t / tiles_w;
        wt = t - xt * tiles_w;
    };

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int stage = 0;
            uint32_t phase = 0, issued_mask = 0, last_phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                int wt, xt;
                unit(t, wt, xt);
                for (int kb = 0; kb < kblocks; kb++) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1u, abort_p, gflags, true)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(stage), NIB_BYTES + 2 * Cfg::X_BYTES);
                    tma_load_2d(nib_s(stage), &tmW, full_bar(stage), kb * (W4_KB / 2), wt * W4_TM);
                    tma_load_2d(xh_s(stage), &tmXh, full_bar(stage), kb * W4_KB, xt * BN);
                    tma_load_2d(xl_s(stage), &tmXl, full_bar(stage), kb * W4_KB, xt * BN);
                    issued_mask |= 1u << stage;
                    last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == S) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            for (int s = 0; s < S; s++)
                if (issued_mask & (1u << s)) mbar_wait(full_bar(s), (last_phase >> s) & 1u, abort_p, gflags, false);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = (1u << 4)  // D: f32
                                       | (0u << 7) | (0u << 10)  // A, B: f16
                                       | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(W4_TM >> 4) << 24);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1u, abort_p, gflags, true)) break;
                tc_fence_after();
                const uint32_t d_base = tmem + (uint32_t)(acc * W4_SUBS * BN);
                for (int kb = 0; kb < kblocks; kb++) {
                    const uint32_t d_tmem = d_base + (uint32_t)((kb % W4_SUBS) * BN);
                    if (!mbar_wait(full_bar(stage), phase, abort_p, gflags, true) ||
                        !mbar_wait(wready_bar(stage), phase, abort_p, gflags, true)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < W4_KB / 16; kk++) {
                        const uint64_t a = sw128_desc(w16_s(stage) + 32 * kk);
                        tc_mma_f16(d_tmem, a, sw128_desc(xh_s(stage) + 32 * kk), idesc,
                                   (kb >= W4_SUBS || kk != 0) ? 1u : 0u);
                        tc_mma_f16(d_tmem, a, sw128_desc(xl_s(stage) + 32 * kk), idesc, 1u);
                    }
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
    } else if (warp < 6) {
        // ---------------- nibble unpack (warps 2..5): thread = weight row ----------------
        const int r = threadIdx.x - 64;  // 0..127
        uint8_t *nib_g = smem_raw + (ring - raw);
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
            for (int kb = 0; kb < kblocks; kb++) {
                // every thread observes the TMA completion of the bytes it reads
                if (!mbar_wait(full_bar(stage), phase, abort_p, gflags, true)) {
                    ok = false;
                    break;
                }
                const uint8_t *src = nib_g + (size_t)stage * Cfg::STAGE_BYTES + r * 32;
                const uint4 p0 = *reinterpret_cast<const uint4 *>(src);
                const uint4 p1 = *reinterpret_cast<const uint4 *>(src + 16);
                uint8_t *dst = nib_g + (size_t)stage * Cfg::STAGE_BYTES + NIB_BYTES + r * 128;
                const uint32_t words[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
                for (int c = 0; c < 8; c++)
                    *reinterpret_cast<uint4 *>(dst + ((c ^ (r & 7)) << 4)) = unpack8(words[c]);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_arrive(wready_bar(stage));
                if (++stage == S) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
    } else {
        // ---------------- epilogue (warps 6..9): thread = weight row ----------------
        const int q = warp & 3;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
            int wt, xt;
            unit(t, wt, xt);
            int okw = 0;
            if (lane == 0) okw = mbar_wait(tfull_bar(acc), acc_phase, abort_p, gflags, true) ? 1 : 0;
            okw = __shfl_sync(0xffffffffu, okw, 0);
            __syncwarp();
            if (!okw) break;
            tc_fence_after();
            const int n = wt * W4_TM + q * 32 + lane;
            const bool nv = n < N;
            const float sc = nv ? __ldg(wscale + n) : 0.0f;
            const float bi = (nv && bias) ? __ldg(bias + n) : 0.0f;
            const uint32_t t_base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * W4_SUBS * BN);
            const int nsubs = kblocks < W4_SUBS ? kblocks : W4_SUBS;
#pragma unroll 1
            for (int c = 0; c < BN / 32; c++) {
                float a[32];
                uint32_t v[32];
                tmem_ld32(t_base + (uint32_t)(c * 32), v);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; j++) a[j] = __uint_as_float(v[j]);
#pragma unroll 1
                for (int sub = 1; sub < nsubs; sub++) {
                    tmem_ld32(t_base + (uint32_t)(sub * BN + c * 32), v);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; j++) a[j] += __uint_as_float(v[j]);
                }
                const int m0 = xt * BN + c * 32;
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    if (nv && m0 + j < M) {
                        float y = a[j] * sc;
                        if (bias) y += bi;
                        Y[(size_t)(m0 + j) * N + n] = apply_act(y, act);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(acc));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
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
    const int ntiles = ((N + W4_TM - 1) / W4_TM) * ((M + BN - 1) / BN);
    const int grid = ntiles < ctx->sm_count ? ntiles : ctx->sm_count;
    k_w4_tc<BN><<<grid, W4_THREADS, Cfg::SMEM_BYTES, ctx->stream>>>(tw, th, tl, M, N, K, ws, bias, act, y, ctx->d_flags);
    return after_launch(ctx, "w4_tc");
}

}  // namespace

// Tensor-core W4 for M >= 3 with K % 64 == 0; returns handled = false otherwise.
int launch_w4_tc(tpt_cuda_ctx *ctx, const float *x, size_t m, const tpt_cuda_weights *w, const float *bias, int act,
                 float *y, bool *handled) {
    *handled = false;
    const size_t n = w->n, k = w->k;
    if (m < 3 || k % W4_KB || m > 0x7fffffff || n > 0x7fffffff || ((uintptr_t)x & 15)) return TPT_OK;
    int st = ensure_ws(ctx, 2 * m * k * sizeof(__half) + 256);
    if (st) return st;
    __half *hi = reinterpret_cast<__half *>(ctx->ws);
    __half *lo = hi + m * k;
    CUtensorMap tw, th, tl;
    const int BN = m <= 32 ? 32 : 64;
    if (!make_tmap_2d(&tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, w->data, n, k / 2, 1, W4_KB / 2, W4_TM,
                      CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_tmap_2d(&th, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, hi, m, k, 2, W4_KB, BN, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_tmap_2d(&tl, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, lo, m, k, 2, W4_KB, BN, CU_TENSOR_MAP_SWIZZLE_128B))
        return TPT_OK;
    *handled = true;
    const size_t groups = m * k / 8;
    k_split_f16<<<grid_1d(groups, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream>>>(x, hi, lo, groups);
    st = after_launch(ctx, "w4_split");
    if (st) return st;
    if (BN == 32) return launch_w4_tc_bn<32>(ctx, tw, th, tl, (int)m, (int)n, (int)k, w->scales, bias, act, y);
    return launch_w4_tc_bn<64>(ctx, tw, th, tl, (int)m, (int)n, (int)k, w->scales, bias, act, y);
}

}  // namespace tpt
