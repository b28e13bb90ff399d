// stem_pool.cu -- the ResNet stem fused with its max pool: an INT8 4x4
// stride-1 convolution over a 16-channel NHWC tensor (the 7x7 stride-2 stem in
// its 2x2 space-to-depth form) with 64 output channels, bias and ReLU, followed
// by the 3x3 stride-2 pad-1 max pool, on the tcgen05 tensor cores.
//
// Semantics: the plan's IM2COL -> LINEAR_W8A8 (+bias, ReLU) -> MAXPOOL_NHWC
// [-> QUANTIZE] (the reference's Conv2d, crates/tpt-infer-ops/src/naive.rs:36-83,
// on quantized operands with the per-channel epilogue of quantized_matmul_i8,
// crates/tpt-infer-quantize/src/ptq.rs:293-324, then MaxPool2d). Every conv
// output is the same f32 value (exact i32 sum, the scale product, one RN
// multiply, one RN add, ReLU); the pool takes exact maxima of those values,
// window positions outside the image skipped; the optional int8 copy is
// clamp(roundf(y / s)). The conv output itself is never written: per pooled
// row only its three conv rows exist, in tensor memory.
//
// Unit: one pooled row (n, py), from conv rows 2 py - 1 .. 2 py + 1, which read
// input rows 2 py - 1 - ph .. 2 py + 2 - ph + 1 (six rows). Each input row is
// one TMA box of whole 256-byte lines (W * 16 bytes) into a row buffer with
// zero guards on both sides (the horizontal padding). The MMA's A operand for
// conv row r and taps (ty, 2j), (ty, 2j + 1) is a descriptor view of row buffer
// r - ph + ty: K-major without swizzle, pixels 16 bytes apart (core-matrix rows),
// 8-pixel groups 128 bytes apart, and the second 16-byte K chunk (the next tap)
// 16 bytes further, i.e. the next pixel's bytes: the im2col rows are never
// materialised. The weights ([64, 256], 128B-swizzled) stay in shared memory.
//
// Roles (320 threads, two CTAs per SM): warp 0 TMA (weights once, then the six
// rows of each unit into a double-buffered row set); warp 1 tensor memory
// (192 columns: three 64-column accumulators) and the MMAs, 8 per conv row;
// warps 2..9 epilogue, two per TMEM lane quarter (one 32-channel half each),
// thread = conv pixel: the conv rows' values (scale products and biases staged
// once in shared memory), their maximum over the three rows, through shared
// memory the maximum over three pixels, the pooled f32 row and its int8 copy.
// Every wait is bounded.
#include "tc_common.cuh"

namespace tpt {

bool make_tmap_2d(CUtensorMap *tm, CUtensorMapDataType dt, const void *base, uint64_t rows, uint64_t cols,
                  uint32_t elem_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz);
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();

namespace {
using namespace tc;

constexpr int SP_OC = 64;                    // output channels (MMA N)
constexpr int SP_ROW_GUARD = 128;            // zero bytes before a row's data (left padding, aligned data)
constexpr int SP_ROW_BYTES = 128 * 16;       // row data: up to 128 pixels of 16 bytes
constexpr int SP_ROW_STRIDE = SP_ROW_GUARD + SP_ROW_BYTES + 128;  // + a zero tail (right padding, MMA overreach)
constexpr int SP_ROWS = 6;                   // input rows per unit
constexpr int SP_SET_BYTES = SP_ROWS * SP_ROW_STRIDE;
constexpr int SP_W_BYTES = SP_OC * 256;      // weights: 2 k-blocks of [64 rows x 128 B]
constexpr int SP_MAX_STRIDE = 68;            // floats per pixel in the row-max buffer (conflict-free float4)
constexpr int SP_MAX_BYTES = 128 * SP_MAX_STRIDE * 4;
constexpr int SP_EPI = 8;                   // epilogue warps
constexpr int SP_THREADS = 64 + 32 * SP_EPI;
constexpr int SP_TMEM_COLS = 256;            // three 64-column accumulators
constexpr int SP_SMEM = 1024 + SP_W_BYTES + 2 * SP_SET_BYTES + SP_MAX_BYTES + 256 + 2 * SP_OC * 4;

struct StemShape {
    int N, H, W;          // input [N, H, W, 16] int8
    int ph, pw;           // conv padding (4x4 taps, stride 1)
    int OH, OW;           // conv output
    int PH, PW;           // pooled output (3x3, stride 2, pad 1)
    int lines;            // 256-byte lines per input row (W * 16 / 256)
};

// K-major operand without swizzle: rows 16 bytes apart, 8-row groups 128 bytes
// apart, the next 16-byte K chunk `lbo` bytes further
__device__ __forceinline__ uint64_t nosw_desc(uint32_t saddr, uint32_t lbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
    d |= (uint64_t)(lbo >> 4) << 16;
    d |= (uint64_t)(128 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// one input row: `lines` 256-byte lines of image n, row y (zero outside the image)
__device__ __forceinline__ void tma_load_row(uint32_t dst, const CUtensorMap *tm, uint32_t bar, int y, int n) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
        "[%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(0), "r"(0), "r"(y), "r"(n)
        : "memory");
}

__global__ void __launch_bounds__(SP_THREADS, 2)
    k_stem_pool(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, StemShape ss,
                float a_scale, const float *__restrict__ wscale, const float *__restrict__ bias,
                float *__restrict__ P, int8_t *__restrict__ Q, float q_scale, unsigned *gflags) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ int abort_flag;
    __shared__ uint32_t tmem_slot;
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t wsm = (raw + 1023u) & ~1023u;  // 128B swizzle: 1 KB aligned
    const uint32_t sets = wsm + SP_W_BYTES;
    const uint32_t maxs = sets + 2 * SP_SET_BYTES;
    const uint32_t bars = maxs + SP_MAX_BYTES;
    float *cprod = reinterpret_cast<float *>(smem_raw + (bars + 256 - raw));  // a_scale * w_scale[n], then bias[n]
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (2 + s); };
    const uint32_t wbar = bars + 32, tfull = bars + 40, tempty = bars + 48, drain = bars + 56;
    auto row_data = [&](int set, int k) { return sets + (uint32_t)(set * SP_SET_BYTES + k * SP_ROW_STRIDE + SP_ROW_GUARD); };
    float *rowmax = reinterpret_cast<float *>(smem_raw + (maxs - raw));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int units = ss.N * ss.PH;
    const uint32_t row_tx = (uint32_t)ss.lines * 256u;

    // zero the row buffers (their guards and tails stay zero: TMA writes only the data)
    for (int i = threadIdx.x; i < 2 * SP_SET_BYTES / 16; i += SP_THREADS)
        *reinterpret_cast<uint4 *>(smem_raw + (sets - raw) + 16 * i) = make_uint4(0, 0, 0, 0);
    if (threadIdx.x < SP_OC) {  // the epilogue's per-channel constants (the scale product first, as the GEMM's)
        cprod[threadIdx.x] = __fmul_rn(a_scale, __ldg(wscale + threadIdx.x));
        cprod[SP_OC + threadIdx.x] = bias ? __ldg(bias + threadIdx.x) : 0.0f;
    }
    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < 2; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(wbar, 1);
        mbar_init(tfull, 1);
        mbar_init(tempty, SP_EPI);
        mbar_init(drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"((uint32_t)SP_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the zeroed buffers, before the async proxy
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_wait();  // the input (the previous kernel's output) is complete from here on
    pdl_trigger();
    const uint32_t tmem = tmem_slot;
    volatile int *abort_p = &abort_flag;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA: weights once, then six input rows per unit ----------------
            mbar_arrive_expect_tx(wbar, SP_W_BYTES);
            tma_load_2d(wsm, &tmW, wbar, 0, 0);
            tma_load_2d(wsm + SP_W_BYTES / 2, &tmW, wbar, 128, 0);
            int set = 0;
            uint32_t phase = 0, issued = 0, last_phase = 0;
            for (int u = blockIdx.x; u < units; u += gridDim.x) {
                if (!mbar_wait(empty_bar(set), phase ^ 1u, abort_p, gflags, true)) break;
                const int n = u / ss.PH, py = u - n * ss.PH;
                const int y0 = 2 * py - 1 - ss.ph;  // input row of row buffer 0
                mbar_arrive_expect_tx(full_bar(set), SP_ROWS * row_tx);
#pragma unroll 1
                for (int k = 0; k < SP_ROWS; k++) tma_load_row(row_data(set, k), &tmX, full_bar(set), y0 + k, n);
                issued |= 1u << set;
                last_phase = (last_phase & ~(1u << set)) | (phase << set);
                if (++set == 2) {
                    set = 0;
                    phase ^= 1u;
                }
            }
            // our copies in flight land before the CTA can exit
            mbar_wait(wbar, 0, abort_p, gflags, false);
            for (int s = 0; s < 2; s++)
                if (issued & (1u << s)) mbar_wait(full_bar(s), (last_phase >> s) & 1u, abort_p, gflags, false);
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA: 8 per conv row (4 tap rows x 2 tap pairs), K = 32 ----------------
            constexpr uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(SP_OC >> 3) << 17) |
                                       ((uint32_t)(128 >> 4) << 24);
            bool ok = mbar_wait(wbar, 0, abort_p, gflags, true);
            int set = 0;
            uint32_t phase = 0, tphase = 0;
            for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
                if (!mbar_wait(tempty, tphase ^ 1u, abort_p, gflags, true)) break;  // the epilogue read the last unit
                tphase ^= 1u;
                if (!mbar_wait(full_bar(set), phase, abort_p, gflags, true)) break;
                tc_fence_after();
#pragma unroll 1
                for (int ri = 0; ri < 3; ri++) {
#pragma unroll
                    for (int ty = 0; ty < 4; ty++)
#pragma unroll
                        for (int j = 0; j < 2; j++) {
                            // pixel m, taps 2j + c: byte (m + 2j + c - pw) * 16 of row buffer ri + ty
                            const uint64_t ad = nosw_desc(row_data(set, ri + ty) - 16u * ss.pw + 32u * j, 16u);
                            const uint64_t bd = sw128_desc(wsm + (uint32_t)((ty >> 1) * (SP_W_BYTES / 2) + (ty & 1) * 64 + 32 * j));
                            tc_mma_i8(tmem + (uint32_t)(ri * SP_OC), ad, bd, idesc, (ty | j) != 0 ? 1u : 0u);
                        }
                }
                tc_commit(empty_bar(set));
                tc_commit(tfull);
                if (++set == 2) {
                    set = 0;
                    phase ^= 1u;
                }
            }
            tc_commit(drain);
            mbar_wait(drain, 0, abort_p, gflags, false);
        }
    } else {
        // ---------------- epilogue (warps 2..9): thread = conv pixel ----------------
        const int q = warp & 3;             // TMEM lane quarter
        const int c = (warp - 2) >> 2;      // this warp's 32-channel half
        const int ox = q * 32 + lane;
        const int et = threadIdx.x - 64;    // 0 .. 32 SP_EPI - 1
        const float qrs = Q ? __frcp_rn(q_scale) : 0.0f;
        const bool qfast = requant_fast_ok(q_scale);
        const bool has_bias = bias != nullptr;
        const uint64_t nz2 = opaque_nz2((uint32_t)ss.PH >> 31);  // PH > 0
        uint32_t tphase = 0;
        for (int u = blockIdx.x; u < units; u += gridDim.x) {
            int okw = 0;
            if (lane == 0) okw = mbar_wait(tfull, tphase, abort_p, gflags, true) ? 1 : 0;
            okw = __shfl_sync(0xffffffffu, okw, 0);
            if (!bar_and(1, 32 * SP_EPI, okw != 0)) break;
            tphase ^= 1u;
            tc_fence_after();
            const int n = u / ss.PH, py = u - n * ss.PH;
            // the unit's three conv rows that exist: 2 py - 1 (not for py = 0) .. 2 py + 1 (below OH)
            const int r_lo = 2 * py - 1 < 0 ? 1 : 0, r_hi = 2 * py + 1 < ss.OH ? 3 : 2;
            float mx[32];
#pragma unroll
            for (int jj = 0; jj < 32; jj++) mx[jj] = 0.0f;  // every value is ReLU'd (>= +0)
#pragma unroll 1
            for (int ri = r_lo; ri < r_hi; ri++) {
                uint32_t v[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ri * SP_OC + c * 32), v);
                tmem_wait_ld();
#pragma unroll
                for (int jj = 0; jj < 32; jj += 2) {
                    // y = (float)acc * (a_scale * w_scale[n]) + bias[n], ReLU (the W8A8 epilogue's
                    // operations), two channels per paired operation
                    const float2 cp = *reinterpret_cast<const float2 *>(cprod + c * 32 + jj);
                    uint64_t y = mulr2(f2pack(__int2float_rn((int)v[jj]), __int2float_rn((int)v[jj + 1])),
                                       f2pack(cp.x, cp.y), nz2);
                    if (has_bias) {
                        const float2 bb = *reinterpret_cast<const float2 *>(cprod + SP_OC + c * 32 + jj);
                        y = add2(y, f2pack(bb.x, bb.y));
                    }
                    float y0, y1;
                    f2unpack(y, y0, y1);
                    mx[jj] = fmaxf(mx[jj], y0 > 0.0f ? y0 : 0.0f);
                    mx[jj + 1] = fmaxf(mx[jj + 1], y1 > 0.0f ? y1 : 0.0f);
                }
            }
            {
                float *dst = rowmax + ox * SP_MAX_STRIDE + c * 32;
#pragma unroll
                for (int c4 = 0; c4 < 8; c4++)
                    reinterpret_cast<float4 *>(dst)[c4] = make_float4(mx[4 * c4], mx[4 * c4 + 1], mx[4 * c4 + 2], mx[4 * c4 + 3]);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty);  // tensor memory is free for the next unit
            bar_sync(1, 32 * SP_EPI);           // every pixel's row maximum is in shared memory
            // the pooled row: px over the conv pixels 2 px - 1 .. 2 px + 1 inside the image
            const size_t orow = ((size_t)n * ss.PH + py) * ss.PW;
            for (int idx = et; idx < ss.PW * 16; idx += 32 * SP_EPI) {
                const int px = idx >> 4, c4 = idx & 15;
                const int x0 = 2 * px - 1 < 0 ? 0 : 2 * px - 1, x1 = 2 * px + 1 < ss.OW ? 2 * px + 1 : ss.OW - 1;
                float4 m = reinterpret_cast<const float4 *>(rowmax + x0 * SP_MAX_STRIDE)[c4];
                for (int x = x0 + 1; x <= x1; x++) {
                    const float4 v = reinterpret_cast<const float4 *>(rowmax + x * SP_MAX_STRIDE)[c4];
                    m.x = fmaxf(m.x, v.x);
                    m.y = fmaxf(m.y, v.y);
                    m.z = fmaxf(m.z, v.z);
                    m.w = fmaxf(m.w, v.w);
                }
                const size_t o = (orow + px) * SP_OC + 4 * c4;
                if (P) *reinterpret_cast<float4 *>(P + o) = m;
                if (Q) {
                    int8_t a, b, cq, d;
                    if (qfast) {
                        requant_i8_fast_x2(m.x, m.y, q_scale, qrs, nz2, a, b);
                        requant_i8_fast_x2(m.z, m.w, q_scale, qrs, nz2, cq, d);
                    } else {
                        a = requant_i8(m.x, q_scale);
                        b = requant_i8(m.y, q_scale);
                        cq = requant_i8(m.z, q_scale);
                        d = requant_i8(m.w, q_scale);
                    }
                    *reinterpret_cast<uint32_t *>(Q + o) = (uint32_t)(uint8_t)a | ((uint32_t)(uint8_t)b << 8) |
                                                           ((uint32_t)(uint8_t)cq << 16) | ((uint32_t)(uint8_t)d << 24);
                }
            }
            bar_sync(1, 32 * SP_EPI);  // the row maxima are read before the next unit writes them
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)SP_TMEM_COLS)
                     : "memory");
    }
}

// 4-D view of the NHWC input [N, H, W, 16] as {256-byte line, line, row, image}:
// one box is a whole row (`lines` lines), rows outside the image read as zero.
bool make_tmap_rows(CUtensorMap *tm, const int8_t *x, const StemShape &ss) {
    auto fn = encode_fn();
    if (!fn) return false;
    const uint64_t rowb = (uint64_t)ss.W * 16;
    cuuint64_t dims[4] = {256, (cuuint64_t)ss.lines, (cuuint64_t)ss.H, (cuuint64_t)ss.N};
    cuuint64_t strides[3] = {256, rowb, rowb * ss.H};
    cuuint32_t box[4] = {256, (cuuint32_t)ss.lines, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t *>(x), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace

// The fused stem + max pool. Handles: 16 input channels, 4x4 taps, stride 1,
// padding <= 3, W % 16 == 0 and W <= 128, OW <= 128 and OW <= W + 2 pw - 3,
// 64 output channels with a tensor map, weights [64, 256]; the pool 3x3 stride
// 2 pad 1 with PH = (OH - 1) / 2 + 1, PW = (OW - 1) / 2 + 1; a 16-byte aligned
// input and outputs. Returns handled = false otherwise.
int launch_stem_pool(tpt_cuda_ctx *ctx, const int8_t *x, int N, int H, int W, int C, int KH, int KW, int sh, int sw,
                     int ph, int pw, int OH, int OW, const tpt_cuda_weights *w, float a_scale, const float *bias,
                     int act, int PH, int PW, float *P, int8_t *Q, float q_scale, bool *handled) {
    *handled = false;
    if (C != 16 || KH != 4 || KW != 4 || sh != 1 || sw != 1 || ph < 0 || ph > 3 || pw < 0 || pw > 3) return TPT_OK;
    if (act != TPT_ACT_RELU || w->kind != 8 || !w->tmap_ok || w->n != SP_OC || w->k != 256) return TPT_OK;
    if (W % 16 != 0 || W > 128 || OW > 128 || OH <= 0 || OW <= 0 || OW > W + 2 * pw - 3 || OH > H + 2 * ph - 3)
        return TPT_OK;
    if (PH != (OH - 1) / 2 + 1 || PW != (OW - 1) / 2 + 1 || (!P && !Q)) return TPT_OK;
    if (((uintptr_t)x | (uintptr_t)P | (uintptr_t)Q) & 15) return TPT_OK;
    if ((long long)N * H * W * C > 0x7fffffffLL) return TPT_OK;
    StemShape ss{N, H, W, ph, pw, OH, OW, PH, PW, W * 16 / 256};
    CUtensorMap tx;
    if (!make_tmap_rows(&tx, x, ss)) return TPT_OK;
    // the weights' 64-row box (tmaps[1]): [64 rows x 128 B], 128B swizzle
    const CUtensorMap *tw = reinterpret_cast<const CUtensorMap *>(w->tmaps[1]);
    static bool attr_done[64] = {};
    const int dev = ctx->device & 63;
    if (!attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(k_stem_pool, cudaFuncAttributeMaxDynamicSharedMemorySize, SP_SMEM);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "stem_pool smem attribute");
        attr_done[dev] = true;
    }
    *handled = true;
    const int units = N * PH;
    const int ctas = 2 * (ctx->sm_count > 0 ? ctx->sm_count : 1);
    launch_pdl(k_stem_pool, units < ctas ? units : ctas, SP_THREADS, SP_SMEM, ctx->stream, tx, *tw, ss, a_scale,
               w->scales, bias, P, Q, q_scale, ctx->d_flags);
    return after_launch(ctx, "stem_pool");
}

}  // namespace tpt
