// attention_tc.cu -- fused attention softmax(scale * Q K^T) V per (batch, head)
// on the tcgen05 tensor cores (kind::tf32, f32 accumulators in tensor memory).
//
// Semantics: the composition the encoder graph runs with the reference's ops,
// MatMul -> Softmax -> MatMul (crates/tpt-infer-ops/src/naive.rs:13-33 and
// :104-125) on each head: S = (scale * Q) K^T, P = softmax(S) by rows (max
// subtract, exp, sum, divide), O = P V. qkv is the packed projection output
// [B*S, 3*H*D] (Q | K | V along columns); the context is [B*S, H*D].
//
// Numerics (3xTF32). Every operand x is split into hi = x rounded to tf32
// (to nearest, ties away: two integer ops on the bits) and lo = x - hi (exact
// in f32; the tensor core reads its leading tf32 bits); each product runs as
// hi*hi + hi*lo + lo*hi with f32 accumulation, which carries ~21 bits of the
// operands -- f32-class accuracy, where a single tf32 pass would give ~2^-11.
// tf32 keeps f32's exponent range, so no scaling is needed.
//
// One CTA per (batch, head), S <= 128 (keys past S masked, queries past S not
// stored), D = 64, 512 threads:
//   all threads   load Q, K, V (f32), split, and store them as 128B-swizzled
//                 K-major tf32 tiles: Q and K [128 rows x 64], V transposed
//                 [64 rows x 128 keys]
//   thread 0      issues S = Q K^T (M=128, N=128, K=8 per MMA; 24 MMAs)
//   all threads   softmax: thread = (query row = TMEM lane, quarter of the
//                 keys); row max and sum meet in shared memory; P = e * (1/sum)
//                 (the correctly rounded reciprocal: within an ulp of the
//                 reference's division) is split and stored as K-major tiles
//                 over the Q/K space
//   thread 0      issues O = P V (M=128, N=64; 48 MMAs)
//   all threads   O from tensor memory through a shared staging tile to
//                 coalesced rows of the context (f32, or int8 at the next
//                 quantization point's scale)
// Waits on the MMA commits are bounded (about 1 s); a timeout records the
// device timeout flag and the CTA skips the rest.
#include "tc_common.cuh"

namespace tpt {
namespace {
using namespace tc;

constexpr int AT_D = 64;      // head dimension
constexpr int AT_S = 128;     // largest sequence length
constexpr int AT_THREADS = 512;
// dynamic shared memory, from a 1 KB aligned base:
//   [0, 128K)    Q hi, Q lo, K hi, K lo (2 sub-tiles of 32 tf32 columns each, 16 KB)
//                -> P hi, P lo after S (4 sub-tiles of 32 keys each, 16 KB)
//                -> the output staging tile after O
//   [128K, 192K) V^T hi, V^T lo (4 sub-tiles [64 rows x 32 keys], 8 KB each)
constexpr uint32_t OFF_QH = 0, OFF_QL = 32768, OFF_KH = 65536, OFF_KL = 98304;
constexpr uint32_t OFF_PH = 0, OFF_PL = 65536;
constexpr uint32_t OFF_VH = 131072, OFF_VL = 163840;
constexpr int OST = AT_D + 4;  // staging row stride (floats)
constexpr int AT_TC_SMEM = 196608 + 1024;
constexpr uint32_t AT_TMEM_COLS = 256;  // S: columns [0, 128); O: [128, 192)

// x rounded to the 10 fraction bits of tf32, to nearest with ties away from
// zero: add half a tf32 ulp to the magnitude bits, clear the 13 low bits (a
// carry into the exponent is the correct rounding up)
__device__ __forceinline__ uint32_t tf32_rna(float x) { return (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u; }
// x -> (hi, lo) with hi + lo = x exactly in f32
__device__ __forceinline__ void split_tf32(float x, uint32_t &hi, uint32_t &lo) {
    hi = tf32_rna(x);
    lo = __float_as_uint(__fsub_rn(x, __uint_as_float(hi)));
}
__device__ __forceinline__ void split4(float4 v, uint4 &hi, uint4 &lo) {
    split_tf32(v.x, hi.x, lo.x);
    split_tf32(v.y, hi.y, lo.y);
    split_tf32(v.z, hi.z, lo.z);
    split_tf32(v.w, hi.w, lo.w);
}

__device__ __forceinline__ void tc_mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D = f32, A = B = tf32, both K-major; N >> 3 at bit 17, M >> 4 at bit 24
__host__ __device__ constexpr uint32_t at_idesc(int m, int n) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__global__ void __launch_bounds__(AT_THREADS, 1)
    k_attention_tc(const float *__restrict__ qkv, float *__restrict__ out, int S, int H, float scale,
                   int8_t *__restrict__ qout, float qs, unsigned *gflags) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bars[2];
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    __shared__ float red[2][4][AT_S];  // [max | sum][key quarter][row]

    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *g = smem_raw + (base - raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.y, h = blockIdx.x;
    const int HD = H * AT_D, ld = 3 * HD;
    const float *src = qkv + (size_t)b * S * ld + h * AT_D;
    const uint32_t s_bar = smem_u32(&bars[0]), o_bar = smem_u32(&bars[1]);

    if (tid == 0) {
        abort_flag = 0;
        mbar_init(s_bar, 1);
        mbar_init(o_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(AT_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }

    pdl_wait();  // the previous kernel's output (qkv) is complete from here on
    pdl_trigger();

    // ---- load and split: item = (row r, 4 consecutive d at 4*c4); rows past S
    // are zero. A warp's 32 items are 8 consecutive rows x 4 consecutive chunks
    // (64-byte global segments; the transposed V stores spread over the banks).
    // Every load of the thread is issued before the first use.
    constexpr int ITEMS = AT_S * (AT_D / 4) / AT_THREADS;  // 4
    auto item = [&](int it, int &r, int &c4) {
        const int i = tid + it * AT_THREADS, w = i >> 5, l = i & 31;
        r = (w >> 2) * 8 + (l & 7);
        c4 = (w & 3) * 4 + (l >> 3);
    };
    float4 qv[ITEMS], kv[ITEMS], vv[ITEMS];
#pragma unroll
    for (int it = 0; it < ITEMS; it++) {
        int r, c4;
        item(it, r, c4);
        qv[it] = kv[it] = vv[it] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (r < S) {
            const float *p = src + (size_t)r * ld + 4 * c4;
            qv[it] = __ldg(reinterpret_cast<const float4 *>(p));
            kv[it] = __ldg(reinterpret_cast<const float4 *>(p + HD));
            vv[it] = __ldg(reinterpret_cast<const float4 *>(p + 2 * HD));
        }
    }
#pragma unroll
    for (int it = 0; it < ITEMS; it++) {
        int r, c4;
        item(it, r, c4);
        const float4 q = make_float4(__fmul_rn(qv[it].x, scale), __fmul_rn(qv[it].y, scale),
                                     __fmul_rn(qv[it].z, scale), __fmul_rn(qv[it].w, scale));
        uint4 hi, lo;
        // Q, K: row r, 32-column sub-tile c4 / 8, 16-byte chunk c4 % 8 (128B swizzle)
        const uint32_t off = (uint32_t)((c4 >> 3) * 16384 + r * 128 + (((c4 & 7) ^ (r & 7)) << 4));
        split4(q, hi, lo);
        *reinterpret_cast<uint4 *>(g + OFF_QH + off) = hi;
        *reinterpret_cast<uint4 *>(g + OFF_QL + off) = lo;
        split4(kv[it], hi, lo);
        *reinterpret_cast<uint4 *>(g + OFF_KH + off) = hi;
        *reinterpret_cast<uint4 *>(g + OFF_KL + off) = lo;
        // V^T: element (key r, dim d) -> row d of key sub-tile r / 32, chunk (r % 32) / 4, word r % 4
        const float ve[4] = {vv[it].x, vv[it].y, vv[it].z, vv[it].w};
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int d = 4 * c4 + e;
            const uint32_t vo =
                (uint32_t)((r >> 5) * 8192 + d * 128 + ((((r & 31) >> 2) ^ (d & 7)) << 4) + (r & 3) * 4);
            uint32_t vh, vl;
            split_tf32(ve[e], vh, vl);
            *reinterpret_cast<uint32_t *>(g + OFF_VH + vo) = vh;
            *reinterpret_cast<uint32_t *>(g + OFF_VL + vo) = vl;
        }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // st.shared -> the tensor core's reads
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    volatile int *abort_p = &abort_flag;

    if (tid == 0) {
        // S = Q K^T: hi*hi + hi*lo + lo*hi, each over 2 sub-tiles x 4 k-steps of 8
        const uint32_t A[3] = {base + OFF_QH, base + OFF_QH, base + OFF_QL};
        const uint32_t B[3] = {base + OFF_KH, base + OFF_KL, base + OFF_KH};
#pragma unroll 1
        for (int p = 0; p < 3; p++)
#pragma unroll
            for (int j = 0; j < 2; j++)
#pragma unroll
                for (int k8 = 0; k8 < 4; k8++)
                    tc_mma_tf32(tmem, sw128_desc(A[p] + j * 16384 + 32 * k8), sw128_desc(B[p] + j * 16384 + 32 * k8),
                                at_idesc(128, 128), (p | j | k8) != 0 ? 1u : 0u);
        tc_commit(s_bar);
    }

    const int row = (warp & 3) * 32 + lane, qtr = warp >> 2;  // TMEM lane; keys / dims quarter
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    bool ok = __syncthreads_and(mbar_wait(s_bar, 0, abort_p, gflags, true));
    if (ok) {
        tc_fence_after();
        // ---- softmax over this thread's 32 keys, combined with the other quarters
        uint32_t sv[32];
        tmem_ld32(lane_base + (uint32_t)(qtr * 32), sv);
        tmem_wait_ld();
        const int nvalid = S - qtr * 32;  // keys of this quarter below S
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < 32; j++)
            if (j < nvalid) m = fmaxf(m, __uint_as_float(sv[j]));
        red[0][qtr][row] = m;
        __syncthreads();
        m = fmaxf(fmaxf(red[0][0][row], red[0][1][row]), fmaxf(red[0][2][row], red[0][3][row]));
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const float e = j < nvalid ? expf(__uint_as_float(sv[j]) - m) : 0.0f;
            sv[j] = __float_as_uint(e);
            sum += e;
        }
        red[1][qtr][row] = sum;
        __syncthreads();
        sum = ((red[1][0][row] + red[1][1][row]) + red[1][2][row]) + red[1][3][row];
        const float rs = __frcp_rn(sum);
        // P = e / sum, split, into key sub-tile `qtr` of row `row`
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const float4 pv = make_float4(__fmul_rn(__uint_as_float(sv[4 * c]), rs),
                                          __fmul_rn(__uint_as_float(sv[4 * c + 1]), rs),
                                          __fmul_rn(__uint_as_float(sv[4 * c + 2]), rs),
                                          __fmul_rn(__uint_as_float(sv[4 * c + 3]), rs));
            uint4 hi, lo;
            split4(pv, hi, lo);
            const uint32_t off = (uint32_t)(qtr * 16384 + row * 128 + ((c ^ (row & 7)) << 4));
            *reinterpret_cast<uint4 *>(g + OFF_PH + off) = hi;
            *reinterpret_cast<uint4 *>(g + OFF_PL + off) = lo;
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            // O = P V: hi*hi + hi*lo + lo*hi, each over 4 key sub-tiles x 4 k-steps of 8
            const uint32_t A[3] = {base + OFF_PH, base + OFF_PH, base + OFF_PL};
            const uint32_t B[3] = {base + OFF_VH, base + OFF_VL, base + OFF_VH};
#pragma unroll 1
            for (int p = 0; p < 3; p++)
#pragma unroll
                for (int j = 0; j < 4; j++)
#pragma unroll
                    for (int k8 = 0; k8 < 4; k8++)
                        tc_mma_tf32(tmem + 128, sw128_desc(A[p] + j * 16384 + 32 * k8),
                                    sw128_desc(B[p] + j * 8192 + 32 * k8), at_idesc(128, 64), (p | j | k8) != 0 ? 1u : 0u);
            tc_commit(o_bar);
        }
        ok = __syncthreads_and(mbar_wait(o_bar, 0, abort_p, gflags, true));
        if (ok) {
            tc_fence_after();
            // ---- O: thread (row, dims qtr*16 + [0, 16)) -> staging [128][OST] -> coalesced rows
            uint32_t ov[16];
            tmem_ld16(lane_base + 128u + (uint32_t)(qtr * 16), ov);
            tmem_wait_ld();
            float *st = reinterpret_cast<float *>(g);  // over P (its MMAs are done)
#pragma unroll
            for (int c = 0; c < 4; c++)
                *reinterpret_cast<float4 *>(st + row * OST + qtr * 16 + 4 * c) =
                    make_float4(__uint_as_float(ov[4 * c]), __uint_as_float(ov[4 * c + 1]),
                                __uint_as_float(ov[4 * c + 2]), __uint_as_float(ov[4 * c + 3]));
            __syncthreads();
            for (int i = tid; i < AT_S * (AT_D / 4); i += AT_THREADS) {
                const int r = i >> 4, c4 = i & 15;
                if (r >= S) continue;
                const float4 o = *reinterpret_cast<const float4 *>(st + r * OST + 4 * c4);
                const size_t off = ((size_t)b * S + r) * HD + h * AT_D + 4 * c4;
                if (qout)  // the following QUANTIZE, fused: the f32 context is not written
                    *reinterpret_cast<uint32_t *>(qout + off) =
                        (uint32_t)(uint8_t)requant_i8(o.x, qs) | ((uint32_t)(uint8_t)requant_i8(o.y, qs) << 8) |
                        ((uint32_t)(uint8_t)requant_i8(o.z, qs) << 16) | ((uint32_t)(uint8_t)requant_i8(o.w, qs) << 24);
                else
                    *reinterpret_cast<float4 *>(out + off) = o;
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(AT_TMEM_COLS) : "memory");
    }
}

}  // namespace

// D = 64 and 0 < S <= 128 (the encoder's shapes); TPT_UNSUPPORTED otherwise.
int launch_attention_tc(tpt_cuda_ctx *ctx, const float *qkv, float *out, int B, int S, int H, int D, float scale,
                        int8_t *q, float qs) {
    if (D != AT_D || S <= 0 || S > AT_S || B <= 0 || H <= 0 || B > 65535 ||
        (((uintptr_t)qkv | (uintptr_t)out) & 15) || ((uintptr_t)q & 3) || ((3 * H * D) & 3))
        return TPT_UNSUPPORTED;
    static bool attr[64] = {};
    if (!attr[ctx->device & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_attention_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, AT_TC_SMEM);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "attention smem attribute");
        attr[ctx->device & 63] = true;
    }
    launch_pdl(k_attention_tc, dim3((unsigned)H, (unsigned)B), AT_THREADS, AT_TC_SMEM, ctx->stream, qkv, out, S, H, scale, q,
                                                                                           qs, ctx->d_flags);
    return after_launch(ctx, "attention_tc");
}

}  // namespace tpt
