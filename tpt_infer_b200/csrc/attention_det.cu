// attention_det.cu -- fused attention softmax(scale * Q K^T) V per (batch,
// head) with a fixed evaluation order, so that a CPU restatement reproduces it
// bit for bit (oracle: tpto_attention_det).
//
// Semantics: the composition MatMul -> Softmax -> MatMul of the encoder graph
// (crates/tpt-infer-ops/src/naive.rs:13-33 and :104-125) on each head. qkv is
// the packed projection output [B*S, 3*H*D] (Q | K | V along columns); the
// context is [B*S, H*D] (f32, or int8 at the next quantization point's scale).
// The reference has no attention operator (its runtime rejects rank-3/4
// MatMul, exec.rs:360-362), so this backend defines the arithmetic:
//   q'  = q * scale                                  (one rounding)
//   s_c = fmaf over d = 0 .. 63 in order of q'_d k_cd, from 0
//   m   = max over the S keys of s_c
//   e_c = exp_det(s_c - m) for c < S, 0 for the padding keys c >= S
//         (exp_det: Cody-Waite + Taylor, det_math.cuh)
//   sum : the 128 key slots c = t + 16 j (t = 0..15, j = 0..7) summed per t in
//         increasing j, then the 16 partial sums by the xor butterfly
//         p[t] + p[t ^ o], o = 8, 4, 2, 1
//   p_c = e_c * (1 / sum)                            (the reciprocal correctly rounded)
//   o_d = fmaf over the 128 key slots in order of p_c v_cd, from 0 (padding
//         keys have p = 0 and v = 0)
//
// Kernel: one CTA per (batch, head, block of RQ query rows), S <= 128, D = 64,
// 256 threads as 16 x 16 (ty, tx). Q (scaled), K and V are staged row-major in
// shared memory (row stride 68 floats: 16-byte rows, conflict-free float4
// reads); thread (ty, tx) computes the scores of query rows ty*RT + i
// (RT = RQ / 16) against keys tx + 16 j in registers (float4 over d), the
// softmax with half-warp shuffles, writes P row-major into the space of Q and
// K, and then the context rows ty*RT + i, columns 4 tx .. 4 tx + 3 (float4
// over keys), stored as coalesced 16-byte (or 4-byte int8) row segments.
// FP32 pipe bound: 4 S^2 D flops per head, all FFMA.
#include "common.cuh"

namespace tpt {
namespace {

constexpr int AD_D = 64, AD_S = 128, AD_T = 256;
constexpr int AD_LD = AD_D + 4;     // Q/K/V row stride (floats)
constexpr int AD_PLD = AD_S + 4;    // P row stride (floats)

template <int RQ>
struct AdSmem {
    static constexpr int Q = 0;                          // [RQ][AD_LD]
    static constexpr int K = RQ * AD_LD;                 // [AD_S][AD_LD]
    static constexpr int V = K + AD_S * AD_LD;           // [AD_S][AD_LD]
    static constexpr int P = 0;                          // [RQ][AD_PLD], over Q and K once the scores are done
    static constexpr int FLOATS = V + AD_S * AD_LD;
    static_assert(RQ * AD_PLD <= K + AD_S * AD_LD, "P must fit in the space of Q and K");
};

template <int RQ>
__global__ void __launch_bounds__(AD_T, 2) k_attention_det(const float *__restrict__ qkv, float *__restrict__ out,
                                                            int S, int H, float scale, int8_t *__restrict__ qout,
                                                            float qs) {
    constexpr int RT = RQ / 16;  // query rows per thread
    extern __shared__ __align__(16) float sm[];
    float *Qs = sm + AdSmem<RQ>::Q, *Ks = sm + AdSmem<RQ>::K, *Vs = sm + AdSmem<RQ>::V, *Ps = sm + AdSmem<RQ>::P;
    pdl_wait();
    pdl_trigger();
    const int h = blockIdx.x, b = blockIdx.y, r0 = blockIdx.z * RQ;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const size_t ld = (size_t)3 * H * AD_D;
    const float *base = qkv + (size_t)b * S * ld + (size_t)h * AD_D;

    // stage Q (rows r0 .. r0+RQ-1), K and V (all 128 key slots) with 16-byte
    // cp.async copies, all in flight at once; rows past S are zero-filled
    for (int e = tid; e < (RQ + 2 * AD_S) * 16; e += AD_T) {
        const int row = e >> 4, d4 = e & 15;
        const int part = row < RQ ? 0 : (row < RQ + AD_S ? 1 : 2);
        const int src = part == 0 ? r0 + row : (part == 1 ? row - RQ : row - RQ - AD_S);
        float *dst = (part == 0 ? Qs + row * AD_LD : (part == 1 ? Ks : Vs) + src * AD_LD) + 4 * d4;
        const bool ok = src < S;
        const float *g = ok ? base + (size_t)src * ld + (size_t)part * H * AD_D + 4 * d4 : base;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                     "l"(g), "r"(ok ? 16 : 0)
                     : "memory");
    }
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    // q' = q * scale, in place
    for (int e = tid; e < RQ * 16; e += AD_T) {
        float4 *p = reinterpret_cast<float4 *>(Qs + (e >> 4) * AD_LD) + (e & 15);
        const float4 v = *p;
        *p = make_float4(__fmul_rn(v.x, scale), __fmul_rn(v.y, scale), __fmul_rn(v.z, scale), __fmul_rn(v.w, scale));
    }
    __syncthreads();

    // scores: rows ty*RT + i, keys tx + 16 j, d in order
    float s[RT][8];
#pragma unroll
    for (int i = 0; i < RT; i++)
#pragma unroll
        for (int j = 0; j < 8; j++) s[i][j] = 0.0f;
#pragma unroll 1
    for (int d4 = 0; d4 < AD_D / 4; d4++) {
        float4 k[8];
#pragma unroll
        for (int j = 0; j < 8; j++) k[j] = *reinterpret_cast<const float4 *>(Ks + (tx + 16 * j) * AD_LD + 4 * d4);
#pragma unroll
        for (int i = 0; i < RT; i++) {
            const float4 q = *reinterpret_cast<const float4 *>(Qs + (ty * RT + i) * AD_LD + 4 * d4);
#pragma unroll
            for (int j = 0; j < 8; j++) {
                float a = s[i][j];
                a = __fmaf_rn(q.x, k[j].x, a);
                a = __fmaf_rn(q.y, k[j].y, a);
                a = __fmaf_rn(q.z, k[j].z, a);
                a = __fmaf_rn(q.w, k[j].w, a);
                s[i][j] = a;
            }
        }
    }
    __syncthreads();  // Q and K are dead: P goes over them

    // softmax of each row over the S keys (half-warp = the 16 threads of one ty)
#pragma unroll
    for (int i = 0; i < RT; i++) {
        float m = -__int_as_float(0x7f800000);
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (tx + 16 * j < S) m = fmaxf(m, s[i][j]);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float part = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float e = tx + 16 * j < S ? exp_det(__fsub_rn(s[i][j], m)) : 0.0f;
            s[i][j] = e;
            part = __fadd_rn(part, e);
        }
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, o));
        const float inv = __fdiv_rn(1.0f, part);
#pragma unroll
        for (int j = 0; j < 8; j++) Ps[(ty * RT + i) * AD_PLD + tx + 16 * j] = __fmul_rn(s[i][j], inv);
    }
    __syncthreads();

    // context: rows ty*RT + i, columns 4 tx .. 4 tx + 3, keys in order
    float o[RT][4];
#pragma unroll
    for (int i = 0; i < RT; i++)
#pragma unroll
        for (int e = 0; e < 4; e++) o[i][e] = 0.0f;
#pragma unroll 2
    for (int c4 = 0; c4 < AD_S / 4; c4++) {
        float4 v[4];
#pragma unroll
        for (int jj = 0; jj < 4; jj++) v[jj] = *reinterpret_cast<const float4 *>(Vs + (4 * c4 + jj) * AD_LD + 4 * tx);
#pragma unroll
        for (int i = 0; i < RT; i++) {
            const float4 p = *reinterpret_cast<const float4 *>(Ps + (ty * RT + i) * AD_PLD + 4 * c4);
            const float pv[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
            for (int jj = 0; jj < 4; jj++) {
                o[i][0] = __fmaf_rn(pv[jj], v[jj].x, o[i][0]);
                o[i][1] = __fmaf_rn(pv[jj], v[jj].y, o[i][1]);
                o[i][2] = __fmaf_rn(pv[jj], v[jj].z, o[i][2]);
                o[i][3] = __fmaf_rn(pv[jj], v[jj].w, o[i][3]);
            }
        }
    }
    const size_t ldo = (size_t)H * AD_D;
#pragma unroll
    for (int i = 0; i < RT; i++) {
        const int r = r0 + ty * RT + i;
        if (r >= S) continue;
        const size_t off = ((size_t)b * S + r) * ldo + (size_t)h * AD_D + 4 * tx;
        if (qout) {
            const uint32_t w = (uint32_t)(uint8_t)requant_i8(o[i][0], qs) |
                               ((uint32_t)(uint8_t)requant_i8(o[i][1], qs) << 8) |
                               ((uint32_t)(uint8_t)requant_i8(o[i][2], qs) << 16) |
                               ((uint32_t)(uint8_t)requant_i8(o[i][3], qs) << 24);
            *reinterpret_cast<uint32_t *>(qout + off) = w;
        } else {
            *reinterpret_cast<float4 *>(out + off) = make_float4(o[i][0], o[i][1], o[i][2], o[i][3]);
        }
    }
}

}  // namespace

int launch_attention_det(tpt_cuda_ctx *ctx, const float *qkv, float *out, int B, int S, int H, int D, float scale,
                         int8_t *q, float qs) {
    if (D != AD_D || S <= 0 || S > AD_S || B <= 0 || H <= 0 || B > 65535 || H > 65535 ||
        (((uintptr_t)qkv | (uintptr_t)out) & 15) || ((uintptr_t)q & 3))
        return TPT_UNSUPPORTED;
    // query rows per CTA: 128, or 64 / 32 when that many heads would leave SMs idle
    // (two CTAs fit per SM); the arithmetic per output is the same for every split
    const size_t heads = (size_t)B * H, slots = (size_t)ctx->sm_count * 2;
    const int rq = heads >= slots ? 128 : (heads * 2 >= slots ? 64 : 32);
    const dim3 grid((unsigned)H, (unsigned)B, (unsigned)((S + rq - 1) / rq));
    static bool attr[64][3] = {};
    const int ai = rq == 128 ? 0 : (rq == 64 ? 1 : 2);
    const size_t smem = (rq == 128 ? AdSmem<128>::FLOATS : rq == 64 ? AdSmem<64>::FLOATS : AdSmem<32>::FLOATS) *
                        sizeof(float);
    const void *fn = rq == 128 ? (const void *)k_attention_det<128>
                     : rq == 64 ? (const void *)k_attention_det<64>
                                : (const void *)k_attention_det<32>;
    if (!attr[ctx->device & 63][ai]) {
        cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "attention smem attribute");
        attr[ctx->device & 63][ai] = true;
    }
    if (rq == 128)
        launch_pdl(k_attention_det<128>, grid, AD_T, smem, ctx->stream, qkv, out, S, H, scale, q, qs);
    else if (rq == 64)
        launch_pdl(k_attention_det<64>, grid, AD_T, smem, ctx->stream, qkv, out, S, H, scale, q, qs);
    else
        launch_pdl(k_attention_det<32>, grid, AD_T, smem, ctx->stream, qkv, out, S, H, scale, q, qs);
    return after_launch(ctx, "attention");
}

}  // namespace tpt
