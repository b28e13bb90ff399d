// attention_i8.cu -- fused attention softmax(scale * Q K^T) V per (batch, head)
// with both products on the integer tensor cores (tcgen05.mma kind::i8, i32
// accumulators in tensor memory), exact and therefore restatable on the CPU
// bit for bit (oracle: tpto_attention_i8).
//
// Semantics: the composition MatMul -> Softmax -> MatMul of the encoder graph
// (crates/tpt-infer-ops/src/naive.rs:13-33 and :104-125) on each head; qkv is
// the packed projection output [B*S, 3*H*D] (Q | K | V along columns), the
// context [B*S, H*D] (f32, or int8 at the next quantization point's scale).
// The reference has no attention operator, so this backend defines the
// arithmetic, with f32-class accuracy (about 2^-22 of each row's largest
// value):
//
//   digits(x[0..n), amax): sc = amax * r127 (r127 = 1/127 rounded to f32),
//     inv = 1 / sc (correctly rounded; 0 when amax is 0), for each x:
//     u = x * inv; d0 = rint(u); r = (u - d0) * 128; d1 = rint(r);
//     r = (r - d1) * 128; d2 = rint(r)      (NaN -> 0; every step but the
//     first product exact), so x ~ (d0 + d1/128 + d2/16384) * sc
//   Q rows: x = q * scale, amax = max |x| over the row;  K rows likewise;
//   V columns: amax = max |v| over the keys of a head dimension;
//   T0 = sum_d a0 b0, T1 = sum_d (a0 b1 + a1 b0), T2 = sum_d (a0 b2 + a1 b1 + a2 b0)
//     (exact integers; the terms of order 3 and 4, below 2^-21, are dropped)
//   s = (T0 + (T1 * 2^-7 + T2 * 2^-14)) * (sc_q * sc_k),
//     as  t = T2 * 2^-14;  t = fmaf(T1, 2^-7, t);  t = T0 + t;  s = t * (sq * sk)
//   m = max over the S keys; e = exp_det(s - m) (0 for the padding keys);
//   the 128 key slots summed per quarter of 32 in order, then ((q0 + q1) + q2) + q3;
//   E digits with amax = 1 (u = 127 e: each row's largest e is exp(0) = 1);
//   U0, U1, U2 as T over the 128 key slots (E digits x V digits);
//   o = ((U0 + (U1 * 2^-7 + U2 * 2^-14)) * (sc_v * r127)) * (1 / sum)
//
// The three Q/K digit planes are packed two per 128-byte K-major row, so each
// sum is one or two K = 128 MMA sequences: QA = [a0 | a1], QB = [a2 | 0],
// KA = [b0 | 0], KB = [b1 | b0], KC = [b2 | b1]: T0 = QA.KA, T1 = QA.KB,
// T2 = QA.KC + QB.KA. E and V^T (keys along K) give one 128-byte row per
// plane: U0 = E0.V0, U1 = E0.V1 + E1.V0, U2 = E0.V2 + E1.V1 + E2.V0.
//
// One CTA per (batch, head), S <= 128, D = 64, 512 threads: every thread turns
// its share of Q, K (a warp per row) and V (a thread per 16 keys of one head
// dimension) into digit tiles (128B-swizzled, K-major); one thread issues the
// 16 score MMAs (M = N = 128) into three TMEM accumulators, the softmax reads
// them (thread = query row and a quarter of the keys) and writes the P digit
// tiles over Q and K; one thread issues the 24 context MMAs (N = 64); the
// context leaves through a shared staging tile as coalesced rows. Tensor
// memory (512 columns) is allocated only after the digit tiles are written, so
// a second CTA on the SM stages its head while the first one computes. Waits
// on the MMA commits are bounded; after a timeout the MMAs issued are drained
// (with the full bound) before tensor memory is freed.
#include "tc_common.cuh"

namespace tpt {
namespace {
using namespace tc;

constexpr int AI_D = 64, AI_S = 128, AI_T = 512;
constexpr uint32_t AI_TMEM_COLS = 512;                 // T0 [0,128), T1 [128,256), T2 [256,384); U0..U2 over [0,192)
constexpr uint32_t OFF_QA = 0, OFF_QB = 16384, OFF_KA = 32768, OFF_KB = 49152, OFF_KC = 65536;
constexpr uint32_t OFF_V0 = 81920, OFF_V1 = 90112, OFF_V2 = 98304;  // V^T digit tiles [64 rows x 128 keys]
constexpr uint32_t OFF_P0 = 0, OFF_P1 = 16384, OFF_P2 = 32768;     // over QA, QB, KA once the scores are done
constexpr int AI_OST = AI_D + 4;                                   // output staging row stride (floats)
constexpr float AI_R127 = 0.00787401572f;                          // 1/127 rounded to f32
constexpr int AI_SMEM = 106496 + 1024;

// byte (row, kb) of a 128B-swizzled K-major tile with 128-byte rows
__device__ __forceinline__ uint32_t swz(int row, int kb) {
    return (uint32_t)(row * 128 + ((((kb >> 4) ^ (row & 7)) << 4) | (kb & 15)));
}

__host__ __device__ constexpr uint32_t ai_idesc(int m, int n) {  // D s32, A s8, B s8, K-major
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}


// pack4 takes the low bytes of four words
__device__ __forceinline__ uint32_t pack4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
    return __byte_perm(__byte_perm(w0, w1, 0x0040), __byte_perm(w2, w3, 0x0040), 0x5410);
}

// The three digits of x (see the header) as their rounding sums' float bits:
// rounding by adding 1.5 * 2^23 (ties to even, as rintf, for |u| < 2^22; here
// |u| <= 127 and the residuals are in [-64, 64]) leaves the integer in the low
// mantissa bits, so the low byte of the bits is the digit's two's-complement
// byte (0x4B400000 has a zero low byte); NaN gives 0.
// Two values at a time (u = x * inv per half; nz from opaque_nz2, since u
// feeds adds).
__device__ __forceinline__ void digits3_bits_x2(float x0, float x1, float inv, uint64_t nz, uint32_t (&b0)[2],
                                                uint32_t (&b1)[2], uint32_t (&b2)[2]) {
    const uint64_t magic = splat2(12582912.0f), nmagic = splat2(-12582912.0f), neg1 = splat2(-1.0f),
                   s128 = splat2(128.0f);
    const uint64_t u = mulr2(f2pack(x0, x1), splat2(inv), nz);
    const uint64_t t0 = add2(u, magic);
    const uint64_t a = add2(t0, nmagic);
    const uint64_t r1 = mul2(fma2(a, neg1, u), s128);  // (u - a) * 128
    const uint64_t t1 = add2(r1, magic);
    const uint64_t c = add2(t1, nmagic);
    const uint64_t r2 = mul2(fma2(c, neg1, r1), s128);
    const uint64_t t2 = add2(r2, magic);
    float uu0, uu1, f0, f1;
    f2unpack(u, uu0, uu1);
    f2unpack(t0, f0, f1);
    b0[0] = __float_as_uint(f0), b0[1] = __float_as_uint(f1);
    f2unpack(t1, f0, f1);
    b1[0] = __float_as_uint(f0), b1[1] = __float_as_uint(f1);
    f2unpack(t2, f0, f1);
    b2[0] = __float_as_uint(f0), b2[1] = __float_as_uint(f1);
    if (uu0 != uu0) b0[0] = b1[0] = b2[0] = 0;
    if (uu1 != uu1) b0[1] = b1[1] = b2[1] = 0;
}


// t = T2 * 2^-14; t = fmaf(T1, 2^-7, t); T0 + t for two accumulator triples on
// paired operations. Each integer becomes a float by adding it to the bits of
// 1.5 * 2^23 and subtracting 1.5 * 2^23 (integer and FMA pipes, no conversion
// unit): exact, since every accumulator is below 2^22 in magnitude
// (|T| <= 64 (2 * 127 * 64 + 64 * 64) about 1.3e6, |U| <= 128 (2 * 127 * 64 +
// 64 * 64) about 2.6e6).
__device__ __forceinline__ uint64_t combine3_x2(uint32_t a0, uint32_t b0, uint32_t a1, uint32_t b1, uint32_t a2,
                                                uint32_t b2) {
    const uint64_t nmagic = splat2(-12582912.0f);
    auto i2f2 = [&](uint32_t x, uint32_t y) {
        return add2(f2pack(__int_as_float((int)x + 0x4B400000), __int_as_float((int)y + 0x4B400000)), nmagic);
    };
    uint64_t t = mul2(i2f2(a2, b2), splat2(0x1p-14f));
    t = fma2(i2f2(a1, b1), splat2(0x1p-7f), t);
    return add2(i2f2(a0, b0), t);
}

// 32 lanes x 8 consecutive 32-bit TMEM columns, load and store
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }


__global__ void __launch_bounds__(AI_T, 2)
    k_attention_i8(const float *__restrict__ qkv, float *__restrict__ out, int S, int H, float scale,
                   int8_t *__restrict__ qout, float qs, unsigned *gflags) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint64_t bars[3];  // scores done, context done, drain
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    __shared__ float red[2][4][AI_S];     // [max | sum][key quarter][row]
    __shared__ float qsc[AI_S], ksc[AI_S];  // amax * r127 of each Q and K row
    __shared__ float vmp[8][AI_D];          // per 16-key group column maxima of V
    __shared__ float vps[AI_D];             // amax_v * r127 * r127 of each head dimension

    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t *g = smem_raw + (base - raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.y, h = blockIdx.x;
    const int HD = H * AI_D, ld = 3 * HD;
    const float *src = qkv + (size_t)b * S * ld + h * AI_D;
    const uint32_t s_bar = smem_u32(&bars[0]), o_bar = smem_u32(&bars[1]), d_bar = smem_u32(&bars[2]);
    const uint64_t nz2 = opaque_nz2((uint32_t)S >> 31);  // S >= 0
    if (tid == 0) {
        abort_flag = 0;
        mbar_init(s_bar, 1);
        mbar_init(o_bar, 1);
        mbar_init(d_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    pdl_wait();  // the previous kernel's output (qkv) is complete from here on
    pdl_trigger();

    // ---- Q and K rows: half a warp per row (rows 2 warp + (lane >> 4) + 32 i), lane
    // % 16 = head dimensions 4 l .. 4 l + 3; all 8 loads of a lane are in flight
    // before the first use, and each plane's four digits leave as one word
    {
        constexpr int RPW = 2 * AI_S / (AI_T / 32) / 2;  // row pairs per warp: 8
        const int l16 = lane & 15, half = lane >> 4;
        float4 xs[RPW];
#pragma unroll
        for (int i = 0; i < RPW; i++) {
            const int rr = 2 * warp + half + (AI_T / 16) * i;
            const bool isq = rr < AI_S;
            const int r = isq ? rr : rr - AI_S;
            xs[i] = r < S ? __ldg(reinterpret_cast<const float4 *>(src + (size_t)r * ld + (isq ? 0 : HD)) + l16)
                          : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int i = 0; i < RPW; i++) {
            const int rr = 2 * warp + half + (AI_T / 16) * i;
            const bool isq = rr < AI_S;  // the same for both halves: 2 warp + half < 32 and the stride is 32
            const int r = isq ? rr : rr - AI_S;
            float4 x = xs[i];
            if (isq) x = make_float4(__fmul_rn(x.x, scale), __fmul_rn(x.y, scale), __fmul_rn(x.z, scale),
                                     __fmul_rn(x.w, scale));
            float am = fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w)));
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));  // within the half
            const float sc = __fmul_rn(am, AI_R127);
            const float inv = am > 0.0f ? __frcp_rn(sc) : 0.0f;
            uint32_t b0[4], b1[4], b2[4];
            {
                uint32_t p0[2], p1[2], p2[2];
                digits3_bits_x2(x.x, x.y, inv, nz2, p0, p1, p2);
                b0[0] = p0[0], b0[1] = p0[1], b1[0] = p1[0], b1[1] = p1[1], b2[0] = p2[0], b2[1] = p2[1];
                digits3_bits_x2(x.z, x.w, inv, nz2, p0, p1, p2);
                b0[2] = p0[0], b0[3] = p0[1], b1[2] = p1[0], b1[3] = p1[1], b2[2] = p2[0], b2[3] = p2[1];
            }
            const uint32_t d0 = pack4(b0[0], b0[1], b0[2], b0[3]), d1 = pack4(b1[0], b1[1], b1[2], b1[3]),
                           d2 = pack4(b2[0], b2[1], b2[2], b2[3]);
            const int kb = 4 * l16;
            if (isq) {  // QA = [a0 | a1], QB = [a2 | 0]
                *reinterpret_cast<uint32_t *>(g + OFF_QA + swz(r, kb)) = d0;
                *reinterpret_cast<uint32_t *>(g + OFF_QA + swz(r, 64 + kb)) = d1;
                *reinterpret_cast<uint32_t *>(g + OFF_QB + swz(r, kb)) = d2;
                *reinterpret_cast<uint32_t *>(g + OFF_QB + swz(r, 64 + kb)) = 0;
                if (l16 == 0) qsc[r] = sc;
            } else {    // KA = [b0 | 0], KB = [b1 | b0], KC = [b2 | b1]
                *reinterpret_cast<uint32_t *>(g + OFF_KA + swz(r, kb)) = d0;
                *reinterpret_cast<uint32_t *>(g + OFF_KA + swz(r, 64 + kb)) = 0;
                *reinterpret_cast<uint32_t *>(g + OFF_KB + swz(r, kb)) = d1;
                *reinterpret_cast<uint32_t *>(g + OFF_KB + swz(r, 64 + kb)) = d0;
                *reinterpret_cast<uint32_t *>(g + OFF_KC + swz(r, kb)) = d2;
                *reinterpret_cast<uint32_t *>(g + OFF_KC + swz(r, 64 + kb)) = d1;
                if (l16 == 0) ksc[r] = sc;
            }
        }
    }
    // ---- V: thread = head dimension d and 16 keys 16 kq .. 16 kq + 15
    {
        const int d = tid & (AI_D - 1), kq = tid >> 6;
        float v[16];
        float m = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const int c = 16 * kq + i;
            v[i] = c < S ? __ldg(src + (size_t)c * ld + 2 * HD + d) : 0.0f;
            m = fmaxf(m, fabsf(v[i]));
        }
        vmp[kq][d] = m;
        __syncthreads();
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++) amax = fmaxf(amax, vmp[j][d]);
        const float sc = __fmul_rn(amax, AI_R127);
        if (kq == 0) vps[d] = __fmul_rn(sc, AI_R127);
        const float inv = amax > 0.0f ? __frcp_rn(sc) : 0.0f;
        uint32_t w0[4], w1[4], w2[4];
#pragma unroll
        for (int i4 = 0; i4 < 4; i4++) {
            uint32_t x0[4], x1[4], x2[4];
#pragma unroll
            for (int k = 0; k < 4; k += 2) {
                uint32_t p0[2], p1[2], p2[2];
                digits3_bits_x2(v[4 * i4 + k], v[4 * i4 + k + 1], inv, nz2, p0, p1, p2);
                x0[k] = p0[0], x0[k + 1] = p0[1], x1[k] = p1[0], x1[k + 1] = p1[1], x2[k] = p2[0], x2[k + 1] = p2[1];
            }
            w0[i4] = pack4(x0[0], x0[1], x0[2], x0[3]);
            w1[i4] = pack4(x1[0], x1[1], x1[2], x1[3]);
            w2[i4] = pack4(x2[0], x2[1], x2[2], x2[3]);
        }
        const uint32_t o = swz(d, 16 * kq);  // V^T row d, keys 16 kq .. 16 kq + 15: one 16-byte chunk
        *reinterpret_cast<uint4 *>(g + OFF_V0 + o) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
        *reinterpret_cast<uint4 *>(g + OFF_V1 + o) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
        *reinterpret_cast<uint4 *>(g + OFF_V2 + o) = make_uint4(w2[0], w2[1], w2[2], w2[3]);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // st.shared -> the tensor core's reads
    __syncthreads();
    if (warp == 0) {  // tensor memory only now: a second CTA on this SM staged its head meanwhile
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(AI_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    volatile int *abort_p = &abort_flag;

    if (tid == 0) {  // scores: T0 = QA.KA, T1 = QA.KB, T2 = QA.KC + QB.KA (K = 128 each: 4 MMAs of K = 32)
        const uint32_t A[4] = {base + OFF_QA, base + OFF_QA, base + OFF_QA, base + OFF_QB};
        const uint32_t Bm[4] = {base + OFF_KA, base + OFF_KB, base + OFF_KC, base + OFF_KA};
        const uint32_t Dc[4] = {0u, 128u, 256u, 256u};
#pragma unroll
        for (int q = 0; q < 4; q++)
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
                tc_mma_i8(tmem + Dc[q], sw128_desc(A[q] + 32 * kk), sw128_desc(Bm[q] + 32 * kk), ai_idesc(128, 128),
                          (q == 3 || kk > 0) ? 1u : 0u);
        tc_commit(s_bar);
    }
    const int row = (warp & 3) * 32 + lane, qtr = warp >> 2;  // TMEM lane (query row); key / dimension quarter
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    bool ok = __syncthreads_and(mbar_wait(s_bar, 0, abort_p, gflags, true));
    if (ok) {
        tc_fence_after();
        // ---- softmax over this thread's 32 keys qtr*32 .. +31, combined with the other quarters.
        // Pass 1, 8 keys at a time: the scores from T0..T2, their max, the scores
        // written back over T0 (tcgen05.st) so that few registers stay live.
        const float sq = qsc[row];
        const int nvalid = S - qtr * 32;  // keys of this quarter below S
        float m = -__int_as_float(0x7f800000);
#pragma unroll
        for (int ch = 0; ch < 4; ch++) {
            const uint32_t col = (uint32_t)(qtr * 32 + ch * 8);
            uint32_t t0[8], t1[8], t2[8];
            tmem_ld8(lane_base + col, t0);
            tmem_ld8(lane_base + 128u + col, t1);
            tmem_ld8(lane_base + 256u + col, t2);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
                float sv0, sv1;
                f2unpack(mul2(combine3_x2(t0[j], t0[j + 1], t1[j], t1[j + 1], t2[j], t2[j + 1]),
                              mul2(splat2(sq), f2pack(ksc[col + j], ksc[col + j + 1]))),
                         sv0, sv1);
                if (ch * 8 + j < nvalid) m = fmaxf(m, sv0);
                if (ch * 8 + j + 1 < nvalid) m = fmaxf(m, sv1);
                t0[j] = __float_as_uint(sv0);
                t0[j + 1] = __float_as_uint(sv1);
            }
            tmem_st8(lane_base + col, t0);
        }
        tmem_wait_st();
        red[0][qtr][row] = m;
        __syncthreads();
        m = fmaxf(fmaxf(red[0][0][row], red[0][1][row]), fmaxf(red[0][2][row], red[0][3][row]));
        // Pass 2: e = exp_det(s - m) summed in key order; the digits of e (amax 1: the
        // row's largest e is exp(0) = 1; u = 127 e) into row `row`, keys qtr*32 .. +31,
        // two 16-byte chunks per plane; 1 / sum is applied to the context
        float sum = 0.0f;
#pragma unroll
        for (int hc = 0; hc < 2; hc++) {
            uint32_t w0[4], w1[4], w2[4];
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                const int k0 = hc * 16 + hh * 8;
                uint32_t sv8[8];
                tmem_ld8(lane_base + (uint32_t)(qtr * 32 + k0), sv8);
                tmem_wait_ld();
                uint32_t x0[8], x1[8], x2[8];
#pragma unroll
                for (int j = 0; j < 8; j += 2) {
                    // s - m <= 0 (m is the row's maximum) or NaN: exp_det's result without
                    // its x > 88 case, two keys per paired operation
                    float e0, e1;
                    exp_det_le0_x2(__fsub_rn(__uint_as_float(sv8[j]), m), __fsub_rn(__uint_as_float(sv8[j + 1]), m), e0,
                                   e1);
                    e0 = k0 + j < nvalid ? e0 : 0.0f;
                    e1 = k0 + j + 1 < nvalid ? e1 : 0.0f;
                    sum = __fadd_rn(sum, e0);
                    sum = __fadd_rn(sum, e1);
                    uint32_t q0[2], q1[2], q2[2];
                    digits3_bits_x2(e0, e1, 127.0f, nz2, q0, q1, q2);
                    x0[j] = q0[0], x0[j + 1] = q0[1];
                    x1[j] = q1[0], x1[j + 1] = q1[1];
                    x2[j] = q2[0], x2[j + 1] = q2[1];
                }
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    w0[2 * hh + c] = pack4(x0[4 * c], x0[4 * c + 1], x0[4 * c + 2], x0[4 * c + 3]);
                    w1[2 * hh + c] = pack4(x1[4 * c], x1[4 * c + 1], x1[4 * c + 2], x1[4 * c + 3]);
                    w2[2 * hh + c] = pack4(x2[4 * c], x2[4 * c + 1], x2[4 * c + 2], x2[4 * c + 3]);
                }
            }
            const uint32_t o = swz(row, 32 * qtr + 16 * hc);
            *reinterpret_cast<uint4 *>(g + OFF_P0 + o) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
            *reinterpret_cast<uint4 *>(g + OFF_P1 + o) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
            *reinterpret_cast<uint4 *>(g + OFF_P2 + o) = make_uint4(w2[0], w2[1], w2[2], w2[3]);
        }
        red[1][qtr][row] = sum;
        __syncthreads();
        sum = __fadd_rn(__fadd_rn(__fadd_rn(red[1][0][row], red[1][1][row]), red[1][2][row]), red[1][3][row]);
        const float rs = __fdiv_rn(1.0f, sum);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {  // context: U0 = P0.V0, U1 = P0.V1 + P1.V0, U2 = P0.V2 + P1.V1 + P2.V0 (N = 64)
            const uint32_t A[6] = {base + OFF_P0, base + OFF_P0, base + OFF_P1, base + OFF_P0, base + OFF_P1,
                                   base + OFF_P2};
            const uint32_t Bm[6] = {base + OFF_V0, base + OFF_V1, base + OFF_V0, base + OFF_V2, base + OFF_V1,
                                    base + OFF_V0};
            const uint32_t Dc[6] = {0u, 64u, 64u, 128u, 128u, 128u};
            const bool first[6] = {true, true, false, true, false, false};
#pragma unroll
            for (int q = 0; q < 6; q++)
#pragma unroll
                for (int kk = 0; kk < 4; kk++)
                    tc_mma_i8(tmem + Dc[q], sw128_desc(A[q] + 32 * kk), sw128_desc(Bm[q] + 32 * kk),
                              ai_idesc(128, 64), (!first[q] || kk > 0) ? 1u : 0u);
            tc_commit(o_bar);
        }
        ok = __syncthreads_and(mbar_wait(o_bar, 0, abort_p, gflags, true));
        if (ok) {
            tc_fence_after();
            // ---- context: thread (row, dims qtr*16 .. +15) -> staging [128][AI_OST] -> coalesced rows
            float *st = reinterpret_cast<float *>(g);  // over the E tiles (their MMAs are done)
#pragma unroll
            for (int ch = 0; ch < 2; ch++) {
                const uint32_t col = (uint32_t)(qtr * 16 + ch * 8);
                uint32_t u0[8], u1[8], u2[8];
                tmem_ld8(lane_base + col, u0);
                tmem_ld8(lane_base + 64u + col, u1);
                tmem_ld8(lane_base + 128u + col, u2);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 2; c++) {
                    float ov[4];
#pragma unroll
                    for (int e = 0; e < 4; e += 2) {
                        const int j = 4 * c + e;
                        f2unpack(mul2(mul2(combine3_x2(u0[j], u0[j + 1], u1[j], u1[j + 1], u2[j], u2[j + 1]),
                                           f2pack(vps[col + j], vps[col + j + 1])),
                                      splat2(rs)),
                                 ov[e], ov[e + 1]);
                    }
                    *reinterpret_cast<float4 *>(st + row * AI_OST + col + 4 * c) = make_float4(ov[0], ov[1], ov[2], ov[3]);
                }
            }
            __syncthreads();
            for (int i = tid; i < AI_S * (AI_D / 4); i += AI_T) {
                const int r = i >> 4, c4 = i & 15;
                if (r >= S) continue;
                const float4 o = *reinterpret_cast<const float4 *>(st + r * AI_OST + 4 * c4);
                const size_t off = ((size_t)b * S + r) * HD + h * AI_D + 4 * c4;
                if (qout) {  // the following QUANTIZE, fused: the f32 context is not written
                    int8_t q4[4];
                    const float ov[4] = {o.x, o.y, o.z, o.w};
                    if (requant_fast_ok(qs)) {
                        const float qrs = __frcp_rn(qs);
#pragma unroll
                        for (int e = 0; e < 4; e++) q4[e] = requant_i8_fast(ov[e], qs, qrs);
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; e++) q4[e] = requant_i8(ov[e], qs);
                    }
                    *reinterpret_cast<uint32_t *>(qout + off) = (uint32_t)(uint8_t)q4[0] |
                                                                ((uint32_t)(uint8_t)q4[1] << 8) |
                                                                ((uint32_t)(uint8_t)q4[2] << 16) |
                                                                ((uint32_t)(uint8_t)q4[3] << 24);
                }
                else
                    *reinterpret_cast<float4 *>(out + off) = o;
            }
        }
    }
    if (!ok && tid == 0) {  // a wait ran out: every MMA issued completes before tensor memory is freed
        tc_commit(d_bar);
        mbar_wait(d_bar, 0, abort_p, gflags, false);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(AI_TMEM_COLS) : "memory");
    }
}
}  // namespace
}  // namespace tpt

namespace tpt {

// D = 64 and 0 < S <= 128 (the encoder's shapes); TPT_UNSUPPORTED otherwise.
int launch_attention_i8(tpt_cuda_ctx *ctx, const float *qkv, float *out, int B, int S, int H, int D, float scale,
                        int8_t *q, float qs) {
    if (D != AI_D || S <= 0 || S > AI_S || B <= 0 || H <= 0 || B > 65535 || H > 65535 ||
        (((uintptr_t)qkv | (uintptr_t)out) & 15) || ((uintptr_t)q & 3))
        return TPT_UNSUPPORTED;
    static bool attr[64] = {};
    if (!attr[ctx->device & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_attention_i8, cudaFuncAttributeMaxDynamicSharedMemorySize, AI_SMEM);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "attention smem attribute");
        attr[ctx->device & 63] = true;
    }
    launch_pdl(k_attention_i8, dim3((unsigned)H, (unsigned)B), AI_T, AI_SMEM, ctx->stream, qkv, out, S, H, scale, q, qs,
               ctx->d_flags);
    return after_launch(ctx, "attention_i8");
}

}  // namespace tpt
