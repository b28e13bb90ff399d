// w4_gemv.cu -- INT4-weight GEMV for decode-like M <= 2: the nibble stream is
// moved by the TMA unit into a shared-memory ring and multiplied in integer
// arithmetic against activation digit planes.
//
// Reference semantics: dequantize_i4_symmetric_per_channel then the f32 matmul
// (crates/tpt-infer-quantize/src/dequant.rs:56-71, crates/tpt-infer-ops/src/
// avx512.rs:55-78): y[m,n] = sum_k x[m,k] * (q[n,k] * s[n]) + bias[n], then act.
//
// Numerics. Each activation row is split, per slice of SL = 256 k (K <= 4096)
// or 512 k (K <= 8192), into three signed 8-bit digit planes:
//   x_k = s (d0_k + d1_k / 128 + d2_k / 16384) (1 + e),  s = max_slice |x| / 127,
//   t = x * (127 / max|x|), d0 = rint(t), d1 = rint((t - d0) 128),
//   d2 = rint(((t - d0) 128 - d1) 128)
// (both residual steps are exact in f32), so each activation is represented to
// s / 32768 plus one f32 rounding. The weights enter as q + 8 in [0, 15]
// (unsigned bytes); the sums sum_k (q_k + 8) d_p,k are exact in i32 and start
// from -8 sum_k d_p,k, which removes the +8. Per row and slice the three plane
// sums A_p are combined as s (A0 + (A1 + A2 / 128) / 128) in f32 (A0 is below
// 2^24, exact). Against the f32 dot product this differs by the digit error (at
// most 8 * SL * s / 32768 per slice, far inside the 1e-3 x output-step bound)
// and f32 rounding. A slice holding a non-finite activation is computed as the
// f32 dot product instead, so inf and NaN propagate as in the reference.
//
// The integer products run on mma.sync m16n8k32 (u8 x s8 -> s32): one
// instruction multiplies 16 weight rows x 32 k by the 8 columns {3 digit planes
// per activation row, zeros}, i.e. 1.5 k multiply-adds of useful work, where a
// dp4a does 4. A weight word (8 nibbles, low first) becomes the two A-fragment
// words of its row with one LOP3 each (even k, odd k); the digit words are
// packed in the same even / odd order, so B's k order matches. The tcgen05 MMA
// is not used here: at N = 8 its per-instruction cost, not the arithmetic,
// would bound an HBM-speed GEMV, while the register-fragment MMA issues from
// the warps that decode the nibbles. Four independent accumulator sets keep
// four MMAs in flight per warp (their i32 sums are added exactly).
//
// Data movement. A CTA takes a contiguous run of 16-row groups; one producer
// thread streams them, one TMA tensor load per group (a 3-D view of the nibble
// matrix: 16 rows x 128 bytes per 128-byte column, 128B-swizzled, no
// multicast), into an S-stage ring guarded by full / empty mbarriers, the first
// S groups before the kernel's dependency wait (two CTAs fit one SM, so under
// programmatic dependent launch the next GEMV's first stages arrive while this
// one computes). The swizzle puts the 8 rows of a fragment load (8 rows x 4
// words per warp) in 32 distinct banks. Consumer warp w owns k slice w (SL k)
// of every row: per stage SL / 32 MMAs, then the plane sums are combined and the
// row's slice sum goes to a shared buffer; the buffered groups are combined
// (slice sums added in slice order, so the result does not depend on the
// launch shape, then scale, bias, act) once per P groups, normally once per
// CTA. All waits are bounded.
#include "ring.cuh"

namespace tpt {

namespace {
using namespace tc;
using namespace ring;

constexpr int WG_MAX_KW = 16;  // consumer warps: K <= 16 x 512
constexpr int WG_PART_BUDGET = 12 * 1024;
constexpr int WG_SMEM_PAIR = 112 * 1024;  // two CTAs per SM: the next launch's CTA streams beside this one
constexpr int WG_SMEM_MAX = 200 * 1024;
constexpr int WG_MAX_THREADS = 32 * (WG_MAX_KW + 1);

// D += A (16 x 32, u8, row) * B (32 x 8, s8, col), s32 accumulate. Not
// volatile: a pure function of its registers, so the compiler may hoist the
// fragment loads of later k-steps above it.
__device__ __forceinline__ void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Digits of one warp's slice [kslice, kslice + 32 CH) for activation rows
// 0..MM-1 (rows >= M read as zero): lane c splits k [kslice + CH c, +CH) and
// writes its words to tab[(i * 3 + p) * 32 + c][CH / 4]; every lane gets the
// slice scale sx[i] (NaN when the slice holds a non-finite activation) and
// corr[i][p] = -8 sum_k d_p,k over the slice.
template <int MM, int CH>
__device__ __forceinline__ void split_slice(const float *__restrict__ X, int M, int K, int kslice, int lane,
                                            uint32_t *tab, float (&sx)[MM], int (&corr)[MM][3]) {
#pragma unroll
    for (int i = 0; i < MM; i++) {
        const int kb = kslice + CH * lane;
        float xv[CH];
#pragma unroll
        for (int j = 0; j < CH; j += 4) {
            float4 t = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if (i < M && kb < K) t = __ldg(reinterpret_cast<const float4 *>(X + (size_t)i * K + kb + j));
            xv[j] = t.x;
            xv[j + 1] = t.y;
            xv[j + 2] = t.z;
            xv[j + 3] = t.w;
        }
        float amax = 0.0f;
        bool fin = true;
#pragma unroll
        for (int j = 0; j < CH; j++) {
            const float a = fabsf(xv[j]);
            fin = fin && a <= 3.402823466e38f;  // false for inf and NaN
            amax = fmaxf(amax, a);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        fin = __all_sync(0xffffffffu, fin);
        const float s = __fdiv_rn(amax, 127.0f), inv = __fdiv_rn(127.0f, amax);
        const bool live = fin && s > 0.0f && inv <= 3.402823466e38f;
        sx[i] = !fin ? __int_as_float(0x7fc00000) : live ? s : 0.0f;
        // Rounding by an addend of 1.5 * 2^23: t + 1.5 * 2^23 lands in
        // [2^23, 2^24), whose ulp is 1, so it rounds t to the nearest integer
        // (ties to even, as rint), its low mantissa byte is that integer mod
        // 256 (the digit as a signed byte), and subtracting the addend back
        // gives rint(t) exactly.
        constexpr float RND = 12582912.0f;
        uint32_t bits[3][CH];
#pragma unroll
        for (int j = 0; j < CH; j++) {
            const float t = live ? xv[j] * inv : 0.0f;
            const float f0 = t + RND;
            const float r1 = (t - (f0 - RND)) * 128.0f;
            const float f1 = r1 + RND;
            const float f2 = (r1 - (f1 - RND)) * 128.0f + RND;
            bits[0][j] = __float_as_uint(f0);
            bits[1][j] = __float_as_uint(f1);
            bits[2][j] = __float_as_uint(f2);
        }
        // chunk word 2q (+1 for odd): the digits of k = 8q + 2bb (+1), bb = 0..3
#pragma unroll
        for (int p = 0; p < 3; p++) {
            uint32_t wd[CH / 4];
            int sum = 0;
#pragma unroll
            for (int wi = 0; wi < CH / 4; wi++) {
                const int j0 = 8 * (wi >> 1) + (wi & 1);
                const uint32_t lo = __byte_perm(bits[p][j0], bits[p][j0 + 2], 0x0040);
                const uint32_t hi = __byte_perm(bits[p][j0 + 4], bits[p][j0 + 6], 0x0040);
                wd[wi] = __byte_perm(lo, hi, 0x5410);
                sum = __dp4a((int)wd[wi], 0x01010101, sum);
            }
#pragma unroll
            for (int wi = 0; wi < CH / 4; wi++) tab[((i * 3 + p) * 32 + lane) * (CH / 4) + wi] = wd[wi];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
            corr[i][p] = -8 * sum;
        }
    }
}

// CH = k per lane (8 or 16): a consumer warp's slice is 32 CH k, CH MMA k-steps.
template <int MM, int CH>
__global__ void __launch_bounds__(WG_MAX_THREADS, 1)
    k_w4_gemv_tma(const __grid_constant__ CUtensorMap tmW, const float *__restrict__ X,
                  const float *__restrict__ scales, const float *__restrict__ bias, int M, int N, int K, int act,
                  float *__restrict__ Y, int S, int P, unsigned *gflags) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int abort_flag;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int SL = 32 * CH;           // k per consumer warp
    const int KW = (K + SL - 1) / SL;     // consumer warps; warp KW is the producer
    const uint32_t stage_bytes = (uint32_t)K * 8u;   // 16 rows x K/2 bytes
    const int groups = (N + WG_ROWS - 1) / WG_ROWS;
    const int g0 = (int)((long long)blockIdx.x * groups / gridDim.x);
    const int g1 = (int)((long long)(blockIdx.x + 1) * groups / gridDim.x);
    const uint32_t raw = smem_u32(smem), ring = (raw + 1023u) & ~1023u;  // 128B swizzle: 1 KB aligned
    // per consumer warp: digit words [MM][3 planes][32 chunks][4 words]; the
    // same bytes later hold the slice sums part[P][MM][KW][16]
    uint32_t *tab = reinterpret_cast<uint32_t *>(smem + (ring - raw) + (size_t)S * stage_bytes);
    float *part = reinterpret_cast<float *>(tab);
    const uint32_t bars = smem_u32(tab + max(KW * MM * 3 * 32 * (CH / 4), P * MM * KW * WG_ROWS));
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (S + s); };

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), (uint32_t)KW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    }
    __syncthreads();
    volatile int *abort_p = &abort_flag;

    if (warp == KW) {
        if (lane == 0) produce(tmW, ring, stage_bytes, bars, S, g0, g1, abort_p, gflags);
        return;
    }
    if (warp > KW) return;
    pdl_wait();  // X (the previous kernel's output) is complete from here on
    pdl_trigger();

    // ---------------- consumers: warp = k slice ----------------
    const int ncons = KW * 32;
    const int gq = lane >> 2, tq = lane & 3;  // MMA fragment group / thread in group
    // Fragment row g is weight row pr = 2 (g & 3) + (g >> 2) (and pr + 8), and
    // MMA k positions 4 tq.. / 16 + 4 tq.. of k-step j hold the 8 consecutive k
    // 64 (j / 2) + 16 tq + 8 (j % 2) (identically in both operands, so the sums
    // are unchanged): a lane's nibbles of a k-step pair are one 8-byte load and
    // a half-warp's rows differ in swizzle bits 1-2 (conflict-free).
    const int pr = ((gq & 3) << 1) | (gq >> 2);
    const int kslice = warp * SL;
    const int ksteps = min(SL, K - kslice) / 32;
    uint32_t *mytab = tab + warp * MM * 3 * 32 * (CH / 4);
    float sx[MM];  // slice scale (NaN: the slice holds a non-finite activation)
    int corr[MM][3];
    split_slice<MM, CH>(X, M, K, kslice, lane, mytab, sx, corr);
    __syncwarp();
    // B fragments of the CH k-steps: column gq = (activation row, plane) or
    // zero; k-step j, word t of B = the 8 k at 32 j + 8 t: chunk (32 j + 8 t) / CH,
    // quad ((32 j + 8 t) % CH) / 8 (even, odd word)
    uint32_t bf[CH][2];
    const int bi = gq / 3, bp = gq - 3 * (gq / 3);
#pragma unroll
    for (int j = 0; j < CH; j++) {
        bf[j][0] = bf[j][1] = 0u;
        if (gq < 3 * MM) {
            const int k8 = 64 * (j >> 1) + 16 * tq + 8 * (j & 1);
            const uint32_t *src = mytab + ((bi * 3 + bp) * 32 + k8 / CH) * (CH / 4) + 2 * ((k8 % CH) / 8);
            bf[j][0] = src[0];
            bf[j][1] = src[1];
        }
    }
    // accumulator init: column 2 tq + e holds -8 sum_k d of its (row, plane)
    int cinit[2];
#pragma unroll
    for (int e = 0; e < 2; e++) {
        const int col = 2 * tq + e;
        int v = 0;
#pragma unroll
        for (int i = 0; i < MM; i++)
#pragma unroll
            for (int p = 0; p < 3; p++)
                if (col == 3 * i + p) v = corr[i][p];
        cinit[e] = v;
    }
    const bool slow = isnan(sx[0]) || (MM > 1 && isnan(sx[MM - 1]));
    // When one flush covers the CTA's run and every output has a thread, each
    // thread's channel scale and bias are loaded now, off the flush's path.
    const bool one_flush = P >= g1 - g0 && (g1 - g0) * WG_ROWS * MM <= ncons;
    float my_sc = 0.0f, my_bi = 0.0f;
    if (one_flush) {
        const int idx = (int)threadIdx.x, n = (g0 + idx / (WG_ROWS * MM)) * WG_ROWS + idx % WG_ROWS;
        if (idx < (g1 - g0) * WG_ROWS * MM && n < N) {
            my_sc = __ldg(scales + n);
            if (bias) my_bi = __ldg(bias + n);
        }
    }
    bar_sync(1, ncons);  // every warp has its B fragments: the table becomes part

    // Row sums are buffered per group in part[P][MM][KW][16] and combined P
    // groups at a time (all scale / bias loads of a flush in flight together,
    // no per-group barrier).
    int s = 0, gl = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int g = g0; g < g1; g++) {
        if (ok) ok = mbar_wait(full_bar(s), ph, abort_p, gflags, true);
        // four independent accumulator sets (k-step j -> set j % 4) keep four
        // MMAs in flight; their i32 sums are added exactly afterwards
        int d[4] = {cinit[0], cinit[1], cinit[0], cinit[1]};
        int e[3][4] = {};
        const uint32_t base = ring + (uint32_t)s * stage_bytes;
        // plain loads (ordered after the barrier wait by its memory clobber),
        // free to be issued all at once ahead of the MMAs
        const uint32_t *stg = reinterpret_cast<const uint32_t *>(smem + (base - raw));
        const uint2 *stg2 = reinterpret_cast<const uint2 *>(stg);
        uint2 r0 = make_uint2(0u, 0u), r1 = make_uint2(0u, 0u);
        if (ok) {
#pragma unroll
            for (int j = 0; j < CH; j++) {
                if (j < ksteps) {
                    if ((j & 1) == 0) {  // the nibbles of k-steps j and j + 1, rows pr and pr + 8
                        const uint32_t o = stage_off(pr, (uint32_t)(kslice >> 1) + 16u * j + 8u * tq) >> 3;
                        r0 = stg2[o];
                        r1 = stg2[o + 128u];
                    }
                    const uint32_t w0 = (j & 1) ? r0.y : r0.x, w1 = (j & 1) ? r1.y : r1.x;
                    uint32_t a[4];
                    a[0] = (w0 ^ 0x88888888u) & 0x0F0F0F0Fu;          // row pr, even k: q + 8
                    a[1] = (w1 ^ 0x88888888u) & 0x0F0F0F0Fu;          // row pr + 8, even k
                    a[2] = ((w0 >> 4) ^ 0x08080808u) & 0x0F0F0F0Fu;   // row pr, odd k
                    a[3] = ((w1 >> 4) ^ 0x08080808u) & 0x0F0F0F0Fu;   // row pr + 8, odd k
                    if (j % 4 == 0)
                        mma_u8s8(d, a, bf[j][0], bf[j][1]);
                    else
                        mma_u8s8(e[j % 4 - 1], a, bf[j][0], bf[j][1]);
                }
            }
#pragma unroll
            for (int c = 0; c < 4; c++) d[c] += e[0][c] + e[1][c] + e[2][c];
        }
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(empty_bar(s));
        // d: rows pr (d0, d1) and pr + 8 (d2, d3), columns 2 tq, 2 tq + 1.
        // Activation row 0 = columns 0..2 (tq 0: A0 A1; tq 1: A2 in d0 / d2),
        // row 1 = columns 3..5 (tq 1: A0 in d1 / d3; tq 2: A1 A2).
        const int nx0 = __shfl_down_sync(0xffffffffu, d[0], 1), nx2 = __shfl_down_sync(0xffffffffu, d[2], 1);
        const int px1 = __shfl_up_sync(0xffffffffu, d[1], 1), px3 = __shfl_up_sync(0xffffffffu, d[3], 1);
        float v[2] = {0.0f, 0.0f};
        int vi = -1;
        if (tq == 0) {
            vi = 0;
            v[0] = sx[0] * fmaf(fmaf((float)nx0, 0.0078125f, (float)d[1]), 0.0078125f, (float)d[0]);
            v[1] = sx[0] * fmaf(fmaf((float)nx2, 0.0078125f, (float)d[3]), 0.0078125f, (float)d[2]);
        } else if (MM > 1 && tq == 2) {
            vi = 1;
            v[0] = sx[MM - 1] * fmaf(fmaf((float)d[1], 0.0078125f, (float)d[0]), 0.0078125f, (float)px1);
            v[1] = sx[MM - 1] * fmaf(fmaf((float)d[3], 0.0078125f, (float)d[2]), 0.0078125f, (float)px3);
        }
        if (slow && vi >= 0 && isnan(sx[vi])) {  // non-finite activations: the slice's f32 dot product
#pragma unroll
            for (int h = 0; h < 2; h++) {
                float acc = 0.0f;
                if (vi < M && ok)
                    for (int kk = 0; kk < ksteps * 32; kk++) {
                        const uint32_t wd = stg[stage_off(pr + 8 * h, (uint32_t)(kslice >> 1) + 4u * (kk >> 3)) >> 2];
                        const int nb = (int)((wd >> (4 * (kk & 7))) & 0xFu);
                        acc = fmaf(__ldg(X + (size_t)vi * K + kslice + kk), (float)(nb - ((nb & 8) << 1)), acc);
                    }
                v[h] = acc;
            }
        }
        if (vi >= 0) {
            float *dst = part + ((gl * MM + vi) * KW + warp) * WG_ROWS;
            dst[pr] = v[0];
            dst[pr + 8] = v[1];
        }
        if (++s == S) {
            s = 0;
            ph ^= 1u;
        }
        if (++gl == P || g + 1 == g1) {  // flush: combine the buffered groups
            ok = bar_and(1, ncons, ok);   // every consumer's sums are in part
            if (ok) {
                const int gb = g + 1 - gl;  // first buffered group
                for (int idx = (int)threadIdx.x; idx < gl * WG_ROWS * MM; idx += ncons) {
                    const int r = idx % WG_ROWS, i = (idx / WG_ROWS) % MM, gi = idx / (WG_ROWS * MM);
                    const int n = (gb + gi) * WG_ROWS + r;
                    if (n >= N || i >= M) continue;
                    float acc = 0.0f;
                    for (int sl = 0; sl < KW; sl++) acc += part[((gi * MM + i) * KW + sl) * WG_ROWS + r];
                    float y = acc * (one_flush ? my_sc : __ldg(scales + n));
                    if (bias) y += one_flush ? my_bi : __ldg(bias + n);
                    Y[(size_t)i * N + n] = apply_act(y, act);
                }
            }
            bar_sync(1, ncons);  // part is free again
            gl = 0;
        }
    }
}

// Small batches (3 <= M <= MM, MM = 4 or 8; K <= 4096, CH = 8): the same
// ring, digit split and weight fragments, with T = ceil(3 MM / 8) MMA column
// tiles per k-step (column 3 i + p = plane p of activation row i). The plane
// sums go through a per-warp shared scratch [16 rows][8 T columns] and each
// lane combines (row, activation row) pairs.
template <int MM>
__global__ void __launch_bounds__(WG_MAX_THREADS, 1)
    k_w4_small(const __grid_constant__ CUtensorMap tmW, const float *__restrict__ X, const float *__restrict__ scales,
               const float *__restrict__ bias, int M, int N, int K, int act, float *__restrict__ Y, int S, int P,
               unsigned *gflags) {
    constexpr int CH = 8, SL = 32 * CH, T = (3 * MM + 7) / 8, SC = 8 * T;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int abort_flag;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int KW = (K + SL - 1) / SL;  // consumer warps; warp KW is the producer
    const uint32_t stage_bytes = (uint32_t)K * 8u;
    const int groups = (N + WG_ROWS - 1) / WG_ROWS;
    const int g0 = (int)((long long)blockIdx.x * groups / gridDim.x);
    const int g1 = (int)((long long)(blockIdx.x + 1) * groups / gridDim.x);
    const uint32_t raw = smem_u32(smem), ring = (raw + 1023u) & ~1023u;
    // digit table [KW][MM][3][32][CH/4] words; afterwards the same bytes hold
    // part[P][MM][KW][16] and the per-warp scratch [KW][16][SC]
    uint32_t *tab = reinterpret_cast<uint32_t *>(smem + (ring - raw) + (size_t)S * stage_bytes);
    float *part = reinterpret_cast<float *>(tab);
    int *scr = reinterpret_cast<int *>(part + P * MM * KW * WG_ROWS);
    const uint32_t bars = smem_u32(tab + max(KW * MM * 3 * 32 * (CH / 4), P * MM * KW * WG_ROWS + KW * 16 * SC));
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (S + s); };

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < S; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), (uint32_t)KW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    }
    __syncthreads();
    volatile int *abort_p = &abort_flag;
    if (warp == KW) {
        if (lane == 0) produce(tmW, ring, stage_bytes, bars, S, g0, g1, abort_p, gflags);
        return;
    }
    if (warp > KW) return;
    pdl_wait();  // X (the previous kernel's output) is complete from here on
    pdl_trigger();

    const int ncons = KW * 32;
    const int gq = lane >> 2, tq = lane & 3;
    const int pr = ((gq & 3) << 1) | (gq >> 2);  // weight row of fragment row gq (see the GEMV)
    const int kslice = warp * SL;
    const int ksteps = min(SL, K - kslice) / 32;
    uint32_t *mytab = tab + warp * MM * 3 * 32 * (CH / 4);
    float sx[MM];
    int corr[MM][3];
    split_slice<MM, CH>(X, M, K, kslice, lane, mytab, sx, corr);
    __syncwarp();
    // B fragments: tile tt, column gq -> c = 8 tt + gq = (row c / 3, plane c % 3)
    uint32_t bf[T][CH][2];
#pragma unroll
    for (int tt = 0; tt < T; tt++) {
        const int c = 8 * tt + gq;
#pragma unroll
        for (int j = 0; j < CH; j++) {
            bf[tt][j][0] = bf[tt][j][1] = 0u;
            if (c < 3 * MM) {
                const int k8 = 64 * (j >> 1) + 16 * tq + 8 * (j & 1);
                const uint32_t *src = mytab + (c * 32 + k8 / CH) * (CH / 4) + 2 * ((k8 % CH) / 8);
                bf[tt][j][0] = src[0];
                bf[tt][j][1] = src[1];
            }
        }
    }
    int cinit[T][2];
#pragma unroll
    for (int tt = 0; tt < T; tt++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int c = 8 * tt + 2 * tq + e;
            int v = 0;
#pragma unroll
            for (int i = 0; i < MM; i++)
#pragma unroll
                for (int p = 0; p < 3; p++)
                    if (c == 3 * i + p) v = corr[i][p];
            cinit[tt][e] = v;
        }
    bool slow = false;
#pragma unroll
    for (int i = 0; i < MM; i++) slow = slow || isnan(sx[i]);
    bar_sync(1, ncons);  // every warp has its B fragments: the table becomes part + scratch
    int *mysc = scr + warp * 16 * SC;

    int s = 0, gl = 0;
    uint32_t ph = 0;
    bool ok = true;
    for (int g = g0; g < g1; g++) {
        if (ok) ok = mbar_wait(full_bar(s), ph, abort_p, gflags, true);
        int d[T][4];
#pragma unroll
        for (int tt = 0; tt < T; tt++) {
            d[tt][0] = d[tt][2] = cinit[tt][0];
            d[tt][1] = d[tt][3] = cinit[tt][1];
        }
        const uint32_t base = ring + (uint32_t)s * stage_bytes;
        const uint32_t *stg = reinterpret_cast<const uint32_t *>(smem + (base - raw));
        const uint2 *stg2 = reinterpret_cast<const uint2 *>(stg);
        uint2 r0 = make_uint2(0u, 0u), r1 = make_uint2(0u, 0u);
        if (ok) {
#pragma unroll
            for (int j = 0; j < CH; j++) {
                if (j < ksteps) {
                    if ((j & 1) == 0) {  // the nibbles of k-steps j and j + 1, rows pr and pr + 8
                        const uint32_t o = stage_off(pr, (uint32_t)(kslice >> 1) + 16u * j + 8u * tq) >> 3;
                        r0 = stg2[o];
                        r1 = stg2[o + 128u];
                    }
                    const uint32_t w0 = (j & 1) ? r0.y : r0.x, w1 = (j & 1) ? r1.y : r1.x;
                    uint32_t a[4];
                    a[0] = (w0 ^ 0x88888888u) & 0x0F0F0F0Fu;
                    a[1] = (w1 ^ 0x88888888u) & 0x0F0F0F0Fu;
                    a[2] = ((w0 >> 4) ^ 0x08080808u) & 0x0F0F0F0Fu;
                    a[3] = ((w1 >> 4) ^ 0x08080808u) & 0x0F0F0F0Fu;
#pragma unroll
                    for (int tt = 0; tt < T; tt++) mma_u8s8(d[tt], a, bf[tt][j][0], bf[tt][j][1]);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(empty_bar(s));
        // plane sums -> scratch [row][column]
#pragma unroll
        for (int tt = 0; tt < T; tt++) {
            const int c = 8 * tt + 2 * tq;
            mysc[pr * SC + c] = d[tt][0];
            mysc[pr * SC + c + 1] = d[tt][1];
            mysc[(pr + 8) * SC + c] = d[tt][2];
            mysc[(pr + 8) * SC + c + 1] = d[tt][3];
        }
        __syncwarp();
        // lane -> (weight row r = lane % 16, activation row i = 2 u + lane / 16)
#pragma unroll
        for (int u = 0; u < MM / 2; u++) {
            const int r = lane & 15, i = 2 * u + (lane >> 4);
            const float si = (lane >> 4) ? sx[2 * u + 1] : sx[2 * u];
            const int *row = mysc + r * SC + 3 * i;
            float v = si * fmaf(fmaf((float)row[2], 0.0078125f, (float)row[1]), 0.0078125f, (float)row[0]);
            if (slow && isnan(si)) {  // non-finite activations: the slice's f32 dot product
                float acc = 0.0f;
                if (i < M && ok)
                    for (int kk = 0; kk < ksteps * 32; kk++) {
                        const uint32_t wd = stg[stage_off(r, (uint32_t)(kslice >> 1) + 4u * (kk >> 3)) >> 2];
                        const int nb = (int)((wd >> (4 * (kk & 7))) & 0xFu);
                        acc = fmaf(__ldg(X + (size_t)i * K + kslice + kk), (float)(nb - ((nb & 8) << 1)), acc);
                    }
                v = acc;
            }
            part[((gl * MM + i) * KW + warp) * WG_ROWS + r] = v;
        }
        __syncwarp();  // the scratch is read before the next stage overwrites it
        if (++s == S) {
            s = 0;
            ph ^= 1u;
        }
        if (++gl == P || g + 1 == g1) {  // flush: combine the buffered groups
            ok = bar_and(1, ncons, ok);
            if (ok) {
                const int gb = g + 1 - gl;
                for (int idx = (int)threadIdx.x; idx < gl * WG_ROWS * MM; idx += ncons) {
                    const int r = idx % WG_ROWS, i = (idx / WG_ROWS) % MM, gi = idx / (WG_ROWS * MM);
                    const int n = (gb + gi) * WG_ROWS + r;
                    if (n >= N || i >= M) continue;
                    float acc = 0.0f;
                    for (int sl = 0; sl < KW; sl++) acc += part[((gi * MM + i) * KW + sl) * WG_ROWS + r];
                    float y = acc * __ldg(scales + n);
                    if (bias) y += __ldg(bias + n);
                    Y[(size_t)i * N + n] = apply_act(y, act);
                }
            }
            bar_sync(1, ncons);
            gl = 0;
        }
    }
}

template <int MM>
int launch_small(tpt_cuda_ctx *ctx, const CUtensorMap &tw, const float *x, const float *scales, const float *bias,
                 int act, float *y, int m, int n, int k, int S, int P, size_t smem) {
    static bool attr_done[64] = {};
    auto kfn = k_w4_small<MM>;
    const int dev = ctx->device & 63;
    if (!attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, WG_SMEM_MAX + 1024);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "w4_small smem attribute");
        attr_done[dev] = true;
    }
    const int kw = (k + 255) / 256, groups = (n + WG_ROWS - 1) / WG_ROWS;
    const unsigned grid = (unsigned)(groups < ctx->sm_count ? groups : ctx->sm_count);
    launch_pdl(kfn, grid, 32 * (kw + 1), smem, ctx->stream, tw, x, scales, bias, m, n, k, act, y, S, P, ctx->d_flags);
    return after_launch(ctx, "w4_small");
}

template <int MM, int CH>
int launch_one(tpt_cuda_ctx *ctx, const CUtensorMap &tw, const float *x, const float *scales, const float *bias,
               int act, float *y, int n, int k, int S, int P, size_t smem) {
    static bool attr_done[64] = {};
    auto kfn = k_w4_gemv_tma<MM, CH>;
    const int dev = ctx->device & 63;
    if (!attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, WG_SMEM_MAX + 1024);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "w4_gemv smem attribute");
        attr_done[dev] = true;
    }
    const int kw = (k + 32 * CH - 1) / (32 * CH), groups = (n + WG_ROWS - 1) / WG_ROWS;
    const unsigned grid = (unsigned)(groups < ctx->sm_count ? groups : ctx->sm_count);  // one CTA per SM
    launch_pdl(kfn, grid, 32 * (kw + 1), smem, ctx->stream, tw, x, scales, bias, MM, n, k, act, y, S, P, ctx->d_flags);
    return after_launch(ctx, "w4_gemv_tma");
}

}  // namespace

// M <= 2, K % 256 == 0, K <= 8192, x 16-byte aligned; returns handled = false
// otherwise.
int launch_w4_gemv_tma(tpt_cuda_ctx *ctx, const float *x, size_t m, const tpt_cuda_weights *w, const float *bias,
                       int act, float *y, bool *handled) {
    *handled = false;
    const size_t n = w->n, k = w->k;
    if (m == 0 || m > 2 || k % 256 != 0 || k > (size_t)WG_MAX_KW * 512 || n > INT32_MAX) return TPT_OK;
    if (((uintptr_t)x & 15) != 0) return TPT_OK;
    CUtensorMap tw;
    if (!make_tmap_rows3d(&tw, w->data, n, k / 2)) return TPT_OK;
    // slices of 256 k (16 consumer warps at K = 4096) while they fit, else 512
    const int ch = k <= (size_t)WG_MAX_KW * 256 ? 8 : 16;
    const int kw = (int)((k + 32 * ch - 1) / (32 * ch));
    const int MM = (int)m;
    const size_t stage = WG_ROWS * (k / 2), table = (size_t)kw * MM * 3 * 32 * ch;
    // groups buffered between flushes: all of a CTA's run when they fit
    const size_t per_group = (size_t)MM * kw * WG_ROWS * 4;
    const size_t groups = (n + WG_ROWS - 1) / WG_ROWS;
    const size_t ctas = groups < (size_t)ctx->sm_count ? groups : (size_t)ctx->sm_count;
    const size_t run = (groups + ctas - 1) / ctas;
    const int P = (int)(run < WG_PART_BUDGET / per_group ? run : WG_PART_BUDGET / per_group);
    const size_t shared = table > (size_t)P * per_group ? table : (size_t)P * per_group;  // table, then part
    // two CTAs per SM when three stages fit beside each other, else one
    size_t budget = WG_SMEM_PAIR - shared - 1024 - 128;
    if (budget / stage < 3) budget = WG_SMEM_MAX - shared - 1024 - 128;
    const int S = (int)(budget / stage < 8 ? budget / stage : 8);
    if (S < 2) return TPT_OK;
    const size_t smem = 1024 + (size_t)S * stage + shared + (size_t)2 * S * 8;
    *handled = true;
    if (ch == 8)
        return MM == 1 ? launch_one<1, 8>(ctx, tw, x, w->scales, bias, act, y, (int)n, (int)k, S, P, smem)
                       : launch_one<2, 8>(ctx, tw, x, w->scales, bias, act, y, (int)n, (int)k, S, P, smem);
    return MM == 1 ? launch_one<1, 16>(ctx, tw, x, w->scales, bias, act, y, (int)n, (int)k, S, P, smem)
                   : launch_one<2, 16>(ctx, tw, x, w->scales, bias, act, y, (int)n, (int)k, S, P, smem);
}

// 3 <= M <= 8, K % 256 == 0, K <= 4096, x 16-byte aligned; returns handled =
// false otherwise.
int launch_w4_small(tpt_cuda_ctx *ctx, const float *x, size_t m, const tpt_cuda_weights *w, const float *bias,
                    int act, float *y, bool *handled) {
    *handled = false;
    const size_t n = w->n, k = w->k;
    if (m < 3 || m > 8 || k % 256 != 0 || k > (size_t)WG_MAX_KW * 256 || n > INT32_MAX) return TPT_OK;
    if (((uintptr_t)x & 15) != 0) return TPT_OK;
    CUtensorMap tw;
    if (!make_tmap_rows3d(&tw, w->data, n, k / 2)) return TPT_OK;
    const int MM = m <= 4 ? 4 : 8, T = (3 * MM + 7) / 8;
    const int kw = (int)((k + 255) / 256);
    const size_t stage = WG_ROWS * (k / 2), table = (size_t)kw * MM * 3 * 32 * 8;
    const size_t per_group = (size_t)MM * kw * WG_ROWS * 4, scratch = (size_t)kw * 16 * 8 * T * 4;
    const size_t groups = (n + WG_ROWS - 1) / WG_ROWS;
    const size_t ctas = groups < (size_t)ctx->sm_count ? groups : (size_t)ctx->sm_count;
    const size_t run = (groups + ctas - 1) / ctas;
    const size_t pmax = (4 * WG_PART_BUDGET) / per_group;
    const int P = (int)(run < pmax ? run : pmax);
    if (P < 1) return TPT_OK;
    const size_t shared = table > (size_t)P * per_group + scratch ? table : (size_t)P * per_group + scratch;
    const size_t budget = WG_SMEM_MAX - shared - 1024 - 128;
    const int S = (int)(budget / stage < 8 ? budget / stage : 8);
    if (S < 2) return TPT_OK;
    const size_t smem = 1024 + (size_t)S * stage + shared + (size_t)2 * S * 8;
    *handled = true;
    return MM == 4 ? launch_small<4>(ctx, tw, x, w->scales, bias, act, y, (int)m, (int)n, (int)k, S, P, smem)
                   : launch_small<8>(ctx, tw, x, w->scales, bias, act, y, (int)m, (int)n, (int)k, S, P, smem);
}

}  // namespace tpt
