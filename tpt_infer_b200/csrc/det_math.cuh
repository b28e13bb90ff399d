// det_math.cuh -- exp, reciprocal and GELU built only from correctly rounded
// IEEE operations (fmaf, multiply, add, exact scaling by a power of two),
// so a C restatement with the same operations in the same order gives the
// same bits on the CPU. The model paths that must match a CPU replay bit for
// bit use these instead of library transcendentals: the attention softmax and
// every GELU epilogue.
//
// exp_det(x): Cody-Waite range reduction (W. J. Cody and W. Waite, "Software
// Manual for the Elementary Functions", 1980): n = x log2 e rounded to the
// nearest integer (by one fma with 1.5 * 2^23: no conversion instructions),
// r = x - n ln2 with ln2 split into a 12-bit head (n * head is exact for
// |n| < 2^12) and a tail, then the degree-7 Taylor polynomial of e^r on
// |r| <= ln2/2 (truncation error < 6e-9 relative) by Horner's rule with fmaf,
// scaled by 2^n through the exponent bits. Within 2 ulp of e^x for
// x in [-87, 88]; 0 below -87 (the softmax terms there are < 2^-125 of the
// row's largest), +inf above 88, NaN propagates.
//
// recip12_det(d): 1/d for d in [1, 2] by Newton-Raphson from the linear start
// 24/17 - 8/17 d (maximum relative error 1/17), three steps (error < 2e-10
// before the last rounding). Not correctly rounded, but deterministic.
//
// gelu_det(x): the tanh form of naive.rs:137-146, inner = K (x + C x x x) with
// the same association, and 0.5 x (1 + tanh(inner)) written without tanh: with
// t = exp(-2 |inner|), 1 + tanh(inner) = 2 / (1 + t) when inner >= 0 and
// 2 t / (1 + t) otherwise, so gelu = (x w) / (1 + t) with w = 1 or t. This
// avoids the cancellation in 1 + tanh for negative inputs and agrees with the
// tanh form to within a few ulp of its largest term.
#pragma once

namespace tpt {

constexpr float DET_LOG2E = 1.44269504f;
constexpr float DET_LN2_HI = 0.693145751953125f;      // 12 significant bits
constexpr float DET_LN2_LO = 1.42860676533018720e-06f;
constexpr float DET_C2 = 0.5f, DET_C3 = 0.166666672f, DET_C4 = 0.0416666679f, DET_C5 = 0.00833333377f,
                DET_C6 = 0.00138888892f, DET_C7 = 0.000198412701f;  // 1/k!

__device__ __forceinline__ float exp_det(float x) {
    // the range cases by selects, not branches: the polynomial runs on x clamped
    // to [-87, 88] and the result is replaced below / above / for NaN
    const float xc = fminf(fmaxf(x, -87.0f), 88.0f);
    // n = x log2 e rounded to an integer inside one fma: adding 1.5 * 2^23 leaves
    // ulp 1, so the sum's low mantissa bits are n (two's complement offset)
    const float t = __fmaf_rn(xc, DET_LOG2E, 12582912.0f);
    const float n = __fsub_rn(t, 12582912.0f);
    float r = __fmaf_rn(n, -DET_LN2_HI, xc);
    r = __fmaf_rn(n, -DET_LN2_LO, r);
    float p = DET_C7;
    p = __fmaf_rn(p, r, DET_C6);
    p = __fmaf_rn(p, r, DET_C5);
    p = __fmaf_rn(p, r, DET_C4);
    p = __fmaf_rn(p, r, DET_C3);
    p = __fmaf_rn(p, r, DET_C2);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    float y = __fmul_rn(p, __int_as_float((__float_as_int(t) - 0x4B400000 + 127) << 23));
    y = x < -87.0f ? 0.0f : y;
    y = x > 88.0f ? __int_as_float(0x7f800000) : y;
    return x != x ? x : y;
}

// exp_det for x <= 0 (and NaN): the same operations and the same result for
// every x <= 0, without the two selects that only x > 88 and NaN reach. A NaN
// argument gives a finite value here, which the GELU below turns back into NaN
// (its x is then NaN too).
__device__ __forceinline__ float exp_det_nonpos(float x) {
    const float xc = fmaxf(x, -87.0f);
    const float t = __fmaf_rn(xc, DET_LOG2E, 12582912.0f);
    const float n = __fsub_rn(t, 12582912.0f);
    float r = __fmaf_rn(n, -DET_LN2_HI, xc);
    r = __fmaf_rn(n, -DET_LN2_LO, r);
    float p = DET_C7;
    p = __fmaf_rn(p, r, DET_C6);
    p = __fmaf_rn(p, r, DET_C5);
    p = __fmaf_rn(p, r, DET_C4);
    p = __fmaf_rn(p, r, DET_C3);
    p = __fmaf_rn(p, r, DET_C2);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const float y = __fmul_rn(p, __int_as_float((__float_as_int(t) - 0x4B400000 + 127) << 23));
    return x < -87.0f ? 0.0f : y;
}

// exp_det for x <= 0 or NaN (a softmax's s - max): the same operations and the
// same result as exp_det there, NaN included, without the select that only
// x > 88 reaches
__device__ __forceinline__ float exp_det_le0(float x) {
    const float xc = fmaxf(x, -87.0f);
    const float t = __fmaf_rn(xc, DET_LOG2E, 12582912.0f);
    const float n = __fsub_rn(t, 12582912.0f);
    float r = __fmaf_rn(n, -DET_LN2_HI, xc);
    r = __fmaf_rn(n, -DET_LN2_LO, r);
    float p = DET_C7;
    p = __fmaf_rn(p, r, DET_C6);
    p = __fmaf_rn(p, r, DET_C5);
    p = __fmaf_rn(p, r, DET_C4);
    p = __fmaf_rn(p, r, DET_C3);
    p = __fmaf_rn(p, r, DET_C2);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    float y = __fmul_rn(p, __int_as_float((__float_as_int(t) - 0x4B400000 + 127) << 23));
    y = x < -87.0f ? 0.0f : y;
    return x != x ? x : y;
}

// 1/d for d in [1, 2]: Newton-Raphson r <- r + r (1 - d r) from the linear start
// 24/17 - 8/17 d (relative error at most 1/17), three steps
__device__ __forceinline__ float recip12_det(float d) {
    float r = __fmaf_rn(d, -0.470588237f, 1.41176474f);
#pragma unroll
    for (int i = 0; i < 3; i++) r = __fmaf_rn(r, __fmaf_rn(-d, r, 1.0f), r);
    return r;
}

__device__ __forceinline__ float gelu_det(float x) {
    const float K = 0.7978846f, Cc = 0.044715f;
    const float cx = __fmul_rn(__fmul_rn(__fmul_rn(Cc, x), x), x);
    const float inner = __fmul_rn(K, __fadd_rn(x, cx));
    const float t = exp_det_nonpos(__fmul_rn(-2.0f, fabsf(inner)));
    const float w = inner >= 0.0f ? 1.0f : t;
    return __fmul_rn(__fmul_rn(x, w), recip12_det(__fadd_rn(1.0f, t)));
}

// Pairs of f32 values in one 64-bit register and the paired IEEE operations
// (fma / add / mul .rn.f32x2: two correctly rounded results per issue, the
// same bits as the scalar operations)
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float &lo, float &hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t splat2(float x) { return f2pack(x, x); }

// A paired product that keeps its own rounding. The compiler fuses a paired
// multiply into a paired add that consumes it (the .rn modifier does not stop
// this for .f32x2, and it sees fma(a, b, -0) and fma(a, 1, c) as a multiply
// and an add), which rounds once where the scalar form rounds twice. An fma
// whose addend it cannot prove to be -0 is kept as written, and fma(a, b, -0)
// is the correctly rounded product for every a and b, signed zeros included.
// nz holds (-0, -0), made by opaque_nz2 from a value that is 0 at run time
// but not known to the compiler (a launch parameter known to be
// non-negative, shifted right by 31). Products that are exact (a power-of-two
// factor) and products that feed no add need none of this.
__device__ __forceinline__ uint64_t opaque_nz2(uint32_t zero) { return splat2(__uint_as_float(0x80000000u | zero)); }
__device__ __forceinline__ uint64_t mulr2(uint64_t a, uint64_t b, uint64_t nz) { return fma2(a, b, nz); }

// exp_det_le0 of two values (x <= 0 or NaN): the same operations in the same
// order on each half (a difference u - v as fma(v, -1, u): one rounding, as
// the subtraction)
__device__ __forceinline__ void exp_det_le0_x2(float x0, float x1, float &y0, float &y1) {
    const uint64_t magic = splat2(12582912.0f);
    const uint64_t xc = f2pack(fmaxf(x0, -87.0f), fmaxf(x1, -87.0f));
    const uint64_t t = fma2(xc, splat2(DET_LOG2E), magic);
    const uint64_t n = add2(t, splat2(-12582912.0f));
    uint64_t r = fma2(n, splat2(-DET_LN2_HI), xc);
    r = fma2(n, splat2(-DET_LN2_LO), r);
    uint64_t p = splat2(DET_C7);
    p = fma2(p, r, splat2(DET_C6));
    p = fma2(p, r, splat2(DET_C5));
    p = fma2(p, r, splat2(DET_C4));
    p = fma2(p, r, splat2(DET_C3));
    p = fma2(p, r, splat2(DET_C2));
    p = fma2(p, r, splat2(1.0f));
    p = fma2(p, r, splat2(1.0f));
    float t0, t1;
    f2unpack(t, t0, t1);
    const uint64_t sc = f2pack(__int_as_float((__float_as_int(t0) - 0x4B400000 + 127) << 23),
                               __int_as_float((__float_as_int(t1) - 0x4B400000 + 127) << 23));
    float z0, z1;
    f2unpack(mul2(p, sc), z0, z1);
    z0 = x0 < -87.0f ? 0.0f : z0;
    z1 = x1 < -87.0f ? 0.0f : z1;
    y0 = x0 != x0 ? x0 : z0;
    y1 = x1 != x1 ? x1 : z1;
}

// exp_det_nonpos of two values (x <= 0; a NaN half gives a finite value, as
// the scalar form): the same operations on each half
__device__ __forceinline__ void exp_det_nonpos_x2(float x0, float x1, float &y0, float &y1) {
    const uint64_t magic = splat2(12582912.0f);
    const uint64_t xc = f2pack(fmaxf(x0, -87.0f), fmaxf(x1, -87.0f));
    const uint64_t t = fma2(xc, splat2(DET_LOG2E), magic);
    const uint64_t n = add2(t, splat2(-12582912.0f));
    uint64_t r = fma2(n, splat2(-DET_LN2_HI), xc);
    r = fma2(n, splat2(-DET_LN2_LO), r);
    uint64_t p = splat2(DET_C7);
    p = fma2(p, r, splat2(DET_C6));
    p = fma2(p, r, splat2(DET_C5));
    p = fma2(p, r, splat2(DET_C4));
    p = fma2(p, r, splat2(DET_C3));
    p = fma2(p, r, splat2(DET_C2));
    p = fma2(p, r, splat2(1.0f));
    p = fma2(p, r, splat2(1.0f));
    float t0, t1;
    f2unpack(t, t0, t1);
    const uint64_t sc = f2pack(__int_as_float((__float_as_int(t0) - 0x4B400000 + 127) << 23),
                               __int_as_float((__float_as_int(t1) - 0x4B400000 + 127) << 23));
    float z0, z1;
    f2unpack(mul2(p, sc), z0, z1);
    y0 = x0 < -87.0f ? 0.0f : z0;
    y1 = x1 < -87.0f ? 0.0f : z1;
}

// recip12_det of two values (both in [1, 2])
__device__ __forceinline__ uint64_t recip12_det_x2(uint64_t d) {
    float d0, d1;
    f2unpack(d, d0, d1);
    const uint64_t nd = f2pack(-d0, -d1);
    uint64_t r = fma2(d, splat2(-0.470588237f), splat2(1.41176474f));
#pragma unroll
    for (int i = 0; i < 3; i++) r = fma2(r, fma2(nd, r, splat2(1.0f)), r);
    return r;
}

// gelu_det of two values: the same operations in the same order on each half
// (nz from opaque_nz2: the product C x x x feeds an add)
__device__ __forceinline__ void gelu_det_x2(float x0, float x1, uint64_t nz, float &g0, float &g1) {
    const uint64_t X = f2pack(x0, x1);
    const uint64_t cx = mulr2(mul2(mul2(splat2(0.044715f), X), X), X, nz);
    const uint64_t inner = mul2(splat2(0.7978846f), add2(X, cx));
    float i0, i1;
    f2unpack(inner, i0, i1);
    float a0, a1;
    f2unpack(mul2(splat2(-2.0f), f2pack(fabsf(i0), fabsf(i1))), a0, a1);
    float t0, t1;
    exp_det_nonpos_x2(a0, a1, t0, t1);
    const uint64_t w = f2pack(i0 >= 0.0f ? 1.0f : t0, i1 >= 0.0f ? 1.0f : t1);
    const uint64_t r = recip12_det_x2(add2(splat2(1.0f), f2pack(t0, t1)));
    f2unpack(mul2(mul2(X, w), r), g0, g1);
}

}  // namespace tpt
