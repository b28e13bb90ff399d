/* Checks, on the CPU, the arithmetic of the division-free requantization in
 * the int8 epilogues (requant_i8_fast in tpt_infer_b200/csrc/common.cuh)
 * against clamp(roundf(y / s), -127, 127) with an IEEE division:
 *  - the quotient: q1 = y * rs (rs = 1/s correctly rounded), two FMA residual
 *    steps; must equal y / s wherever |y / s| >= 2^-20 (the second step is
 *    Markstein's correction; below that only an underflowing residual can
 *    differ, and those quotients round to 0);
 *  - the rounding: truncation (saturating, NaN -> 0) plus the fraction test
 *    against roundf-then-clamp;
 *  - the int8 result, for every y of one scale's whole range |y / s| in
 *    [2^-3, 2^8), for values within 64 ulps of every half-integer multiple of
 *    the scale, and for random y, over many scales in [2^-40, 2^40].
 * C's fmaf and float division are correctly rounded, as __fmaf_rn and the
 * IEEE division are on the GPU. Exit status 0 when nothing differs. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static float f_of(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t u_of(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

static int ref_i8(float y, float s) {
    float v = roundf(y / s);
    if (isnan(v)) return 0;
    return (int)fminf(fmaxf(v, -127.0f), 127.0f);
}
static float quotient(float y, float s, float rs) {
    const float q1 = y * rs;
    const float q2 = fmaf(fmaf(-s, q1, y), rs, q1);
    return fmaf(fmaf(-s, q2, y), rs, q2);
}
static int32_t cvt_rzi(float q) {  /* cvt.rzi.s32.f32 */
    if (isnan(q)) return 0;
    if (q >= 2147483648.0f) return INT32_MAX;
    if (q <= -2147483904.0f) return INT32_MIN;
    return (int32_t)truncf(q);
}
static int fast_i8(float y, float s, float rs) {
    float q = quotient(y, s, rs);
    q = fabsf(y) <= 0x1p80f ? q : y;
    const float f = q - truncf(q);
    int64_t n = (int64_t)cvt_rzi(q) + (f >= 0.5f ? 1 : 0) - (f <= -0.5f ? 1 : 0);
    return (int)(n > 127 ? 127 : (n < -127 ? -127 : n));
}

static uint64_t rng = 88172645463325252ull;
static uint64_t xr(void) { rng ^= rng << 13; rng ^= rng >> 7; rng ^= rng << 17; return rng; }
static long checked, bad_q, bad_i8;

static void check(float y, float s, float rs) {
    checked++;
    const float a = quotient(y, s, rs), b = y / s;
    if (a != b && fabsf(b) >= 0x1p-20f && fabsf(y) <= 0x1p80f && bad_q++ < 5)
        printf("quotient differs: s=%a y=%a %a %a\n", s, y, a, b);
    if (fast_i8(y, s, rs) != ref_i8(y, s) && bad_i8++ < 5)
        printf("int8 differs: s=%a y=%a %d %d\n", s, y, fast_i8(y, s, rs), ref_i8(y, s));
}

int main(int argc, char **argv) {
    const int nscales = argc > 1 ? atoi(argv[1]) : 300;
    for (int i = 0; i < nscales; i++) {
        float s;
        if (i == 0) s = 1.0f / 127.0f;
        else if (i == 1) s = f_of(0x3fffffffu);
        else if (i == 2) s = 1.0f;
        else s = f_of(0x3f800000u | (uint32_t)(xr() & 0x7fffffu)) * ldexpf(1.0f, (int)(xr() % 81) - 40);
        const float rs = 1.0f / s;
        if (i == 0)  /* every y of the scale's range */
            for (uint32_t u = u_of(s * 0.125f); u <= u_of(s * 256.0f); u++) {
                check(f_of(u), s, rs);
                check(-f_of(u), s, rs);
            }
        for (int k = -140; k <= 140; k++) {
            const uint32_t c = u_of(((float)k + 0.5f) * s);
            for (int d = -64; d <= 64; d++) {
                const float y = f_of(c + (uint32_t)d);
                if (isfinite(y)) check(y, s, rs);
            }
        }
        for (int j = 0; j < 20000; j++) check(f_of((uint32_t)xr()), s, rs);
        const float sp[] = {0.0f, -0.0f, INFINITY, -INFINITY, NAN, 0x1p80f, -0x1p81f, 3e38f, 1e-45f};
        for (int j = 0; j < 9; j++) check(sp[j], s, rs);
    }
    /* the rounding alone, over a stride of all 2^32 bit patterns */
    long bad_r = 0;
    for (uint64_t u = 0; u < (1ull << 32); u += 61) {
        const float v = f_of((uint32_t)u);
        float r = roundf(v);
        const int want = isnan(r) ? 0 : (int)fminf(fmaxf(r, -127.0f), 127.0f);
        const float f = v - truncf(v);
        int64_t n = (int64_t)cvt_rzi(v) + (f >= 0.5f ? 1 : 0) - (f <= -0.5f ? 1 : 0);
        n = n > 127 ? 127 : (n < -127 ? -127 : n);
        if (n != want && bad_r++ < 5) printf("rounding differs at %a\n", v);
    }
    printf("checked %ld values; quotient mismatches %ld, int8 mismatches %ld, rounding mismatches %ld\n", checked,
           bad_q, bad_i8, bad_r);
    return (bad_q || bad_i8 || bad_r) ? 1 : 0;
}
