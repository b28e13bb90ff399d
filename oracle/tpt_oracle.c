/*
 * tpt_oracle.c -- CPU restatement of tpt-infer's reference CPU kernels.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker and the timed CPU baseline);
 * see tpt_oracle.h. Build with -O3 -ffp-contract=off (oracle/Makefile).
 * Paths cited below are relative to the tpt-infer repository root.
 */
#include "tpt_oracle.h"

#include <float.h>
#include <math.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static _Thread_local size_t g_expected, g_actual;

void tpto_last_size_mismatch(size_t *expected, size_t *actual) {
    *expected = g_expected;
    *actual = g_actual;
}

static int size_mismatch(size_t expected, size_t actual) {
    g_expected = expected;
    g_actual = actual;
    return TPTO_SIZE_MISMATCH;
}

/* checked multiply, the `checked_mul(..).ok_or(OpError::Invalid)` of backend.rs */
static int cmul(size_t a, size_t b, size_t *r) {
    if (a != 0 && b > SIZE_MAX / a) return 0;
    *r = a * b;
    return 1;
}

static void set_threads(int threads) {
#ifdef _OPENMP
    omp_set_num_threads(threads > 0 ? threads : 1);
#else
    (void)threads;
#endif
}

/* ------------------------------------------------------------------ */
/* Generators                                                          */
/* ------------------------------------------------------------------ */

/* crates/tpt-infer-ops/src/dispatch.rs:274-282: s = s*1664525 + 1013904223
 * (wrapping u32), value = ((s>>8) as f32 / 2^24) * 2 - 1. */
void tpto_lcg_sym(float *out, size_t n, uint32_t seed) {
    uint32_t s = seed;
    for (size_t i = 0; i < n; i++) {
        s = s * 1664525u + 1013904223u;
        out[i] = ((float)(s >> 8) / (float)(1u << 24)) * 2.0f - 1.0f;
    }
}

/* Same LCG, U[0,1) = (s>>8)/2^24 (the dispatch.rs value before the affine map). */
void tpto_lcg_uniform(float *out, size_t n, uint32_t seed) {
    uint32_t s = seed;
    for (size_t i = 0; i < n; i++) {
        s = s * 1664525u + 1013904223u;
        out[i] = (float)(s >> 8) / (float)(1u << 24);
    }
}

/* N(mean, std): Box-Muller on consecutive LCG pairs (u1 in (0,1], u2 in [0,1)),
 * evaluated in double and rounded once to f32. The reference has no normal
 * sampler; this one is defined for the seeded workloads. */
void tpto_normal(float *out, size_t n, uint32_t seed, float mean, float std) {
    uint32_t s = seed;
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t i = 0; i < n; i += 2) {
        s = s * 1664525u + 1013904223u;
        double u1 = 1.0 - (double)(s >> 8) / 16777216.0;
        s = s * 1664525u + 1013904223u;
        double u2 = (double)(s >> 8) / 16777216.0;
        double r = sqrt(-2.0 * log(u1));
        out[i] = (float)((double)mean + (double)std * r * cos(two_pi * u2));
        if (i + 1 < n) out[i + 1] = (float)((double)mean + (double)std * r * sin(two_pi * u2));
    }
}

/* ------------------------------------------------------------------ */
/* Backend ops                                                         */
/* ------------------------------------------------------------------ */

/* crates/tpt-infer-ops/src/backend.rs:149-183 (validate_matmul), same order. */
static int validate_matmul(size_t a_len, size_t m, size_t k, size_t b_len, size_t kb, size_t n,
                           size_t out_len) {
    size_t e;
    if (k != kb) return TPTO_SHAPE_MISMATCH;
    if (!cmul(m, k, &e)) return TPTO_INVALID;
    if (a_len != e) return size_mismatch(e, a_len);
    if (!cmul(k, n, &e)) return TPTO_INVALID;
    if (b_len != e) return size_mismatch(e, b_len);
    if (!cmul(m, n, &e)) return TPTO_INVALID;
    if (out_len != e) return size_mismatch(e, out_len);
    return TPTO_OK;
}

/* crates/tpt-infer-ops/src/naive.rs:13-33: per output, sequential k,
 * acc += a*b (a multiply and an add, never fused). */
int tpto_matmul_naive(const float *a, size_t a_len, size_t m, size_t k,
                      const float *b, size_t b_len, size_t kb, size_t n,
                      float *out, size_t out_len) {
    int st = validate_matmul(a_len, m, k, b_len, kb, n, out_len);
    if (st) return st;
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            float acc = 0.0f;
            for (size_t kk = 0; kk < k; kk++) acc += a[i * k + kk] * b[kk * n + j];
            out[i * n + j] = acc;
        }
    return TPTO_OK;
}

/* ONNX Gemm, Y = alpha * op(A) op(B) + beta * C: the semantics tpt-infer's
 * loader drops when it maps "Gemm" to a plain MatMul (crates/tpt-infer-onnx/
 * src/registry.rs:21; the transA/transB/alpha/beta attributes fall through the
 * attribute match in load.rs:410-445). Defined here, restated by the device
 * kernel: op(A) = A [m,k] or A^T of a stored [k,m]; op(B) = B [k,n] or B^T of a
 * stored [n,k]; the sum runs in increasing k with a separate multiply and add
 * (as naive.rs:13-33); then y = alpha*acc, plus beta*C when C is given, each
 * product and the sum rounded separately. C is [n] (broadcast over rows) or
 * [m,n]; c_len = 0 means no C. */
int tpto_gemm(const float *a, size_t a_len, size_t m, size_t k, int trans_a,
              const float *b, size_t b_len, size_t n, int trans_b,
              const float *c, size_t c_len, float alpha, float beta,
              float *out, size_t out_len) {
    if (a_len != m * k) return TPTO_SIZE_MISMATCH;
    if (b_len != k * n) return TPTO_SIZE_MISMATCH;
    if (c_len != 0 && c_len != n && c_len != m * n) return TPTO_SHAPE_MISMATCH;
    if (out_len != m * n) return TPTO_SIZE_MISMATCH;
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            float acc = 0.0f;
            for (size_t kk = 0; kk < k; kk++) {
                const float av = trans_a ? a[kk * m + i] : a[i * k + kk];
                const float bv = trans_b ? b[j * k + kk] : b[kk * n + j];
                const float p = av * bv;
                acc = acc + p;
            }
            float y = alpha * acc;
            if (c_len) {
                const float cv = c_len == n ? c[j] : c[i * n + j];
                const float t = beta * cv;
                y = y + t;
            }
            out[i * n + j] = y;
        }
    return TPTO_OK;
}

/* crates/tpt-infer-ops/src/avx512.rs:55-78 (and avx2.rs:47-66): out.fill(0);
 * for i, kk: out[i, :] = out[i, :] + a[i,kk]*b[kk, :] with a separate mul and
 * add. Bit-identical to naive (same k order, same two roundings). The j loop
 * vectorises under -O3; rows run on `threads` OpenMP threads. */
int tpto_matmul_avx(const float *a, size_t a_len, size_t m, size_t k,
                    const float *b, size_t b_len, size_t kb, size_t n,
                    float *out, size_t out_len, int threads) {
    int st = validate_matmul(a_len, m, k, b_len, kb, n, out_len);
    if (st) return st;
    set_threads(threads);
#pragma omp parallel for schedule(static) if (threads > 1)
    for (size_t i = 0; i < m; i++) {
        float *o = out + i * n;
        for (size_t j = 0; j < n; j++) o[j] = 0.0f;
        for (size_t kk = 0; kk < k; kk++) {
            const float av = a[i * k + kk];
            const float *br = b + kk * n;
            for (size_t j = 0; j < n; j++) o[j] = o[j] + av * br[j];
        }
    }
    return TPTO_OK;
}

/* crates/tpt-infer-ops/src/backend.rs:219-284 (validate_conv2d), same order.
 * Writes the output dims on success. */
static int validate_conv2d(size_t in_len, const size_t is[4], size_t w_len, const size_t ws[4],
                           size_t out_len, size_t sh, size_t sw, size_t ph, size_t pw,
                           size_t *oh, size_t *ow) {
    size_t e, ph2, pw2;
    if (ws[1] != is[1]) return TPTO_SHAPE_MISMATCH;
    if (ws[2] == 0 || ws[3] == 0) return TPTO_INVALID;
    if (sh == 0 || sw == 0) return TPTO_INVALID;
    if (!cmul(ph, 2, &ph2) || is[2] > SIZE_MAX - ph2) return TPTO_INVALID;
    if (!cmul(pw, 2, &pw2) || is[3] > SIZE_MAX - pw2) return TPTO_INVALID;
    size_t hp = is[2] + ph2, wp = is[3] + pw2;
    if (hp < ws[2] || wp < ws[3]) return TPTO_INVALID;
    *oh = (hp - ws[2]) / sh + 1;
    *ow = (wp - ws[3]) / sw + 1;
    if (!cmul(is[0], is[1], &e) || !cmul(e, is[2], &e) || !cmul(e, is[3], &e)) return TPTO_INVALID;
    if (in_len != e) return size_mismatch(e, in_len);
    if (!cmul(ws[0], ws[1], &e) || !cmul(e, ws[2], &e) || !cmul(e, ws[3], &e)) return TPTO_INVALID;
    if (w_len != e) return size_mismatch(e, w_len);
    if (!cmul(is[0], ws[0], &e) || !cmul(e, *oh, &e) || !cmul(e, *ow, &e)) return TPTO_INVALID;
    if (out_len != e) return size_mismatch(e, out_len);
    return TPTO_OK;
}

/* crates/tpt-infer-ops/src/naive.rs:36-83: direct conv, loop order
 * n, oc, oy, ox, ci, ky, kx; padded taps skipped. */
int tpto_conv2d(const float *in, size_t in_len, const size_t is[4],
                const float *w, size_t w_len, const size_t ws[4],
                float *out, size_t out_len, size_t sh, size_t sw,
                size_t ph, size_t pw, int threads) {
    size_t oh, ow;
    int st = validate_conv2d(in_len, is, w_len, ws, out_len, sh, sw, ph, pw, &oh, &ow);
    if (st) return st;
    const size_t N = is[0], C = is[1], H = is[2], W = is[3];
    const size_t OC = ws[0], KH = ws[2], KW = ws[3];
    set_threads(threads);
#pragma omp parallel for collapse(2) schedule(static) if (threads > 1)
    for (size_t ni = 0; ni < N; ni++)
        for (size_t o = 0; o < OC; o++)
            for (size_t oy = 0; oy < oh; oy++)
                for (size_t ox = 0; ox < ow; ox++) {
                    float acc = 0.0f;
                    for (size_t ci = 0; ci < C; ci++)
                        for (size_t ky = 0; ky < KH; ky++) {
                            size_t y = oy * sh + ky;
                            if (y < ph || y - ph >= H) continue;
                            size_t iy = y - ph;
                            for (size_t kx = 0; kx < KW; kx++) {
                                size_t x = ox * sw + kx;
                                if (x < pw || x - pw >= W) continue;
                                size_t ix = x - pw;
                                acc += in[((ni * C + ci) * H + iy) * W + ix] *
                                       w[((o * C + ci) * KH + ky) * KW + kx];
                            }
                        }
                    out[((ni * OC + o) * oh + oy) * ow + ox] = acc;
                }
    return TPTO_OK;
}

/* backend.rs:185-199 (validate_binary) + naive.rs:86-92 */
int tpto_elementwise_add(const float *a, size_t a_len, const float *b, size_t b_len,
                         float *out, size_t out_len) {
    if (a_len != b_len) return size_mismatch(a_len, b_len);
    if (out_len != a_len) return size_mismatch(a_len, out_len);
    for (size_t i = 0; i < a_len; i++) out[i] = a[i] + b[i];
    return TPTO_OK;
}

/* backend.rs:201-209 (validate_unary) + naive.rs:95-101 */
int tpto_relu(const float *a, size_t a_len, float *out, size_t out_len) {
    if (out_len != a_len) return size_mismatch(a_len, out_len);
    for (size_t i = 0; i < a_len; i++) out[i] = a[i] > 0.0f ? a[i] : 0.0f;
    return TPTO_OK;
}

/* backend.rs:211-217 (validate_softmax) + naive.rs:104-125: running max,
 * exp(v - max) (std => libm expf, math.rs:3-6), sequential sum, divide. */
int tpto_softmax(const float *a, size_t a_len, float *out, size_t out_len, size_t row_len) {
    if (out_len != a_len) return size_mismatch(a_len, out_len);
    if (row_len == 0 || a_len % row_len != 0) return TPTO_INVALID;
    for (size_t r = 0; r < a_len / row_len; r++) {
        const float *src = a + r * row_len;
        float *dst = out + r * row_len;
        float mx = -INFINITY;
        for (size_t i = 0; i < row_len; i++)
            if (src[i] > mx) mx = src[i];
        for (size_t i = 0; i < row_len; i++) dst[i] = expf(src[i] - mx);
        float sum = 0.0f;
        for (size_t i = 0; i < row_len; i++) sum += dst[i];
        for (size_t i = 0; i < row_len; i++) dst[i] /= sum;
    }
    return TPTO_OK;
}

/* naive.rs:128-134 */
int tpto_sigmoid(const float *a, size_t a_len, float *out, size_t out_len) {
    if (out_len != a_len) return size_mismatch(a_len, out_len);
    for (size_t i = 0; i < a_len; i++) out[i] = 1.0f / (1.0f + expf(-a[i]));
    return TPTO_OK;
}

/* naive.rs:137-146: K = 0.797_884_6, C = 0.044_715,
 * inner = K*(x + C*x*x*x) (left-associated), 0.5*x*(1 + tanh(inner)). */
static float gelu1(float x) {
    const float K = 0.7978846f, C = 0.044715f;
    float inner = K * (x + C * x * x * x);
    return 0.5f * x * (1.0f + tanhf(inner));
}

/* The device's deterministic exp / reciprocal / GELU (tpt_infer_b200/csrc/
 * det_math.cuh), restated with the same correctly rounded operations in the
 * same order: Cody-Waite reduction + degree-7 Taylor polynomial for exp,
 * three Newton steps from 24/17 - 8/17 d for 1/d on [1, 2], and
 * GELU = x w / (1 + t) with t = exp(-2 |inner|). Used by the W8A8 epilogue's
 * GELU and the attention softmax, which this backend defines. */
float tpto_exp_det(float x) {
    if (!(x >= -87.0f)) return x != x ? x : 0.0f;
    if (x > 88.0f) return INFINITY;
    const float t = fmaf(x, 1.44269504f, 12582912.0f);
    const float n = t - 12582912.0f;
    float r = fmaf(n, -0.693145751953125f, x);
    r = fmaf(n, -1.42860676533018720e-06f, r);
    float p = 0.000198412701f;
    p = fmaf(p, r, 0.00138888892f);
    p = fmaf(p, r, 0.00833333377f);
    p = fmaf(p, r, 0.0416666679f);
    p = fmaf(p, r, 0.166666672f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int32_t tb;
    memcpy(&tb, &t, 4);
    uint32_t eb = (uint32_t)(tb - 0x4B400000 + 127) << 23;
    float sc;
    memcpy(&sc, &eb, 4);
    return p * sc;
}

static float recip12_det(float d) {
    float r = fmaf(d, -0.470588237f, 1.41176474f);
    for (int i = 0; i < 3; i++) r = fmaf(r, fmaf(-d, r, 1.0f), r);
    return r;
}

float tpto_gelu_det(float x) {
    const float K = 0.7978846f, C = 0.044715f;
    const float cx = ((C * x) * x) * x;
    const float inner = K * (x + cx);
    const float t = tpto_exp_det(-2.0f * fabsf(inner));
    const float w = inner >= 0.0f ? 1.0f : t;
    return (x * w) * recip12_det(1.0f + t);
}

void tpto_gelu_det_array(const float *a, size_t n, float *out) {
    for (size_t i = 0; i < n; i++) out[i] = tpto_gelu_det(a[i]);
}

void tpto_exp_det_array(const float *a, size_t n, float *out) {
    for (size_t i = 0; i < n; i++) out[i] = tpto_exp_det(a[i]);
}

int tpto_gelu(const float *a, size_t a_len, float *out, size_t out_len) {
    if (out_len != a_len) return size_mismatch(a_len, out_len);
    for (size_t i = 0; i < a_len; i++) out[i] = gelu1(a[i]);
    return TPTO_OK;
}

/* ------------------------------------------------------------------ */
/* Quantization                                                        */
/* ------------------------------------------------------------------ */

/* Rust `v.clamp(lo, hi) as i8`: NaN passes clamp and the saturating cast
 * maps it to 0. `round` is f32::round = half away from zero = roundf. */
static int8_t clamp_cast_i8(float v, float lo, float hi) {
    if (isnan(v)) return 0;
    if (v < lo) v = lo;
    if (v > hi) v = hi;
    return (int8_t)v;
}

/* fold(0.0, |m, x| m.max(x.abs())): f32::max ignores a NaN operand = fmaxf */
static float max_abs(const float *x, size_t n) {
    float m = 0.0f;
    for (size_t i = 0; i < n; i++) m = fmaxf(m, fabsf(x[i]));
    return m;
}

/* crates/tpt-infer-quantize/src/quant.rs:25-40 */
float tpto_quantize_i8_symmetric(const float *x, size_t n, int8_t *q) {
    float ma = max_abs(x, n);
    float scale = ma == 0.0f ? 1.0f : ma / 127.0f;
    for (size_t i = 0; i < n; i++) q[i] = clamp_cast_i8(roundf(x[i] / scale), -127.0f, 127.0f);
    return scale;
}

/* quant.rs:45-90 */
void tpto_quantize_i8_asymmetric(const float *x, size_t n, int8_t *q, float *scale_out,
                                 int32_t *zp_out) {
    const float QMIN = -128.0f, QMAX = 127.0f;
    float mn = INFINITY, mx = -INFINITY;
    for (size_t i = 0; i < n; i++) {
        mn = fminf(mn, x[i]);
        mx = fmaxf(mx, x[i]);
    }
    if (mn > mx || !isfinite(mn) || !isfinite(mx)) {
        mn = 0.0f;
        mx = 0.0f;
    }
    float scale;
    int32_t zp;
    if (fabsf(mx - mn) < FLT_EPSILON) {
        scale = 1.0f;
        zp = 0;
    } else {
        float scale0 = (mx - mn) / (QMAX - QMIN);
        float zp0 = roundf(QMIN - mn / scale0);
        if (zp0 < QMIN) {
            float s = mx / (QMAX - QMIN);
            scale = s <= 0.0f ? scale0 : s;
            zp = (int32_t)QMIN;
        } else if (zp0 > QMAX) {
            float s = mn / (QMIN - QMAX);
            scale = s <= 0.0f ? scale0 : fabsf(s);
            zp = (int32_t)QMAX;
        } else {
            scale = scale0;
            zp = (int32_t)zp0; /* finite, within [-128,127] here */
        }
    }
    for (size_t i = 0; i < n; i++) q[i] = clamp_cast_i8(roundf(x[i] / scale + (float)zp), QMIN, QMAX);
    *scale_out = scale;
    *zp_out = zp;
}

/* quant.rs:95-107 (assert rows>0 && len%rows==0 -> TPTO_INVALID) */
int tpto_quantize_i8_symmetric_per_channel(const float *x, size_t len, size_t rows, int8_t *q,
                                           float *scales) {
    if (rows == 0 || len % rows != 0) return TPTO_INVALID;
    size_t cols = len / rows;
    for (size_t r = 0; r < rows; r++) scales[r] = tpto_quantize_i8_symmetric(x + r * cols, cols, q + r * cols);
    return TPTO_OK;
}

/* quant.rs:123-140: low nibble first, odd tail padded with 0 in the high
 * nibble; out-of-range values panic in the reference (TPTO_INVALID here). */
int tpto_pack_i4(const int8_t *v, size_t n, uint8_t *out) {
    for (size_t i = 0; i < n; i += 2) {
        int8_t lo = v[i];
        if (lo < -8 || lo > 7) return TPTO_INVALID;
        int8_t hi = 0;
        if (i + 1 < n) {
            hi = v[i + 1];
            if (hi < -8 || hi > 7) return TPTO_INVALID;
        }
        out[i / 2] = (uint8_t)((((uint8_t)hi & 0x0f) << 4) | ((uint8_t)lo & 0x0f));
    }
    return TPTO_OK;
}

/* quant.rs:159-166 */
static int8_t sign_extend_i4(uint8_t nib) { return (nib & 0x08) ? (int8_t)(nib | 0xf0) : (int8_t)(nib & 0x0f); }

/* quant.rs:143-157: returns the number of values written (<= n) */
size_t tpto_unpack_i4(const uint8_t *packed, size_t packed_len, size_t n, int8_t *out) {
    size_t c = 0;
    for (size_t i = 0; i < packed_len && c < n; i++) {
        out[c++] = sign_extend_i4(packed[i] & 0x0f);
        if (c >= n) break;
        out[c++] = sign_extend_i4((packed[i] >> 4) & 0x0f);
    }
    return c;
}

/* quant.rs:171-186: scale = max_abs/7, q in [-7, 7] (-8 is never produced) */
float tpto_quantize_i4_symmetric(const float *x, size_t n, uint8_t *packed) {
    float ma = max_abs(x, n);
    float scale = ma == 0.0f ? 1.0f : ma / 7.0f;
    for (size_t i = 0; i < n; i += 2) {
        int8_t lo = clamp_cast_i8(roundf(x[i] / scale), -7.0f, 7.0f);
        int8_t hi = i + 1 < n ? clamp_cast_i8(roundf(x[i + 1] / scale), -7.0f, 7.0f) : 0;
        packed[i / 2] = (uint8_t)((((uint8_t)hi & 0x0f) << 4) | ((uint8_t)lo & 0x0f));
    }
    return scale;
}

/* quant.rs:192-204: each row packed separately into ceil(cols/2) bytes */
int tpto_quantize_i4_symmetric_per_channel(const float *x, size_t len, size_t rows,
                                           uint8_t *packed, float *scales) {
    if (rows == 0 || len % rows != 0) return TPTO_INVALID;
    size_t cols = len / rows, rb = (cols + 1) / 2;
    for (size_t r = 0; r < rows; r++) scales[r] = tpto_quantize_i4_symmetric(x + r * cols, cols, packed + r * rb);
    return TPTO_OK;
}

/* crates/tpt-infer-quantize/src/dequant.rs:13-15 */
void tpto_dequantize_i8_symmetric(const int8_t *q, size_t n, float scale, float *out) {
    for (size_t i = 0; i < n; i++) out[i] = (float)q[i] * scale;
}

/* dequant.rs:18-22 */
void tpto_dequantize_i8_asymmetric(const int8_t *q, size_t n, float scale, int32_t zp, float *out) {
    for (size_t i = 0; i < n; i++) out[i] = ((float)q[i] - (float)zp) * scale;
}

/* dequant.rs:26-37 */
int tpto_dequantize_i8_symmetric_per_channel(const int8_t *q, size_t n, const float *scales,
                                             size_t n_scales, float *out) {
    if (n_scales == 0 || n % n_scales != 0) return TPTO_INVALID;
    size_t cols = n / n_scales;
    for (size_t r = 0; r < n_scales; r++)
        for (size_t c = 0; c < cols; c++) out[r * cols + c] = (float)q[r * cols + c] * scales[r];
    return TPTO_OK;
}

/* dequant.rs:45-50 (unpack_i4 then q*scale; missing tail values are absent) */
void tpto_dequantize_i4_symmetric(const uint8_t *packed, size_t packed_len, size_t n, float scale,
                                  float *out) {
    for (size_t i = 0; i < n && i / 2 < packed_len; i++) {
        uint8_t b = packed[i / 2];
        out[i] = (float)sign_extend_i4((i & 1) ? (b >> 4) & 0x0f : b & 0x0f) * scale;
    }
}

/* dequant.rs:56-71: rows of ceil(row_elems/2) bytes */
void tpto_dequantize_i4_symmetric_per_channel(const uint8_t *packed, size_t packed_len,
                                              size_t row_elems, const float *scales,
                                              size_t n_scales, float *out) {
    size_t rb = (row_elems + 1) / 2;
    for (size_t r = 0; r < n_scales; r++) {
        size_t start = r * rb;
        size_t end = start + rb < packed_len ? start + rb : packed_len;
        size_t avail = start < end ? end - start : 0;
        for (size_t i = 0; i < row_elems && i / 2 < avail; i++) {
            uint8_t b = packed[start + i / 2];
            out[r * row_elems + i] = (float)sign_extend_i4((i & 1) ? (b >> 4) & 0x0f : b & 0x0f) * scales[r];
        }
    }
}

/* crates/tpt-infer-quantize/src/ptq.rs:293-324: acc:i32 = sum_k a*b with b
 * strided by n; out = acc as f32 * (a_scale * b_scales[0]) (product of scales
 * first); b_scales empty -> 1.0. */
int tpto_quantized_matmul_i8(const int8_t *a, size_t a_len, size_t m, size_t k, float a_scale,
                             const int8_t *b, size_t b_len, size_t kb, size_t n,
                             const float *b_scales, size_t n_scales, float *out, size_t out_len) {
    if (k != kb) return TPTO_SHAPE_MISMATCH;
    if (a_len != m * k || b_len != k * n || out_len != m * n) return TPTO_SIZE_MISMATCH;
    float b_scale = n_scales ? b_scales[0] : 1.0f;
    float out_scale = a_scale * b_scale;
    for (size_t mi = 0; mi < m; mi++)
        for (size_t ni = 0; ni < n; ni++) {
            int32_t acc = 0;
            for (size_t ki = 0; ki < k; ki++) acc += (int32_t)a[mi * k + ki] * (int32_t)b[ki * n + ni];
            out[mi * n + ni] = (float)acc * out_scale;
        }
    return TPTO_OK;
}

/* ------------------------------------------------------------------ */
/* Per-output-channel W8A8 and W4 (defined by this backend)            */
/* ------------------------------------------------------------------ */

void tpto_i8_gemm_acc(const int8_t *a, const int8_t *wt, size_t m, size_t n, size_t k,
                      int32_t *acc, int threads) {
    set_threads(threads);
#pragma omp parallel for collapse(2) schedule(static) if (threads > 1)
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            const int8_t *ar = a + i * k, *wr = wt + j * k;
            int32_t s = 0;
            for (size_t kk = 0; kk < k; kk++) s += (int32_t)ar[kk] * (int32_t)wr[kk];
            acc[i * n + j] = s;
        }
}

/* The reference's activation nodes (naive.rs:95-101, :137-146): the W4 path's
 * semantics is dequant -> f32 MatMul -> bias add -> the activation node. */
static float apply_act_ref(float y, int act) {
    if (act == TPTO_ACT_RELU) return y > 0.0f ? y : 0.0f;
    if (act == TPTO_ACT_GELU) return gelu1(y);
    return y;
}

/* The W8A8 epilogue's activation: ReLU, or this backend's deterministic GELU. */
static float apply_act(float y, int act) {
    if (act == TPTO_ACT_RELU) return y > 0.0f ? y : 0.0f;
    if (act == TPTO_ACT_GELU) return tpto_gelu_det(y);  /* the device epilogue's GELU */
    return y;
}

/* The per-output-channel extension of ptq.rs:310-318: the scale product is
 * formed first (a_scale * w_scale[n]), one multiply by the i32 accumulator
 * converted to f32, then the bias add (two roundings, no FMA), then act. */
void tpto_w8a8_gemm(const int8_t *a, const int8_t *wt, size_t m, size_t n, size_t k,
                    float a_scale, const float *w_scales, const float *bias, int act,
                    float *y, int threads) {
    set_threads(threads);
#pragma omp parallel for collapse(2) schedule(static) if (threads > 1)
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            const int8_t *ar = a + i * k, *wr = wt + j * k;
            int32_t s = 0;
            for (size_t kk = 0; kk < k; kk++) s += (int32_t)ar[kk] * (int32_t)wr[kk];
            float v = (float)s * (a_scale * w_scales[j]);
            if (bias) v = v + bias[j];
            y[i * n + j] = apply_act(v, act);
        }
}

void tpto_w8a8_gemm_refloop(const int8_t *a, const int8_t *b_kn, size_t m, size_t n, size_t k,
                            float a_scale, const float *w_scales, const float *bias,
                            float *y, size_t row0, size_t row1, int threads) {
    (void)m;
    set_threads(threads);
#pragma omp parallel for collapse(2) schedule(static) if (threads > 1)
    for (size_t mi = row0; mi < row1; mi++)
        for (size_t ni = 0; ni < n; ni++) {
            int32_t acc = 0;
            for (size_t ki = 0; ki < k; ki++) acc += (int32_t)a[mi * k + ki] * (int32_t)b_kn[ki * n + ni];
            float v = (float)acc * (a_scale * w_scales[ni]);
            if (bias) v = v + bias[ni];
            y[mi * n + ni] = v;
        }
}

/* q = clamp(round(x / scale), -127, 127) with a given (static) scale: the
 * per-element rule of quant.rs:32-38. */
void tpto_quantize_i8_static(const float *x, size_t n, float scale, int8_t *q) {
    for (size_t i = 0; i < n; i++) q[i] = clamp_cast_i8(roundf(x[i] / scale), -127.0f, 127.0f);
}

/* max |x| (NaN ignored), the fold of quant.rs:26 */
float tpto_absmax(const float *x, size_t n) { return max_abs(x, n); }

/* Requantisation of an epilogue value for the next quantized op:
 * q = clamp(round(y / s), -127, 127), the rule of quant.rs:35-36. */
float tpto_requant_i8(float y, float out_scale, int8_t *q) {
    *q = clamp_cast_i8(roundf(y / out_scale), -127.0f, 127.0f);
    return (float)*q;
}

/* W4 reference: w[k,n] = q[n,k] * s[n] (dequant.rs:56-71, rounded to f32),
 * then the avx512.rs:55-78 matmul (sequential k, mul then add), then the
 * runtime's separate bias add (exec.rs:388-391) and the activation. */
void tpto_w4_gemm(const float *x, const uint8_t *wt_packed, const float *w_scales,
                  size_t m, size_t n, size_t k, const float *bias, int act, float *y, int threads) {
    size_t rb = (k + 1) / 2;
    set_threads(threads);
#pragma omp parallel for collapse(2) schedule(static) if (threads > 1)
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            const uint8_t *wr = wt_packed + j * rb;
            const float *xr = x + i * k;
            float acc = 0.0f;
            for (size_t kk = 0; kk < k; kk++) {
                uint8_t b = wr[kk / 2];
                float w = (float)sign_extend_i4((kk & 1) ? (b >> 4) & 0x0f : b & 0x0f) * w_scales[j];
                acc = acc + xr[kk] * w;
            }
            if (bias) acc = acc + bias[j];
            y[i * n + j] = apply_act_ref(acc, act);
        }
}

/* ------------------------------------------------------------------ */
/* Runtime kernels                                                     */
/* ------------------------------------------------------------------ */

/* crates/tpt-infer-runtime/src/kernels.rs:271-325: padding acts as -inf */
void tpto_max_pool2d(const float *in, size_t n, size_t c, size_t h, size_t w,
                     size_t kh, size_t kw, size_t sh, size_t sw, size_t ph, size_t pw,
                     float *out, size_t oh, size_t ow) {
    for (size_t ni = 0; ni < n; ni++)
        for (size_t ci = 0; ci < c; ci++)
            for (size_t oy = 0; oy < oh; oy++)
                for (size_t ox = 0; ox < ow; ox++) {
                    float best = -INFINITY;
                    for (size_t ky = 0; ky < kh; ky++) {
                        size_t y = oy * sh + ky;
                        if (y < ph || y - ph >= h) continue;
                        for (size_t kx = 0; kx < kw; kx++) {
                            size_t x = ox * sw + kx;
                            if (x < pw || x - pw >= w) continue;
                            float v = in[((ni * c + ci) * h + (y - ph)) * w + (x - pw)];
                            if (v > best) best = v;
                        }
                    }
                    out[((ni * c + ci) * oh + oy) * ow + ox] = best;
                }
}

/* kernels.rs:335-390: count_include_pad = 0, sequential sum, acc / count */
void tpto_average_pool2d(const float *in, size_t n, size_t c, size_t h, size_t w,
                         size_t kh, size_t kw, size_t sh, size_t sw, size_t ph, size_t pw,
                         float *out, size_t oh, size_t ow) {
    for (size_t ni = 0; ni < n; ni++)
        for (size_t ci = 0; ci < c; ci++)
            for (size_t oy = 0; oy < oh; oy++)
                for (size_t ox = 0; ox < ow; ox++) {
                    float acc = 0.0f;
                    size_t count = 0;
                    for (size_t ky = 0; ky < kh; ky++) {
                        size_t y = oy * sh + ky;
                        if (y < ph || y - ph >= h) continue;
                        for (size_t kx = 0; kx < kw; kx++) {
                            size_t x = ox * sw + kx;
                            if (x < pw || x - pw >= w) continue;
                            acc += in[((ni * c + ci) * h + (y - ph)) * w + (x - pw)];
                            count++;
                        }
                    }
                    out[((ni * c + ci) * oh + oy) * ow + ox] = count == 0 ? 0.0f : acc / (float)count;
                }
}

/* kernels.rs:150-178 with bias dims [1,C,1,1] against [N,C,H,W] */
void tpto_add_bias_nchw(float *out, size_t n, size_t c, size_t hw, const float *bias) {
    for (size_t ni = 0; ni < n; ni++)
        for (size_t ci = 0; ci < c; ci++)
            for (size_t i = 0; i < hw; i++) out[(ni * c + ci) * hw + i] += bias[ci];
}

/* kernels.rs:150-178 with bias dims [cols] against [rows, cols] */
void tpto_add_bias_rows(float *out, size_t rows, size_t cols, const float *bias) {
    for (size_t r = 0; r < rows; r++)
        for (size_t j = 0; j < cols; j++) out[r * cols + j] += bias[j];
}

/* LayerNorm as this backend defines it (the reference has none:
 * crates/tpt-infer-onnx/src/registry.rs:62 maps LayerNormalization to Custom):
 * ONNX semantics over the last axis, biased variance, evaluated in the device
 * kernels' order (tpt_infer_b200/csrc/model_ops.cu k_layernorm / k_layernorm4):
 * 32 lanes, lane l owning columns l + 32 i (cols != 768) or the float4 groups
 * 4 (l + 32 i) .. +3 (cols == 768); sequential partial sums per lane, a xor
 * butterfly (o = 16, 8, 4, 2, 1) across lanes, mean = s / cols, variance by
 * fmaf(d, d, q) in the same order, inv = 1 / sqrtf(var + eps),
 * y = fmaf((x - mean) * inv, gamma, beta). res (may be NULL) is added first. */
static float ln_butterfly(float p[32]) {
    float t[32];
    for (int o = 16; o > 0; o >>= 1) {
        for (int l = 0; l < 32; l++) t[l] = p[l] + p[l ^ o];
        memcpy(p, t, sizeof t);
    }
    return p[0];
}

void tpto_layernorm_res(const float *x, const float *res, size_t rows, size_t cols, const float *gamma,
                        const float *beta, float eps, float *y) {
    const int vec4 = cols == 768;
    float *v = malloc(cols * sizeof(float));
    for (size_t r = 0; r < rows; r++) {
        const float *xr = x + r * cols;
        for (size_t c = 0; c < cols; c++) v[c] = res ? xr[c] + res[r * cols + c] : xr[c];
        float p[32], q[32];
        for (int l = 0; l < 32; l++) {
            float s = 0.0f;
            if (vec4) {
                for (size_t gi = (size_t)l; gi < cols / 4; gi += 32) {
                    const float *e = v + 4 * gi;
                    s = s + (((e[0] + e[1]) + e[2]) + e[3]);
                }
            } else {
                for (size_t i = 0; i < 32; i++) {
                    size_t c = (size_t)l + 32 * i;
                    s = s + (c < cols ? v[c] : 0.0f);
                }
            }
            p[l] = s;
        }
        const float mean = ln_butterfly(p) / (float)cols;
        for (int l = 0; l < 32; l++) {
            float a = 0.0f;
            if (vec4) {
                for (size_t gi = (size_t)l; gi < cols / 4; gi += 32)
                    for (int j = 0; j < 4; j++) {
                        float d = v[4 * gi + j] - mean;
                        a = fmaf(d, d, a);
                    }
            } else {
                for (size_t i = 0; i < 32; i++) {
                    size_t c = (size_t)l + 32 * i;
                    float d = c < cols ? v[c] - mean : 0.0f;
                    a = fmaf(d, d, a);
                }
            }
            q[l] = a;
        }
        const float var = ln_butterfly(q) / (float)cols;
        const float inv = 1.0f / sqrtf(var + eps);
        for (size_t c = 0; c < cols; c++) y[r * cols + c] = fmaf((v[c] - mean) * inv, gamma[c], beta[c]);
    }
    free(v);
}

void tpto_layernorm(const float *x, size_t rows, size_t cols, const float *gamma, const float *beta, float eps,
                    float *y) {
    tpto_layernorm_res(x, NULL, rows, cols, gamma, beta, eps, y);
}

/* ------------------------------------------------------------------ */
/* The rest of the runtime's dispatch table (exec.rs:347-533)          */
/* ------------------------------------------------------------------ */

/* kernels::binary (crates/tpt-infer-runtime/src/kernels.rs:92-137): numpy
 * broadcasting over dims padded to rank 8 (pad, :33-41; map_coord, :60-66),
 * out[i] = a[ai] op b[bi], op 0 add 1 sub 2 mul 3 div. Shapes were checked by
 * the caller (check_broadcast, :43-58). */
void tpto_binary(int op, const float *a, const size_t *ad, size_t ar, const float *b, const size_t *bd, size_t br,
                 float *out, const size_t *od, size_t orank) {
    size_t A[8], B[8], O[8], n = 1;
    for (int d = 0; d < 8; d++) A[d] = B[d] = O[d] = 1;
    for (size_t d = 0; d < ar; d++) A[8 - ar + d] = ad[d];
    for (size_t d = 0; d < br; d++) B[8 - br + d] = bd[d];
    for (size_t d = 0; d < orank; d++) O[8 - orank + d] = od[d];
    for (int d = 0; d < 8; d++) n *= O[d];
    for (size_t i = 0; i < n; i++) {
        size_t rem = i, ai = 0, bi = 0, as = 1, bs = 1;
        for (int d = 7; d >= 0; d--) {
            size_t c = rem % O[d];
            rem /= O[d];
            ai += (A[d] == 1 ? 0 : c) * as;
            as *= A[d];
            bi += (B[d] == 1 ? 0 : c) * bs;
            bs *= B[d];
        }
        float x = a[ai], y = b[bi];
        out[i] = op == 0 ? x + y : op == 1 ? x - y : op == 2 ? x * y : x / y;
    }
}

/* sqrt_f32 (kernels.rs:397-411): the exponent halved through the bits, four
 * Newton steps. */
static float sqrt_ref(float x) {
    if (x != x || x < 0.0f) return NAN;
    if (x == 0.0f || isinf(x)) return x;
    uint32_t u;
    memcpy(&u, &x, 4);
    u = (u >> 1) + (1u << 29);
    float y;
    memcpy(&y, &u, 4);
    for (int i = 0; i < 4; i++) y = 0.5f * (y + x / y);
    return y;
}

/* kernels::batch_norm (kernels.rs:425-476), channel mode (x [N, C, H, W],
 * plen = C: hw = H*W) or element mode (hw = 0, plen = n). */
void tpto_batch_norm(const float *x, size_t n, const float *scale, const float *bias, const float *mean,
                     const float *var, size_t plen, size_t hw, float eps, float *out) {
    if (hw) {
        size_t c = plen, nb = n / (c * hw);
        for (size_t ni = 0; ni < nb; ni++)
            for (size_t ci = 0; ci < c; ci++) {
                float inv = 1.0f / sqrt_ref(var[ci] + eps);
                float f = scale[ci] * inv;
                float g = bias[ci] - mean[ci] * f;
                size_t base = (ni * c + ci) * hw;
                for (size_t i = base; i < base + hw; i++) out[i] = x[i] * f + g;
            }
    } else {
        for (size_t i = 0; i < n; i++) {
            float inv = 1.0f / sqrt_ref(var[i] + eps);
            float f = scale[i] * inv;
            out[i] = (x[i] - mean[i]) * f + bias[i];
        }
    }
}

/* kernels::transpose (kernels.rs:484-532): out axis d reads input axis perm[d]. */
void tpto_transpose(const float *x, const size_t *xd, size_t rank, const size_t *perm, float *out) {
    size_t od[8], xs[8], n = 1, s = 1;
    for (size_t d = 0; d < rank; d++) od[d] = xd[perm[d]];
    for (size_t d = rank; d-- > 0;) {
        xs[d] = s;
        s *= xd[d];
    }
    for (size_t d = 0; d < rank; d++) n *= od[d];
    for (size_t i = 0; i < n; i++) {
        size_t rem = i, xi = 0;
        for (size_t d = rank; d-- > 0;) {
            size_t c = rem % od[d];
            rem /= od[d];
            xi += c * xs[perm[d]];
        }
        out[i] = x[xi];
    }
}

/* kernels::concat_copy_one (kernels.rs:548-588) */
void tpto_concat_copy_one(float *out, size_t c_total, size_t c_offset, size_t c_src, size_t inner, const float *src,
                          size_t src_len) {
    size_t sb = c_src * inner, ob = c_total * inner, outer = src_len / sb;
    for (size_t o = 0; o < outer; o++) memcpy(out + o * ob + c_offset * inner, src + o * sb, sb * 4);
}


/* The fused attention of the encoder plans on the integer tensor cores
 * (tpt_infer_b200/csrc/attention_i8.cu), restated: three 8-bit digits per
 * value (scale sc = amax * r127 per Q and K row and per V column, r127 the f32
 * nearest 1/127, digits of x * (1/sc); P with u = 127 p),
 * exact integer sums of the digit products up to order 2, recombined in f32 in
 * a fixed order; softmax with exp_det, quarters of 32 keys summed in order then
 * ((q0 + q1) + q2) + q3. qkv [B*S, 3*H*64], out [B*S, H*64]; batches [b0, b1). */
static void digits3(float x, float inv, int *d0, int *d1, int *d2) {
    const float u = x * inv;
    if (u != u) {
        *d0 = *d1 = *d2 = 0;
        return;
    }
    const float a = rintf(u);
    const float r1 = (u - a) * 128.0f;
    const float b = rintf(r1);
    const float r2 = (r1 - b) * 128.0f;
    *d0 = (int)a;
    *d1 = (int)b;
    *d2 = (int)rintf(r2);
}

static float combine3(int32_t t0, int32_t t1, int32_t t2) {
    float t = (float)t2 * 0x1p-14f;
    t = fmaf((float)t1, 0x1p-7f, t);
    return (float)t0 + t;
}

void tpto_attention_i8(const float *qkv, size_t B, size_t S, size_t H, float scale, float *out, size_t b0,
                       size_t b1) {
    (void)B;
    const size_t D = 64, HD = H * D, ld = 3 * HD;
#pragma omp parallel for collapse(2) schedule(static)
    for (size_t b = b0; b < b1; b++)
        for (size_t h = 0; h < H; h++) {
            const float *src = qkv + b * S * ld + h * D;
            static _Thread_local int8_t qd[3][128][64], kd[3][128][64], vd[3][128][64], pd[3][128];
            static _Thread_local float qsc[128], ksc[128], vps[64];
            for (size_t r = 0; r < 128; r++)
                for (int which = 0; which < 2; which++) {
                    float x[64], amax = 0.0f;
                    for (size_t d = 0; d < D; d++) {
                        float v = r < S ? src[r * ld + (which ? HD : 0) + d] : 0.0f;
                        x[d] = which ? v : v * scale;
                        amax = fmaxf(amax, fabsf(x[d]));
                    }
                    const float sc = amax * 0.00787401572f;
                    const float inv = amax > 0.0f ? 1.0f / sc : 0.0f;
                    for (size_t d = 0; d < D; d++) {
                        int a0, a1, a2;
                        digits3(x[d], inv, &a0, &a1, &a2);
                        int8_t(*t)[128][64] = which ? kd : qd;
                        t[0][r][d] = (int8_t)a0;
                        t[1][r][d] = (int8_t)a1;
                        t[2][r][d] = (int8_t)a2;
                    }
                    (which ? ksc : qsc)[r] = sc;
                }
            for (size_t d = 0; d < D; d++) {
                float amax = 0.0f;
                for (size_t c = 0; c < 128; c++) amax = fmaxf(amax, fabsf(c < S ? src[c * ld + 2 * HD + d] : 0.0f));
                const float sc = amax * 0.00787401572f;
                vps[d] = sc * 0.00787401572f;
                const float inv = amax > 0.0f ? 1.0f / sc : 0.0f;
                for (size_t c = 0; c < 128; c++) {
                    int e0, e1, e2;
                    digits3(c < S ? src[c * ld + 2 * HD + d] : 0.0f, inv, &e0, &e1, &e2);
                    vd[0][c][d] = (int8_t)e0;
                    vd[1][c][d] = (int8_t)e1;
                    vd[2][c][d] = (int8_t)e2;
                }
            }
            for (size_t r = 0; r < S; r++) {
                float sv[128];
                for (size_t c = 0; c < 128; c++) {
                    int32_t t0 = 0, t1 = 0, t2 = 0;
                    for (size_t d = 0; d < D; d++) {
                        const int a0 = qd[0][r][d], a1 = qd[1][r][d], a2 = qd[2][r][d];
                        const int c0 = kd[0][c][d], c1 = kd[1][c][d], c2 = kd[2][c][d];
                        t0 += a0 * c0;
                        t1 += a0 * c1 + a1 * c0;
                        t2 += a0 * c2 + a1 * c1 + a2 * c0;
                    }
                    sv[c] = combine3(t0, t1, t2) * (qsc[r] * ksc[c]);
                }
                float m = -INFINITY;
                for (size_t c = 0; c < S; c++) m = fmaxf(m, sv[c]);
                float part[4];
                for (int q = 0; q < 4; q++) {
                    float acc = 0.0f;
                    for (int j = 0; j < 32; j++) {
                        const size_t c = (size_t)(32 * q + j);
                        const float e = c < S ? tpto_exp_det(sv[c] - m) : 0.0f;
                        sv[c] = e;
                        acc = acc + e;
                    }
                    part[q] = acc;
                }
                const float rs = 1.0f / (((part[0] + part[1]) + part[2]) + part[3]);
                for (size_t c = 0; c < 128; c++) {
                    int p0, p1, p2;
                    digits3(sv[c], 127.0f, &p0, &p1, &p2);  /* digits of e; 1 / sum on the context */
                    pd[0][c] = (int8_t)p0;
                    pd[1][c] = (int8_t)p1;
                    pd[2][c] = (int8_t)p2;
                }
                float *orow = out + (b * S + r) * HD + h * D;
                for (size_t d = 0; d < D; d++) {
                    int32_t u0 = 0, u1 = 0, u2 = 0;
                    for (size_t c = 0; c < 128; c++) {
                        const int p0 = pd[0][c], p1 = pd[1][c], p2 = pd[2][c];
                        const int e0 = vd[0][c][d], e1 = vd[1][c][d], e2 = vd[2][c][d];
                        u0 += p0 * e0;
                        u1 += p0 * e1 + p1 * e0;
                        u2 += p0 * e2 + p1 * e1 + p2 * e0;
                    }
                    orow[d] = (combine3(u0, u1, u2) * vps[d]) * rs;
                }
            }
        }
}
