/*
 * tpt_oracle.h -- CPU restatement of tpt-infer's reference CPU kernels.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * backend and the timed CPU baseline. Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline / reference legs may load it. The CUDA product
 * path never links or calls it and has no CPU fallback.
 *
 * Parity is pinned by the reference's own known-answer tests (the KATs in
 * crates/tpt-infer-ops/src/naive.rs, crates/tpt-infer-quantize/src/quant.rs,
 * dequant.rs, ptq.rs and crates/tpt-infer-runtime/src/kernels.rs), which the
 * pytest suite replays against these functions. The reference itself is
 * Rust and no Rust toolchain exists here, so it cannot be built or run.
 *
 * Every function restates one reference function; the citation in front of
 * each names the file:line range it follows. Floating-point functions are
 * compiled with -ffp-contract=off so that "mul then add" stays two roundings,
 * exactly as the Rust code (which never contracts to FMA) computes it.
 *
 * Status codes mirror OpError (crates/tpt-infer-ops/src/backend.rs:6-20).
 */
#ifndef TPT_ORACLE_H
#define TPT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    TPTO_OK = 0,
    TPTO_SIZE_MISMATCH = 1,
    TPTO_SHAPE_MISMATCH = 2,
    TPTO_UNSUPPORTED = 3,
    TPTO_INVALID = 4,
};

/* Out-parameters of the last SIZE_MISMATCH (expected, actual). Per thread. */
void tpto_last_size_mismatch(size_t *expected, size_t *actual);

/* ---- seeded generators (test LCG of crates/tpt-infer-ops/src/dispatch.rs:274-282) ---- */
void tpto_lcg_sym(float *out, size_t n, uint32_t seed);      /* [-1, 1), exactly dispatch.rs */
void tpto_lcg_uniform(float *out, size_t n, uint32_t seed);  /* [0, 1) = (s>>8)/2^24 */
void tpto_normal(float *out, size_t n, uint32_t seed, float mean, float std); /* Box-Muller on LCG pairs */

/* ---- Backend ops (naive.rs / avx512.rs) ---- */
int tpto_matmul_naive(const float *a, size_t a_len, size_t m, size_t k,
                      const float *b, size_t b_len, size_t kb, size_t n,
                      float *out, size_t out_len);
int tpto_gemm(const float *a, size_t a_len, size_t m, size_t k, int trans_a,
              const float *b, size_t b_len, size_t n, int trans_b,
              const float *c, size_t c_len, float alpha, float beta,
              float *out, size_t out_len);
int tpto_matmul_avx(const float *a, size_t a_len, size_t m, size_t k,
                    const float *b, size_t b_len, size_t kb, size_t n,
                    float *out, size_t out_len, int threads);
int tpto_conv2d(const float *in, size_t in_len, const size_t in_shape[4],
                const float *w, size_t w_len, const size_t w_shape[4],
                float *out, size_t out_len, size_t stride_h, size_t stride_w,
                size_t pad_h, size_t pad_w, int threads);
int tpto_elementwise_add(const float *a, size_t a_len, const float *b, size_t b_len,
                         float *out, size_t out_len);
int tpto_relu(const float *a, size_t a_len, float *out, size_t out_len);
int tpto_softmax(const float *a, size_t a_len, float *out, size_t out_len, size_t row_len);
int tpto_sigmoid(const float *a, size_t a_len, float *out, size_t out_len);
int tpto_gelu(const float *a, size_t a_len, float *out, size_t out_len);

/* ---- quantize crate (quant.rs / dequant.rs / ptq.rs) ---- */
float tpto_quantize_i8_symmetric(const float *x, size_t n, int8_t *q);
void tpto_quantize_i8_asymmetric(const float *x, size_t n, int8_t *q, float *scale, int32_t *zp);
int tpto_quantize_i8_symmetric_per_channel(const float *x, size_t len, size_t rows,
                                           int8_t *q, float *scales);
/* returns TPTO_INVALID where the reference panics (value outside [-8,7]) */
int tpto_pack_i4(const int8_t *v, size_t n, uint8_t *out);
size_t tpto_unpack_i4(const uint8_t *packed, size_t packed_len, size_t n, int8_t *out);
float tpto_quantize_i4_symmetric(const float *x, size_t n, uint8_t *packed);
int tpto_quantize_i4_symmetric_per_channel(const float *x, size_t len, size_t rows,
                                           uint8_t *packed, float *scales);
void tpto_dequantize_i8_symmetric(const int8_t *q, size_t n, float scale, float *out);
void tpto_dequantize_i8_asymmetric(const int8_t *q, size_t n, float scale, int32_t zp, float *out);
int tpto_dequantize_i8_symmetric_per_channel(const int8_t *q, size_t n, const float *scales,
                                             size_t n_scales, float *out);
void tpto_dequantize_i4_symmetric(const uint8_t *packed, size_t packed_len, size_t n,
                                  float scale, float *out);
void tpto_dequantize_i4_symmetric_per_channel(const uint8_t *packed, size_t packed_len,
                                              size_t row_elems, const float *scales,
                                              size_t n_scales, float *out);
/* ptq.rs:293-324, per-tensor, B laid out [k,n]; returns TPTO_SHAPE_MISMATCH /
 * TPTO_SIZE_MISMATCH where the reference returns Err(String). */
int tpto_quantized_matmul_i8(const int8_t *a, size_t a_len, size_t m, size_t k, float a_scale,
                             const int8_t *b, size_t b_len, size_t kb, size_t n,
                             const float *b_scales, size_t n_scales, float *out, size_t out_len);

/* ---- definitions the reference lacks, fixed once here (per-channel W8A8, W4) ---- */
enum { TPTO_ACT_NONE = 0, TPTO_ACT_RELU = 1, TPTO_ACT_GELU = 2 };
/* Integer accumulators acc[m,n] = sum_k a[m,k]*wt[n,k] (wt is W^T, [N,K] row-major). */
void tpto_i8_gemm_acc(const int8_t *a, const int8_t *wt, size_t m, size_t n, size_t k,
                      int32_t *acc, int threads);
/* y = (float)acc*(a_scale*w_scale[n]) + bias[n]; then act */
void tpto_w8a8_gemm(const int8_t *a, const int8_t *wt, size_t m, size_t n, size_t k,
                    float a_scale, const float *w_scales, const float *bias, int act,
                    float *y, int threads);
/* The reference's own loop order (ptq.rs:312-319, B = [k,n], strided) with the
 * per-channel + bias epilogue; rows [row0,row1) only. Used as the timed CPU
 * reference arm. */
void tpto_w8a8_gemm_refloop(const int8_t *a, const int8_t *b_kn, size_t m, size_t n, size_t k,
                            float a_scale, const float *w_scales, const float *bias,
                            float *y, size_t row0, size_t row1, int threads);
float tpto_requant_i8(float y, float out_scale, int8_t *q);
void tpto_quantize_i8_static(const float *x, size_t n, float scale, int8_t *q);
float tpto_absmax(const float *x, size_t n);
/* W4 reference: dequantize_i4_symmetric_per_channel (dequant.rs:56-71) then the
 * f32 matmul of avx512.rs:55-78, with W^T nibble rows [N, ceil(K/2)]. */
void tpto_w4_gemm(const float *x, const uint8_t *wt_packed, const float *w_scales,
                  size_t m, size_t n, size_t k, const float *bias, int act, float *y, int threads);

/* ---- runtime kernels (crates/tpt-infer-runtime/src/kernels.rs) ---- */
void tpto_max_pool2d(const float *in, size_t n, size_t c, size_t h, size_t w,
                     size_t kh, size_t kw, size_t sh, size_t sw, size_t ph, size_t pw,
                     float *out, size_t oh, size_t ow);
void tpto_average_pool2d(const float *in, size_t n, size_t c, size_t h, size_t w,
                         size_t kh, size_t kw, size_t sh, size_t sw, size_t ph, size_t pw,
                         float *out, size_t oh, size_t ow);
/* out[N,C,H,W] += bias[C]  (add_inplace_broadcast with bias dims [1,C,1,1]) */
void tpto_add_bias_nchw(float *out, size_t n, size_t c, size_t hw, const float *bias);
/* out[rows, cols] += bias[cols] */
void tpto_add_bias_rows(float *out, size_t rows, size_t cols, const float *bias);
/* LayerNormalization over the last axis (ONNX semantics, biased variance). */
void tpto_layernorm(const float *x, size_t rows, size_t cols, const float *gamma,
                    const float *beta, float eps, float *y);

/* The rest of the runtime's dispatch table (kernels.rs) */
void tpto_binary(int op, const float *a, const size_t *ad, size_t ar, const float *b, const size_t *bd, size_t br,
                 float *out, const size_t *od, size_t orank);
void tpto_batch_norm(const float *x, size_t n, const float *scale, const float *bias, const float *mean,
                     const float *var, size_t plen, size_t hw, float eps, float *out);
void tpto_transpose(const float *x, const size_t *xd, size_t rank, const size_t *perm, float *out);
void tpto_concat_copy_one(float *out, size_t c_total, size_t c_offset, size_t c_src, size_t inner, const float *src,
                          size_t src_len);

/* deterministic exp / GELU of the device (det_math.cuh) */
float tpto_exp_det(float x);
float tpto_gelu_det(float x);
void tpto_gelu_det_array(const float *a, size_t n, float *out);
void tpto_exp_det_array(const float *a, size_t n, float *out);

void tpto_layernorm_res(const float *x, const float *res, size_t rows, size_t cols, const float *gamma,
                        const float *beta, float eps, float *y);


void tpto_attention_i8(const float *qkv, size_t B, size_t S, size_t H, float scale, float *out, size_t b0,
                       size_t b1);

#ifdef __cplusplus
}
#endif
#endif
