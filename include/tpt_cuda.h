/*
 * tpt_cuda.h -- C ABI of the B200 (sm_100a) CUDA backend for tpt-infer.
 *
 * This is the boundary a tpt-infer `CudaBackend` binds through `extern "C"`:
 * plain pointers and sizes, no CUDA or torch types in any signature. Every
 * entry point names the reference interface it replaces (paths relative to the
 * tpt-infer repository root).
 *
 * Conventions
 *  - Every function returns a tpt_status. Validation happens before any device
 *    work and follows the reference's checks in the reference's order, so a
 *    call the reference rejects is rejected here with the same OpError
 *    variant (crates/tpt-infer-ops/src/backend.rs:6-20, 149-284).
 *    TPT_SIZE_MISMATCH additionally records (expected, actual), readable with
 *    tpt_cuda_last_size_mismatch().
 *  - Functions without a `_dev` suffix take HOST buffers (the `&[f32]` slices
 *    of the Backend trait), stage them to the device on the context's stream
 *    and return after the result is back in host memory. Pinned host memory
 *    makes the copies faster but is not required.
 *  - `_dev` functions take DEVICE pointers, enqueue on the context's stream and
 *    return without synchronising (tpt_cuda_ctx_sync waits).
 *  - Calls on one context are serialised on its stream. One context per GPU;
 *    use one host thread per context for several GPUs.
 *  - There is no CPU fallback: an op the CUDA path lacks returns
 *    TPT_UNSUPPORTED.
 */
#ifndef TPT_CUDA_H
#define TPT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. 1-4 mirror OpError (crates/tpt-infer-ops/src/backend.rs:6-20):
 * SizeMismatch{expected, actual}, ShapeMismatch, Unsupported, Invalid. */
typedef enum tpt_status {
    TPT_OK = 0,
    TPT_SIZE_MISMATCH = 1,
    TPT_SHAPE_MISMATCH = 2,
    TPT_UNSUPPORTED = 3,
    TPT_INVALID = 4,
    TPT_CUDA_ERROR = 5,   /* a CUDA runtime/driver call failed (message: tpt_cuda_last_error) */
    TPT_OUT_OF_MEMORY = 6,/* device arena or allocation exhausted (TensorError::OutOfMemory) */
    TPT_TIMEOUT = 7,      /* a bounded device-side wait ran out; the kernel returned early */
    TPT_NCCL_ERROR = 8,
    TPT_DEVICE_CHECK = 9  /* a kernel's own bounds/alignment check recorded a violation */
} tpt_status;

/* Epilogue activation (the Relu / Gelu nodes of exec.rs:416-445, fused). */
typedef enum tpt_act { TPT_ACT_NONE = 0, TPT_ACT_RELU = 1, TPT_ACT_GELU = 2 } tpt_act;

typedef struct tpt_cuda_ctx tpt_cuda_ctx;
typedef struct tpt_cuda_weights tpt_cuda_weights;

/* ------------------------------------------------------------------ */
/* Context                                                             */
/* ------------------------------------------------------------------ */

/* Creates a context on `device`. `stream` is a cudaStream_t passed as void*;
 * NULL makes the context create and own a non-blocking stream. Replaces the
 * zero-sized CPU backends' construction and WebGpuBackend::new() -> Option
 * (crates/tpt-infer-ops/src/webgpu.rs:272); a machine without a usable sm_100
 * device yields TPT_UNSUPPORTED. */
int tpt_cuda_ctx_create(int device, void *stream, tpt_cuda_ctx **out);
int tpt_cuda_ctx_destroy(tpt_cuda_ctx *ctx);
/* Waits for the context's stream; reports device-side error words
 * (TPT_TIMEOUT / TPT_DEVICE_CHECK) raised by earlier _dev launches. */
int tpt_cuda_ctx_sync(tpt_cuda_ctx *ctx);
/* The context's stream (cudaStream_t as void*). */
void *tpt_cuda_ctx_stream(tpt_cuda_ctx *ctx);
int tpt_cuda_ctx_device(tpt_cuda_ctx *ctx);
/* Backend::name (crates/tpt-infer-ops/src/backend.rs:100): "cuda". */
const char *tpt_cuda_backend_name(void);
const char *tpt_cuda_status_str(int status);
/* Text of the last CUDA error on this context ("" if none). */
const char *tpt_cuda_last_error(tpt_cuda_ctx *ctx);
/* (expected, actual) of the last TPT_SIZE_MISMATCH on this context. */
void tpt_cuda_last_size_mismatch(tpt_cuda_ctx *ctx, size_t *expected, size_t *actual);
/* Number of kernels this library launched on the context since creation. */
uint64_t tpt_cuda_ctx_launch_count(tpt_cuda_ctx *ctx);
/* Bound of the device-side waits in this context's kernels, in SM clock
 * cycles (0 = the default of 2e9 cycles, about 1 s at the B200's boost clock).
 * Every mbarrier wait in the tensor-core and TMA-ring kernels is bounded; a
 * wait that runs out makes the kernel leave its loops, wait (with the default
 * bound) for its own copies and MMAs still in flight, free its tensor memory
 * and return, and the next synchronising call reports TPT_TIMEOUT. A short
 * bound makes a normal launch run out, so the timeout path can be exercised
 * without a stuck GPU. No counterpart in the reference (a CPU runtime). */
int tpt_cuda_ctx_set_wait_limit(tpt_cuda_ctx *ctx, uint32_t cycles);
/* Self-test of that mechanism: one CTA waits, through the same bounded wait,
 * on a barrier nothing arrives on. *outcome receives bit 0 = the wait
 * succeeded (never expected), bit 1 = the CTA's abort was raised. Returns
 * TPT_TIMEOUT when the expiry was recorded and reported, as a real kernel's
 * would be; the context stays usable. Takes the context's wait limit. */
int tpt_cuda_selftest_bounded_wait(tpt_cuda_ctx *ctx, unsigned *outcome);

/* CUDA graphs of device-pointer calls. The reference runtime walks the graph
 * node by node on every call (crates/tpt-infer-runtime/src/exec.rs:570-635);
 * on the device a fixed sequence of launches is recorded once and replayed
 * with one launch. tpt_cuda_capture_begin starts recording what is issued on
 * the context's stream; tpt_cuda_capture_end ends it (always call it once
 * begin succeeded) and returns the graph. Only device-pointer (_dev) entry
 * points and tpt_cuda_plan_run_device can be recorded: a call that would
 * synchronise or grow a context workspace returns TPT_INVALID while
 * recording, so run each call once before recording it. A graph keeps the
 * context's workspace addresses: once a later call grows a workspace,
 * tpt_cuda_graph_launch returns TPT_INVALID and the graph must be recorded
 * again. */
typedef struct tpt_cuda_graph tpt_cuda_graph;
int tpt_cuda_capture_begin(tpt_cuda_ctx *ctx);
int tpt_cuda_capture_end(tpt_cuda_ctx *ctx, tpt_cuda_graph **graph);
/* enqueues one replay on the context's stream (async) */
int tpt_cuda_graph_launch(tpt_cuda_ctx *ctx, tpt_cuda_graph *graph);
/* kernels one replay launches */
uint64_t tpt_cuda_graph_kernels(const tpt_cuda_graph *graph);
int tpt_cuda_graph_destroy(tpt_cuda_graph *graph);

/* ------------------------------------------------------------------ */
/* Backend trait, host slices (crates/tpt-infer-ops/src/backend.rs:98-147) */
/* ------------------------------------------------------------------ */

/* Backend::matmul (backend.rs:106-113): out[m,n] = a[m,k] @ b[kb,n], f32.
 * Validation = validate_matmul (backend.rs:149-183). Each output is summed in
 * increasing k with separately rounded multiply and add, bit-identical to
 * naive.rs:13-33 / avx512.rs:55-78 (never TF32). */
int tpt_cuda_matmul(tpt_cuda_ctx *ctx, const float *a, size_t a_len, size_t m, size_t k,
                    const float *b, size_t b_len, size_t kb, size_t n, float *out, size_t out_len);
/* Backend::conv2d (backend.rs:119-127): NCHW input, OIHW weight, groups 1,
 * no bias; Conv2dOptions (backend.rs:49-58) passed as four sizes.
 * Validation = validate_conv2d (backend.rs:219-284). */
int tpt_cuda_conv2d(tpt_cuda_ctx *ctx, const float *input, size_t in_len, const size_t in_shape[4],
                    const float *weight, size_t w_len, const size_t w_shape[4], float *out,
                    size_t out_len, size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w);
/* Backend::elementwise_add (backend.rs:130) */
int tpt_cuda_elementwise_add(tpt_cuda_ctx *ctx, const float *a, size_t a_len, const float *b,
                             size_t b_len, float *out, size_t out_len);
/* Backend::relu (backend.rs:133) */
int tpt_cuda_relu(tpt_cuda_ctx *ctx, const float *a, size_t a_len, float *out, size_t out_len);
/* Backend::softmax (backend.rs:139), rows of row_len */
int tpt_cuda_softmax(tpt_cuda_ctx *ctx, const float *a, size_t a_len, float *out, size_t out_len,
                     size_t row_len);
/* Backend::sigmoid (backend.rs:142) */
int tpt_cuda_sigmoid(tpt_cuda_ctx *ctx, const float *a, size_t a_len, float *out, size_t out_len);
/* Backend::gelu (backend.rs:146), tanh approximation of naive.rs:137-146 */
int tpt_cuda_gelu(tpt_cuda_ctx *ctx, const float *a, size_t a_len, float *out, size_t out_len);

/* Device-pointer forms of the same ops (validated shapes, async). */
int tpt_cuda_matmul_dev(tpt_cuda_ctx *ctx, const float *a, size_t m, size_t k, const float *b,
                        size_t n, float *out);

/* ONNX Gemm: Y = alpha * op(A) op(B) + beta * C. tpt-infer's ONNX loader maps
 * "Gemm" to a plain MatMul and drops transA/transB/alpha/beta/C
 * (crates/tpt-infer-onnx/src/registry.rs:21, load.rs:410-445); this is the full
 * semantics. op(A) is A [m,k], or A^T of a stored [k,m] when trans_a; op(B) is
 * B [k,n], or B^T of a stored [n,k] when trans_b. C is [n] (broadcast over rows)
 * or [m,n]; c_len = 0 (c may be NULL) means no C term. Sequential k with a
 * separately rounded multiply and add per term (the MatMul arithmetic), then
 * alpha*acc + beta*c, each product and the sum rounded separately. Errors:
 * SIZE_MISMATCH for a_len, b_len, out_len; SHAPE_MISMATCH for another c_len. */
int tpt_cuda_gemm(tpt_cuda_ctx *ctx, const float *a, size_t a_len, size_t m, size_t k, int trans_a,
                  const float *b, size_t b_len, size_t n, int trans_b, const float *c, size_t c_len,
                  float alpha, float beta, float *out, size_t out_len);
int tpt_cuda_gemm_dev(tpt_cuda_ctx *ctx, const float *a, size_t m, size_t k, int trans_a, const float *b,
                      size_t n, int trans_b, const float *c, size_t c_len, float alpha, float beta, float *out);
int tpt_cuda_conv2d_dev(tpt_cuda_ctx *ctx, const float *input, const size_t in_shape[4],
                        const float *weight, const size_t w_shape[4], float *out,
                        size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w);
int tpt_cuda_elementwise_add_dev(tpt_cuda_ctx *ctx, const float *a, const float *b, float *out, size_t n);
int tpt_cuda_relu_dev(tpt_cuda_ctx *ctx, const float *a, float *out, size_t n);
int tpt_cuda_softmax_dev(tpt_cuda_ctx *ctx, const float *a, float *out, size_t n, size_t row_len);
int tpt_cuda_sigmoid_dev(tpt_cuda_ctx *ctx, const float *a, float *out, size_t n);
int tpt_cuda_gelu_dev(tpt_cuda_ctx *ctx, const float *a, float *out, size_t n);

/* ------------------------------------------------------------------ */
/* Quantization (crates/tpt-infer-quantize/src/{quant,dequant,ptq}.rs)  */
/* ------------------------------------------------------------------ */

/* quantize_i8_symmetric (quant.rs:25-40): per-tensor, scale = max|x|/127
 * (1.0 for an all-zero tensor), q = clamp(round_half_away(x/scale), -127, 127).
 * Bit-exact with the reference. */
int tpt_cuda_quantize_i8_symmetric(tpt_cuda_ctx *ctx, const float *x, size_t n, int8_t *q,
                                   float *scale);
/* quantize_i8_symmetric_per_channel (quant.rs:95-107): one scale per row of
 * a [rows, len/rows] view. len % rows != 0 or rows == 0 -> TPT_INVALID (the
 * reference asserts). */
int tpt_cuda_quantize_i8_symmetric_per_channel(tpt_cuda_ctx *ctx, const float *x, size_t len,
                                               size_t rows, int8_t *q, float *scales);
/* quantize_i8_asymmetric (quant.rs:45-90) */
int tpt_cuda_quantize_i8_asymmetric(tpt_cuda_ctx *ctx, const float *x, size_t n, int8_t *q,
                                    float *scale, int32_t *zero_point);
/* pack_i4 (quant.rs:123-140): low nibble first; out holds ceil(n/2) bytes.
 * A value outside [-8, 7] -> TPT_INVALID (the reference panics). */
int tpt_cuda_pack_i4(tpt_cuda_ctx *ctx, const int8_t *values, size_t n, uint8_t *out);
/* unpack_i4 (quant.rs:143-157): writes min(n, 2*packed_len) values,
 * count returned in *written. */
int tpt_cuda_unpack_i4(tpt_cuda_ctx *ctx, const uint8_t *packed, size_t packed_len, size_t n,
                       int8_t *out, size_t *written);
/* quantize_i4_symmetric (quant.rs:171-186): scale = max|x|/7, q in [-7, 7]. */
int tpt_cuda_quantize_i4_symmetric(tpt_cuda_ctx *ctx, const float *x, size_t n, uint8_t *packed,
                                   float *scale);
/* quantize_i4_symmetric_per_channel (quant.rs:192-204): rows padded to
 * ceil(cols/2) bytes. */
int tpt_cuda_quantize_i4_symmetric_per_channel(tpt_cuda_ctx *ctx, const float *x, size_t len,
                                               size_t rows, uint8_t *packed, float *scales);
/* dequantize_i8_symmetric (dequant.rs:13-15) */
int tpt_cuda_dequantize_i8_symmetric(tpt_cuda_ctx *ctx, const int8_t *q, size_t n, float scale,
                                     float *out);
/* dequantize_i8_asymmetric (dequant.rs:18-22): out = (q - zero_point) * scale,
 * the QuantParams of quantize_i8_asymmetric (quant.rs:6-12) passed as two values. */
int tpt_cuda_dequantize_i8_asymmetric(tpt_cuda_ctx *ctx, const int8_t *q, size_t n, float scale,
                                      int32_t zero_point, float *out);
/* dequantize_i8_symmetric_per_channel (dequant.rs:26-37) */
int tpt_cuda_dequantize_i8_symmetric_per_channel(tpt_cuda_ctx *ctx, const int8_t *q, size_t n,
                                                 const float *scales, size_t n_scales, float *out);
/* dequantize_i4_symmetric (dequant.rs:45-50): unpack_i4(packed, n) (quant.rs:143-157)
 * times one per-tensor scale; writes min(n, 2*packed_len) values, the count
 * returned in *written. */
int tpt_cuda_dequantize_i4_symmetric(tpt_cuda_ctx *ctx, const uint8_t *packed, size_t packed_len, size_t n,
                                     float scale, float *out, size_t *written);
/* dequantize_i4_symmetric_per_channel (dequant.rs:56-71); n_scales rows of
 * row_elems values, rows ceil(row_elems/2) bytes apart. */
int tpt_cuda_dequantize_i4_symmetric_per_channel(tpt_cuda_ctx *ctx, const uint8_t *packed,
                                                 size_t packed_len, size_t row_elems,
                                                 const float *scales, size_t n_scales, float *out);
/* quantized_matmul_i8 (crates/tpt-infer-quantize/src/ptq.rs:293-324), the
 * reference contract as is: B is [kb, n], per-tensor b_scales[0] (1.0 when
 * n_scales == 0), out = (float)acc * (a_scale * b_scale). Mismatched k ->
 * TPT_SHAPE_MISMATCH, mismatched buffer sizes -> TPT_SIZE_MISMATCH (the
 * reference's Err(String) cases). i32 accumulation, bit-exact. */
int tpt_cuda_quantized_matmul_i8(tpt_cuda_ctx *ctx, const int8_t *a, size_t a_len, size_t m,
                                 size_t k, float a_scale, const int8_t *b, size_t b_len, size_t kb,
                                 size_t n, const float *b_scales, size_t n_scales, float *out,
                                 size_t out_len);

/* Device-pointer forms used by the device-resident plans. */
/* quantize_i8_symmetric on device buffers; the per-tensor max-abs reduction
 * goes through a cell of context scratch. The scale lands in *scale_dev. */
int tpt_cuda_quantize_i8_symmetric_dev(tpt_cuda_ctx *ctx, const float *x, size_t n, int8_t *q,
                                       float *scale_dev);
/* q = clamp(round(x / scale), -127, 127) with a known (calibrated) scale. */
int tpt_cuda_quantize_i8_static_dev(tpt_cuda_ctx *ctx, const float *x, size_t n, float scale,
                                    int8_t *q);

/* ------------------------------------------------------------------ */
/* Packed quantized weights, uploaded once                              */
/* ------------------------------------------------------------------ */

/* Uploads an INT8 per-output-channel weight: `wt` is W^T as [n, k] row-major
 * int8 -- exactly the `packed` bytes of a QuantizedTensor produced by
 * quantize_i8_symmetric_per_channel(W^T, rows = n) (quant.rs:95-107,
 * ptq.rs:77-86) -- with n scales. k must be a multiple of 16. */
int tpt_cuda_weights_upload_i8(tpt_cuda_ctx *ctx, const int8_t *wt, const float *scales,
                               size_t n, size_t k, tpt_cuda_weights **out);
/* Uploads an INT4 per-output-channel weight: `packed` holds n rows of
 * k/2 bytes, low nibble first along k, exactly the bytes of
 * quantize_i4_symmetric_per_channel(W^T, rows = n) (quant.rs:192-204);
 * k must be a multiple of 32. */
int tpt_cuda_weights_upload_i4(tpt_cuda_ctx *ctx, const uint8_t *packed, size_t packed_len,
                               const float *scales, size_t n, size_t k, tpt_cuda_weights **out);
int tpt_cuda_weights_free(tpt_cuda_weights *w);
/* Shape of an uploaded weight (n output channels, k inputs). */
int tpt_cuda_weights_shape(const tpt_cuda_weights *w, size_t *n, size_t *k);

/* W8A8 GEMM with per-output-channel weights: the per-channel extension of
 * quantized_matmul_i8 (ptq.rs:293-324). acc[m,n] = sum_k a[m,k]*wt[n,k] in
 * i32, then y = (float)acc * (a_scale * w_scale[n]) + bias[n] (two roundings,
 * no FMA; bias may be NULL), then `act`. Host buffers: a is [m, k] int8,
 * out is [m, n] f32. */
int tpt_cuda_w8a8_gemm(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, size_t k, float a_scale,
                       const tpt_cuda_weights *w, const float *bias, int act, float *out);
/* Same on device pointers (async). */
int tpt_cuda_w8a8_gemm_dev(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, float a_scale,
                           const tpt_cuda_weights *w, const float *bias, int act, float *out);
/* Same, writing the raw i32 accumulators instead (bit-exactness checks). */
int tpt_cuda_w8a8_gemm_acc_dev(tpt_cuda_ctx *ctx, const int8_t *a, size_t m,
                               const tpt_cuda_weights *w, int32_t *acc);

/* W4 GEMM, f32 activations: y = x @ dequant(W4)^T + bias, then act -- the
 * reference semantics of dequantize_i4_symmetric_per_channel (dequant.rs:56-71)
 * followed by the f32 matmul. Host buffers x [m, k], out [m, n]. */
int tpt_cuda_w4_gemm(tpt_cuda_ctx *ctx, const float *x, size_t m, size_t k,
                     const tpt_cuda_weights *w, const float *bias, int act, float *out);
int tpt_cuda_w4_gemm_dev(tpt_cuda_ctx *ctx, const float *x, size_t m, const tpt_cuda_weights *w,
                         const float *bias, int act, float *out);

/* ------------------------------------------------------------------ */
/* Device-resident plans (execute_graph on the device)                  */
/* ------------------------------------------------------------------ */

/* The device counterpart of execute_graph / required_arena_bytes
 * (crates/tpt-infer-runtime/src/exec.rs:117-131, 570-635): every activation
 * tensor gets a disjoint offset in ONE device arena allocated at finalize
 * (the reference's assign_offsets + single alloc_slice, exec.rs:276-294,595),
 * constants are uploaded once, ops run in order on the context's stream, and
 * host copies happen only at graph inputs and outputs (tpt_cuda_plan_run).
 * INT8 activations carry a per-tensor scale; a quantization point either has a
 * static scale (op.f0 > 0) or is calibrated: runs made with calibration on
 * record max|x| per point, tpt_cuda_plan_freeze_scales sets
 * scale = max / 127 (1.0 if max == 0), the quantize_i8_symmetric rule
 * (crates/tpt-infer-quantize/src/quant.rs:25-31). */
typedef struct tpt_cuda_plan tpt_cuda_plan;

enum { TPT_DT_F32 = 0, TPT_DT_I8 = 1 };

enum tpt_op_kind {
    TPT_OP_QUANTIZE = 1,        /* in0 f32 [d0] -> out i8, per-tensor scale; d1 != 0: the calibration max is
                                   reduced over the plan's communicator (a column-sharded tensor) */
    TPT_OP_LINEAR_W8A8 = 2,     /* in0 i8 [d0, w.k] x w -> out f32 [d0, w.n]; in1 bias (or -1); act */
    TPT_OP_MATMUL_F32 = 3,      /* in0 [d0,d1] x in1 [d1,d2] -> out; in2 bias (or -1); act (Backend::matmul) */
    TPT_OP_BIAS_ACT = 4,        /* out[d0,d1] = act(in0 + in1[d1]) (in1 may be -1) */
    TPT_OP_ADD_ACT = 5,         /* out[d0] = act(in0 + in1) (residual add) */
    TPT_OP_SOFTMAX = 6,         /* rows d0 of length d1 (Backend::softmax) */
    TPT_OP_LAYERNORM = 7,       /* rows d0 of d1; in1 gamma, in2 beta; eps f0 */
    TPT_OP_ATTENTION = 8,       /* in0 qkv [d0*d1, 3*d2*d3] -> out [d0*d1, d2*d3]; B=d0 S=d1 H=d2 D=d3; scale f0 */
    TPT_OP_NCHW_TO_NHWC_Q8 = 9, /* in0 f32 NCHW [d0, d1, d2=H*W] -> out i8 NHWC with d3 channels (d3 > d1:
                                   zero-padded; 0: d1), per-tensor scale. d5 = 2 (with d4 = W): space-to-depth,
                                   out [d0, H/2, W/2, 4*d3], channel (dy*2 + dx)*d3 + c */
    TPT_OP_IM2COL = 10,         /* in0 i8 NHWC -> out i8 [N*OH*OW, Kp]; d0..d12 = N,H,W,C,KH,KW,sh,sw,ph,pw,OH,OW,Kp */
    TPT_OP_MAXPOOL_NHWC = 11,   /* f32; d0..d11 = N,H,W,C,KH,KW,sh,sw,ph,pw,OH,OW */
    TPT_OP_GAP_NHWC = 12,       /* f32 [d0, d1=H*W, d2] -> [d0, d2] */
    TPT_OP_ALLGATHER = 13,      /* in0 [d0 elements] on every rank -> out [world * d0] in rank order (NCCL,
                                   on the context stream; the plan needs a communicator) */
    TPT_OP_PANELS_TO_ROWS = 14, /* i8 [d0 = P][d1 = T][d2 = C] -> i8 [T][P * C] (gathered column shards ->
                                   the K-contiguous rows of the next GEMM) */
    TPT_OP_GEMM_F32 = 15        /* ONNX Gemm: out [d0=m, d2=n] = f0 * op(in0) op(in1) + C; in0 [m,k] (d3: stored
                                   [k,m]), in1 [d1=k, n] (d4: stored [n,k]), in2 C [n] or [m,n] already scaled
                                   by beta, or -1 */,
    /* The rest of the reference runtime's dispatch table (exec.rs:347-533), f32, bit-exact with its kernels.
       Shapes are padded to rank 8 (MAX_RANK, crates/tpt-infer-core/src/shape.rs:4) with leading 1s. */
    TPT_OP_BINARY = 16,         /* out = in0 op in1, numpy broadcasting (kernels.rs:92-137); act = 0 add, 1 sub,
                                   2 mul, 3 div; d0..d7 out dims; d8 / d9: masks of the dims where in0 / in1 is 1 */
    TPT_OP_UNARY = 17,          /* act = 1 relu, 2 sigmoid, 3 gelu (Backend::relu/sigmoid/gelu); d0 = n */
    TPT_OP_POOL_NCHW = 18,      /* act = 0 max (kernels.rs:271-325), 1 average (count_include_pad 0, :335-390);
                                   d0..d11 = N,C,H,W,KH,KW,sh,sw,ph,pw,OH,OW */
    TPT_OP_BATCHNORM = 19,      /* in1 = [scale|bias|mean|var] (d1 values each), eps f0 (kernels.rs:425-476);
                                   d0 = numel, d2 = 1: channel mode with d3 = H*W, 0: element mode */
    TPT_OP_TRANSPOSE = 20,      /* d0..d7 input dims, d8..d15 perm (out axis i reads input axis perm[i]) */
    TPT_OP_CONCAT_COPY = 21,    /* one Concat input into out (concat_copy_one, kernels.rs:548-588): d0 outer,
                                   d1 source block, d2 output block, d3 offset (elements) */
    TPT_OP_CONV2D_F32 = 22,     /* Backend::conv2d NCHW f32, in1 OIHW weight; d0..d10 = N,C,H,W,OC,KH,KW,sh,sw,
                                   ph,pw */
    TPT_OP_BATCHED_MATMUL = 23  /* in0 [batch.., m, k] x in1 [batch.., k, n] -> [batch.., m, n] (shapes.rs:163-186);
                                   d0..d5 output batch dims, d6 / d7 masks of the batch dims where in0 / in1 is 1,
                                   d8 m, d9 k, d10 n */
};

typedef struct tpt_plan_op {
    int kind;
    int in0, in1, in2, out;     /* tensor ids, -1 = unused */
    const tpt_cuda_weights *w;  /* LINEAR_W8A8 */
    int act;                    /* tpt_act */
    float f0;                   /* static scale / eps / attention scale */
    size_t dims[16];
} tpt_plan_op;

int tpt_cuda_plan_create(tpt_cuda_ctx *ctx, tpt_cuda_plan **out);
int tpt_cuda_plan_destroy(tpt_cuda_plan *plan);
/* an activation tensor in the arena (dtype TPT_DT_F32 / TPT_DT_I8) */
int tpt_cuda_plan_add_tensor(tpt_cuda_plan *plan, int dtype, size_t numel, int *id);
/* an f32 constant, uploaded now (weights of f32 MatMuls, biases, LN params) */
int tpt_cuda_plan_add_const(tpt_cuda_plan *plan, const float *host, size_t numel, int *id);
int tpt_cuda_plan_add_op(tpt_cuda_plan *plan, const tpt_plan_op *op);
/* Before finalize: lay the arena out by liveness instead of one disjoint slot
 * per tensor (the reference's assign_offsets, exec.rs:276-294, gives every
 * node its own range). A tensor then occupies its bytes only from its first
 * writer to its last reader, so tensors with disjoint lifetimes share memory;
 * results are identical. Only the tensors listed here (kept to the end of a
 * run) can be fetched by tpt_cuda_plan_run (another id -> TPT_INVALID);
 * tpt_cuda_plan_tensor_ptr of any other tensor may alias a later tensor. */
int tpt_cuda_plan_reuse_arena(tpt_cuda_plan *plan, const int *keep_ids, size_t n_keep);
/* lays the arena out and allocates it (the only allocation of a run) */
int tpt_cuda_plan_finalize(tpt_cuda_plan *plan);
int tpt_cuda_plan_arena_bytes(tpt_cuda_plan *plan, size_t *bytes);
int tpt_cuda_plan_tensor_ptr(tpt_cuda_plan *plan, int id, void **dev);
int tpt_cuda_plan_set_calibration(tpt_cuda_plan *plan, int on);
int tpt_cuda_plan_freeze_scales(tpt_cuda_plan *plan);
/* The static scales of the quantization points, in op order (0 = none yet);
 * *count receives the number of points. Lets a calibration be exported. */
int tpt_cuda_plan_get_scales(tpt_cuda_plan *plan, float *scales, size_t n, size_t *count);
/* Imports a calibration: n must equal the number of points, every scale > 0;
 * the plan leaves calibration mode. (Batch-sharded ranks share one.) */
int tpt_cuda_plan_set_scales(tpt_cuda_plan *plan, const float *scales, size_t n);
/* With graphs on (default off), a run with frozen scales records the op
 * sequence once (after one direct run that sizes the workspaces) and replays
 * it from then on; calibration, new scales, a different output set or a moved
 * workspace make it record again. Plans with a communicator run directly. */
int tpt_cuda_plan_set_graph(tpt_cuda_plan *plan, int on);
/* ops only, inputs already resident (async) */
int tpt_cuda_plan_run_device(tpt_cuda_plan *plan);
/* H2D of the inputs, the ops, D2H of the outputs, then synchronise */
int tpt_cuda_plan_run(tpt_cuda_plan *plan, const int *in_ids, const float *const *inputs, size_t n_in,
                      const int *out_ids, float *const *outputs, size_t n_out);
/* n_steps runs of tpt_cuda_plan_run over consecutive batches (a serving loop):
 * step s reads inputs[s * n_in + i] and writes outputs[s * n_out + j]. The next
 * batch's inputs are copied to the device (on a copy stream, into a staging
 * buffer) while the current batch computes; with page-locked host buffers the
 * copy hides behind the forward pass. Results are those of n_steps separate
 * runs. Returns after the last outputs are in host memory. */
int tpt_cuda_plan_run_batches(tpt_cuda_plan *plan, const int *in_ids, const float *const *inputs, size_t n_in,
                              const int *out_ids, float *const *outputs, size_t n_out, size_t n_steps);

/* ------------------------------------------------------------------ */
/* Multi-GPU (one process per GPU on one node)                          */
/* ------------------------------------------------------------------ */

/* No counterpart in the reference (tpt-infer is single-process): the
 * exchange step of the column-sharded configuration. An NCCL communicator is
 * made from a unique id that rank 0 creates and the caller distributes to the
 * other ranks over any out-of-band channel. Collectives are enqueued on the
 * context's stream; every rank must issue the same ones in the same order.
 * NCCL is loaded at run time (libnccl.so.2): TPT_UNSUPPORTED when absent;
 * set-up that does not complete within 120 s returns TPT_NCCL_ERROR. Destroy a
 * communicator before its context. */
#define TPT_COMM_ID_BYTES 128
typedef struct tpt_cuda_comm tpt_cuda_comm;
int tpt_cuda_comm_unique_id(unsigned char *id, size_t id_bytes);
int tpt_cuda_comm_create(tpt_cuda_ctx *ctx, const unsigned char *id, size_t id_bytes, int world, int rank,
                         tpt_cuda_comm **out);
/* Deadline of communicator set-up and of each enqueue's completion report, in
 * seconds (0 = the default of 120 s); process-wide. */
int tpt_cuda_comm_set_timeout(double seconds);
int tpt_cuda_comm_destroy(tpt_cuda_comm *comm);
int tpt_cuda_comm_size(const tpt_cuda_comm *comm, int *world, int *rank);
/* out [world * bytes_per_rank] = the ranks' in [bytes_per_rank], rank order (device pointers, async) */
int tpt_cuda_all_gather_dev(tpt_cuda_comm *comm, const void *in, void *out, size_t bytes_per_rank);
/* The communicator of a plan's ALLGATHER ops and rank-global quantization points. */
int tpt_cuda_plan_set_comm(tpt_cuda_plan *plan, tpt_cuda_comm *comm);

/* ------------------------------------------------------------------ */
/* Allocation-free quantization                                         */
/* ------------------------------------------------------------------ */

/* Scratch of the allocation-free entry point below: TPT_NOALLOC_PARTIALS
 * 32-bit words (128 KiB) in the library's device image, which bounds its input
 * to TPT_NOALLOC_QUANT_MAX_ELEMS elements (2^28 floats, 1 GiB). */
#define TPT_NOALLOC_PARTIALS 32768u
#define TPT_NOALLOC_QUANT_MAX_ELEMS 268435456ull

/* No counterpart in the reference: an extra entry point for callers that
 * cannot allocate device memory -- code living inside another engine's memory
 * budget, real-time paths that cannot afford cudaMalloc's implicit device
 * synchronisation, and code that must not run out of memory halfway through.
 * It needs no context (creating one allocates) and calls no cudaMalloc,
 * cudaFree or other allocating routine.
 *
 * Same result as tpt_cuda_quantize_i8_symmetric_dev (quantize_i8_symmetric
 * semantics, bit-exact): x, q and scale are DEVICE pointers (x: n floats,
 * q: n int8, scale: one float written on the device), enqueued on `stream`
 * (a cudaStream_t passed as void*, NULL = legacy default stream) on the
 * current device; the call does not synchronise.
 *
 * Its reduction scratch is a fixed 128 KiB array that every GPU loading this
 * library holds until the process exits. n > TPT_NOALLOC_QUANT_MAX_ELEMS is
 * rejected with TPT_INVALID before any work is enqueued. The first call on a
 * device looks up the scratch's device address (cudaGetSymbolAddress, with
 * that device current) and caches it, so make that first call before any
 * stream capture. The cached address belongs to the device's primary context:
 * after cudaDeviceReset on that device the library's device image may be
 * loaded at another address, so do not use this entry point in a process that
 * resets a device it has already been called on. All calls on a device share
 * the scratch: calls whose kernels may overlap on the GPU (different streams
 * without ordering) race on it. Nothing in the scratch needs to start at
 * zero: a call only reads what it wrote itself earlier in stream order. */
int tpt_cuda_quantize_i8_symmetric_noalloc(const float *x, size_t n, int8_t *q, float *scale,
                                           void *stream);

#ifdef __cplusplus
}
#endif
#endif /* TPT_CUDA_H */
