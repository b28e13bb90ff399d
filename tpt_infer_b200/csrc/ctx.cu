// ctx.cu -- context lifecycle, error plumbing and the host-slice entry points
// that mirror tpt-infer's Backend trait (crates/tpt-infer-ops/src/backend.rs:98-147).
#include <stdio.h>
#include <string.h>

#include <new>

#include "common.cuh"

namespace tpt {

bool checked_mul(size_t a, size_t b, size_t *r) {
    if (a != 0 && b > SIZE_MAX / a) return false;
    *r = a * b;
    return true;
}

int set_size_mismatch(tpt_cuda_ctx *ctx, size_t expected, size_t actual) {
    ctx->last_expected = expected;
    ctx->last_actual = actual;
    return TPT_SIZE_MISMATCH;
}

int cuda_fail(tpt_cuda_ctx *ctx, cudaError_t e, const char *what) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s: %s", what, cudaGetErrorString(e));
    if (ctx) ctx->last_error = buf;
    return e == cudaErrorMemoryAllocation ? TPT_OUT_OF_MEMORY : TPT_CUDA_ERROR;
}

int after_launch(tpt_cuda_ctx *ctx, const char *what, int n) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(ctx, e, what);
    ctx->launches += (uint64_t)n;
    return TPT_OK;
}

// Workspaces cannot move while a graph is being recorded: the graph would
// keep the old address. The caller runs the call once before recording it.
static int refuse_in_capture(tpt_cuda_ctx *ctx, const char *what) {
    ctx->last_error = std::string(what) + " while a graph is being recorded (run the call once before recording)";
    return TPT_INVALID;
}

int ensure_scratch(tpt_cuda_ctx *ctx, size_t bytes) {
    if (bytes <= ctx->scratch_cap) return TPT_OK;
    if (ctx->capturing) return refuse_in_capture(ctx, "scratch grows");
    ctx->ws_gen++;
    size_t cap = ctx->scratch_cap ? ctx->scratch_cap : (size_t)1 << 20;
    while (cap < bytes) cap *= 2;
    if (ctx->scratch) {
        cudaError_t e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "scratch sync");
        cudaFree(ctx->scratch);
        ctx->scratch = nullptr;
        ctx->scratch_cap = 0;
    }
    cudaError_t e = cudaMalloc(&ctx->scratch, cap);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_fail(ctx, e, "scratch cudaMalloc");
    }
    ctx->scratch_cap = cap;
    return TPT_OK;
}

int ensure_ws(tpt_cuda_ctx *ctx, size_t bytes) {
    if (bytes <= ctx->ws_cap) return TPT_OK;
    if (ctx->capturing) return refuse_in_capture(ctx, "workspace grows");
    ctx->ws_gen++;
    size_t cap = ctx->ws_cap ? ctx->ws_cap : (size_t)1 << 20;
    while (cap < bytes) cap *= 2;
    if (ctx->ws) {
        cudaError_t e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "workspace sync");
        cudaFree(ctx->ws);
        ctx->ws = nullptr;
        ctx->ws_cap = 0;
    }
    cudaError_t e = cudaMalloc(&ctx->ws, cap);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_fail(ctx, e, "workspace cudaMalloc");
    }
    ctx->ws_cap = cap;
    return TPT_OK;
}

int ensure_sk(tpt_cuda_ctx *ctx, size_t slot_bytes) {
    const size_t bytes = TPT_SK_SLOTS_OFFSET + slot_bytes;
    if (bytes > ctx->sk_cap) {
        if (ctx->capturing) return refuse_in_capture(ctx, "stream-K workspace grows");
        ctx->ws_gen++;
        size_t cap = ctx->sk_cap ? ctx->sk_cap : (size_t)1 << 20;
        while (cap < bytes) cap *= 2;
        if (ctx->sk) {
            cudaError_t e = cudaStreamSynchronize(ctx->stream);
            if (e != cudaSuccess) return cuda_fail(ctx, e, "stream-K workspace sync");
            cudaFree(ctx->sk);
            ctx->sk = nullptr;
            ctx->sk_cap = 0;
        }
        cudaError_t e = cudaMalloc(&ctx->sk, cap);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return cuda_fail(ctx, e, "stream-K workspace cudaMalloc");
        }
        ctx->sk_cap = cap;
        ctx->sk_dirty = true;
    }
    if (ctx->sk_dirty) {
        if (ctx->capturing) return refuse_in_capture(ctx, "stream-K workspace clear");
        cudaError_t e = cudaMemsetAsync(ctx->sk, 0, ctx->sk_cap, ctx->stream);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "stream-K workspace clear");
        ctx->sk_dirty = false;
    }
    return TPT_OK;
}

int h2d(tpt_cuda_ctx *ctx, void *dst, const void *src, size_t bytes) {
    if (!bytes) return TPT_OK;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream);
    return e == cudaSuccess ? TPT_OK : cuda_fail(ctx, e, "H2D copy");
}

int d2h(tpt_cuda_ctx *ctx, void *dst, const void *src, size_t bytes) {
    if (!bytes) return TPT_OK;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream);
    return e == cudaSuccess ? TPT_OK : cuda_fail(ctx, e, "D2H copy");
}

int ensure_copy_streams(tpt_cuda_ctx *ctx) {
    if (ctx->copy_in) return TPT_OK;
    cudaError_t e = cudaStreamCreateWithFlags(&ctx->copy_in, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->copy_out, cudaStreamNonBlocking);
    for (int i = 0; e == cudaSuccess && i < (int)(sizeof(ctx->pipe_ev) / sizeof(ctx->pipe_ev[0])); i++)
        e = cudaEventCreateWithFlags(&ctx->pipe_ev[i], cudaEventDisableTiming);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "copy streams");
    return TPT_OK;
}

bool is_pinned_host(const void *p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeHost;
}

int sync_and_check(tpt_cuda_ctx *ctx) {
    if (ctx->capturing) return refuse_in_capture(ctx, "a synchronising call");
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "stream sync");
    unsigned flags[TPT_FLAG_WORDS];
    e = cudaMemcpy(flags, ctx->d_flags, sizeof flags, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "flag read");
    if (flags[TPT_FLAG_TIMEOUT] || flags[TPT_FLAG_CHECK]) {
        if (flags[TPT_FLAG_TIMEOUT]) ctx->sk_dirty = true;  // a stream-K launch may have stopped mid-tile
        cudaMemsetAsync(ctx->d_flags, 0, 2 * sizeof(unsigned), ctx->stream);  // the error words, not the wait limit
        cudaStreamSynchronize(ctx->stream);
        char buf[160];
        snprintf(buf, sizeof buf, "device flags: timeout=0x%x check=0x%x", flags[TPT_FLAG_TIMEOUT],
                 flags[TPT_FLAG_CHECK]);
        ctx->last_error = buf;
        return flags[TPT_FLAG_TIMEOUT] ? TPT_TIMEOUT : TPT_DEVICE_CHECK;
    }
    return TPT_OK;
}

}  // namespace tpt

using namespace tpt;

#define CHECK_CTX(c)                          \
    do {                                      \
        if (!(c)) return TPT_INVALID;         \
        cudaSetDevice((c)->device);           \
    } while (0)
#define TRY(x)                  \
    do {                        \
        int _st = (x);          \
        if (_st) return _st;    \
    } while (0)

extern "C" {

const char *tpt_cuda_backend_name(void) { return "cuda"; }

const char *tpt_cuda_status_str(int s) {
    switch (s) {
        case TPT_OK: return "ok";
        case TPT_SIZE_MISMATCH: return "size mismatch";
        case TPT_SHAPE_MISMATCH: return "shape mismatch";
        case TPT_UNSUPPORTED: return "operation not supported by this backend";
        case TPT_INVALID: return "invalid argument";
        case TPT_CUDA_ERROR: return "CUDA error";
        case TPT_OUT_OF_MEMORY: return "out of memory";
        case TPT_TIMEOUT: return "device wait timed out";
        case TPT_NCCL_ERROR: return "NCCL error";
        case TPT_DEVICE_CHECK: return "device-side check failed";
        default: return "unknown status";
    }
}

int tpt_cuda_ctx_create(int device, void *stream, tpt_cuda_ctx **out) {
    if (!out) return TPT_INVALID;
    *out = nullptr;
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
        cudaGetLastError();
        return TPT_UNSUPPORTED;
    }
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return TPT_UNSUPPORTED;
    // The kernels are built for sm_100a only.
    if (prop.major != 10) return TPT_UNSUPPORTED;
    tpt_cuda_ctx *ctx = new (std::nothrow) tpt_cuda_ctx();
    if (!ctx) return TPT_OUT_OF_MEMORY;
    ctx->device = device;
    ctx->sm_count = prop.multiProcessorCount;
    cudaSetDevice(device);
    cudaError_t e;
    if (stream) {
        ctx->stream = (cudaStream_t)stream;
    } else {
        e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) {
            delete ctx;
            return TPT_CUDA_ERROR;
        }
        ctx->own_stream = true;
    }
    e = cudaMalloc(&ctx->d_flags, (TPT_FLAG_WORDS + 64) * sizeof(unsigned));
    if (e != cudaSuccess) {
        if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
        delete ctx;
        return TPT_OUT_OF_MEMORY;
    }
    ctx->d_reduce = ctx->d_flags + TPT_FLAG_WORDS;
    cudaMemset(ctx->d_flags, 0, (TPT_FLAG_WORDS + 64) * sizeof(unsigned));
    cudaDeviceSynchronize();
    *out = ctx;
    return TPT_OK;
}

int tpt_cuda_ctx_destroy(tpt_cuda_ctx *ctx) {
    if (!ctx) return TPT_INVALID;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->ws) cudaFree(ctx->ws);
    if (ctx->sk) cudaFree(ctx->sk);
    if (ctx->d_flags) cudaFree(ctx->d_flags);
    if (ctx->copy_in) {
        cudaStreamSynchronize(ctx->copy_in);
        cudaStreamSynchronize(ctx->copy_out);
        for (cudaEvent_t ev : ctx->pipe_ev)
            if (ev) cudaEventDestroy(ev);
        cudaStreamDestroy(ctx->copy_in);
        cudaStreamDestroy(ctx->copy_out);
    }
    if (ctx->own_stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
    return TPT_OK;
}

int tpt_cuda_ctx_sync(tpt_cuda_ctx *ctx) {
    CHECK_CTX(ctx);
    return sync_and_check(ctx);
}

void *tpt_cuda_ctx_stream(tpt_cuda_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }
int tpt_cuda_ctx_device(tpt_cuda_ctx *ctx) { return ctx ? ctx->device : -1; }
const char *tpt_cuda_last_error(tpt_cuda_ctx *ctx) { return ctx ? ctx->last_error.c_str() : ""; }
void tpt_cuda_last_size_mismatch(tpt_cuda_ctx *ctx, size_t *expected, size_t *actual) {
    if (!ctx) return;
    if (expected) *expected = ctx->last_expected;
    if (actual) *actual = ctx->last_actual;
}
uint64_t tpt_cuda_ctx_launch_count(tpt_cuda_ctx *ctx) { return ctx ? ctx->launches : 0; }

// ---- CUDA graphs of device-pointer calls ----

struct tpt_cuda_graph {
    int device = 0;
    cudaGraphExec_t exec = nullptr;
    uint64_t kernels = 0;  // kernel launches recorded (added to the launch count per replay)
    uint64_t ws_gen = 0;   // workspace generation the recorded addresses belong to
};

int tpt_cuda_capture_begin(tpt_cuda_ctx *ctx) {
    CHECK_CTX(ctx);
    if (ctx->capturing) return TPT_INVALID;
    if (ctx->sk_dirty && ctx->sk) {  // clear a timed-out launch's leftovers outside the graph
        int st = ensure_sk(ctx, 0);
        if (st) return st;
    }
    cudaError_t e = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "begin capture");
    ctx->capturing = true;
    ctx->capture_launches0 = ctx->launches;
    return TPT_OK;
}

int tpt_cuda_capture_end(tpt_cuda_ctx *ctx, tpt_cuda_graph **out) {
    CHECK_CTX(ctx);
    if (!ctx->capturing || !out) return TPT_INVALID;
    *out = nullptr;
    ctx->capturing = false;
    const uint64_t kernels = ctx->launches - ctx->capture_launches0;
    ctx->launches = ctx->capture_launches0;  // recorded, not run
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(ctx->stream, &g);
    if (e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return cuda_fail(ctx, e, "end capture");
    }
    cudaGraphExec_t exec = nullptr;
    e = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "graph instantiate");
    tpt_cuda_graph *gr = new (std::nothrow) tpt_cuda_graph();
    if (!gr) {
        cudaGraphExecDestroy(exec);
        return TPT_OUT_OF_MEMORY;
    }
    gr->device = ctx->device;
    gr->exec = exec;
    gr->kernels = kernels;
    gr->ws_gen = ctx->ws_gen;
    *out = gr;
    return TPT_OK;
}

int tpt_cuda_graph_launch(tpt_cuda_ctx *ctx, tpt_cuda_graph *g) {
    CHECK_CTX(ctx);
    if (!g || ctx->capturing || g->device != ctx->device) return TPT_INVALID;
    if (g->ws_gen != ctx->ws_gen) {
        ctx->last_error = "a workspace moved since the graph was recorded (record it again)";
        return TPT_INVALID;
    }
    cudaError_t e = cudaGraphLaunch(g->exec, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "graph launch");
    ctx->launches += g->kernels;
    return TPT_OK;
}

uint64_t tpt_cuda_graph_kernels(const tpt_cuda_graph *g) { return g ? g->kernels : 0; }

int tpt_cuda_graph_destroy(tpt_cuda_graph *g) {
    if (!g) return TPT_INVALID;
    cudaSetDevice(g->device);
    cudaGraphExecDestroy(g->exec);
    delete g;
    return TPT_OK;
}

// ------------------------------------------------------------------ Backend::matmul
int tpt_cuda_matmul(tpt_cuda_ctx *ctx, const float *a, size_t a_len, size_t m, size_t k,
                    const float *b, size_t b_len, size_t kb, size_t n, float *out, size_t out_len) {
    CHECK_CTX(ctx);
    // validate_matmul (backend.rs:149-183), same checks in the same order
    size_t e;
    if (k != kb) return TPT_SHAPE_MISMATCH;
    if (!checked_mul(m, k, &e)) return TPT_INVALID;
    if (a_len != e) return set_size_mismatch(ctx, e, a_len);
    if (!checked_mul(k, n, &e)) return TPT_INVALID;
    if (b_len != e) return set_size_mismatch(ctx, e, b_len);
    if (!checked_mul(m, n, &e)) return TPT_INVALID;
    if (out_len != e) return set_size_mismatch(ctx, e, out_len);
    if (out_len == 0) return TPT_OK;
    Staging st(ctx);
    st.reserve(a_len * 4);
    st.reserve(b_len * 4);
    st.reserve(out_len * 4);
    TRY(st.commit());
    float *da = st.take<float>(a_len), *db = st.take<float>(b_len), *dc = st.take<float>(out_len);
    TRY(h2d(ctx, da, a, a_len * 4));
    TRY(h2d(ctx, db, b, b_len * 4));
    TRY(launch_matmul_f32(ctx, da, db, dc, m, k, n));
    TRY(d2h(ctx, out, dc, out_len * 4));
    return sync_and_check(ctx);
}

int tpt_cuda_matmul_dev(tpt_cuda_ctx *ctx, const float *a, size_t m, size_t k, const float *b,
                        size_t n, float *out) {
    CHECK_CTX(ctx);
    size_t e;
    if (!checked_mul(m, k, &e) || !checked_mul(k, n, &e) || !checked_mul(m, n, &e)) return TPT_INVALID;
    if (m * n == 0) return TPT_OK;
    return launch_matmul_f32(ctx, a, b, out, m, k, n);
}

// ------------------------------------------------------------------ ONNX Gemm
// Checks: a_len = m*k, b_len = k*n (size mismatches report expected/actual),
// c_len in {0, n, m*n} (else ShapeMismatch), out_len = m*n.
static int validate_gemm(tpt_cuda_ctx *ctx, size_t a_len, size_t m, size_t k, size_t b_len, size_t n, const float *c,
                         size_t c_len, size_t out_len, int *c_mode) {
    size_t e, mn;
    if (!checked_mul(m, k, &e)) return TPT_INVALID;
    if (a_len != e) return set_size_mismatch(ctx, e, a_len);
    if (!checked_mul(k, n, &e)) return TPT_INVALID;
    if (b_len != e) return set_size_mismatch(ctx, e, b_len);
    if (!checked_mul(m, n, &mn)) return TPT_INVALID;
    if (c_len != 0 && c_len != n && c_len != mn) return TPT_SHAPE_MISMATCH;
    if (c_len && !c) return TPT_INVALID;
    if (out_len != mn) return set_size_mismatch(ctx, mn, out_len);
    *c_mode = c_len == 0 ? 0 : (c_len == n ? 1 : 2);
    return TPT_OK;
}

int tpt_cuda_gemm(tpt_cuda_ctx *ctx, const float *a, size_t a_len, size_t m, size_t k, int trans_a, const float *b,
                  size_t b_len, size_t n, int trans_b, const float *c, size_t c_len, float alpha, float beta,
                  float *out, size_t out_len) {
    CHECK_CTX(ctx);
    int c_mode = 0;
    TRY(validate_gemm(ctx, a_len, m, k, b_len, n, c, c_len, out_len, &c_mode));
    if (out_len == 0) return TPT_OK;
    Staging st(ctx);
    st.reserve(a_len * 4);
    st.reserve(b_len * 4);
    st.reserve(c_len * 4);
    st.reserve(out_len * 4);
    TRY(st.commit());
    float *da = st.take<float>(a_len), *db = st.take<float>(b_len);
    float *dcm = c_len ? st.take<float>(c_len) : nullptr;
    float *dy = st.take<float>(out_len);
    TRY(h2d(ctx, da, a, a_len * 4));
    TRY(h2d(ctx, db, b, b_len * 4));
    if (c_len) TRY(h2d(ctx, dcm, c, c_len * 4));
    TRY(launch_gemm_onnx(ctx, da, db, dcm, c_mode, alpha, beta, dy, m, k, n, trans_a != 0, trans_b != 0));
    TRY(d2h(ctx, out, dy, out_len * 4));
    return sync_and_check(ctx);
}

int tpt_cuda_gemm_dev(tpt_cuda_ctx *ctx, const float *a, size_t m, size_t k, int trans_a, const float *b, size_t n,
                      int trans_b, const float *c, size_t c_len, float alpha, float beta, float *out) {
    CHECK_CTX(ctx);
    size_t e;
    int c_mode = 0;
    if (!checked_mul(m, k, &e) || !checked_mul(k, n, &e) || !checked_mul(m, n, &e)) return TPT_INVALID;
    TRY(validate_gemm(ctx, m * k, m, k, k * n, n, c, c_len, m * n, &c_mode));
    if (m * n == 0) return TPT_OK;
    return launch_gemm_onnx(ctx, a, b, c, c_mode, alpha, beta, out, m, k, n, trans_a != 0, trans_b != 0);
}

// ------------------------------------------------------------------ Backend::conv2d
static int validate_conv2d(tpt_cuda_ctx *ctx, size_t in_len, const size_t is[4], size_t w_len,
                           const size_t ws[4], size_t out_len, size_t sh, size_t sw, size_t ph,
                           size_t pw, size_t *oh, size_t *ow) {
    // validate_conv2d (backend.rs:219-284), same checks in the same order
    size_t e, ph2, pw2;
    if (ws[1] != is[1]) return TPT_SHAPE_MISMATCH;
    if (ws[2] == 0 || ws[3] == 0) return TPT_INVALID;
    if (sh == 0 || sw == 0) return TPT_INVALID;
    if (!checked_mul(ph, 2, &ph2) || is[2] > SIZE_MAX - ph2) return TPT_INVALID;
    if (!checked_mul(pw, 2, &pw2) || is[3] > SIZE_MAX - pw2) return TPT_INVALID;
    size_t hp = is[2] + ph2, wp = is[3] + pw2;
    if (hp < ws[2] || wp < ws[3]) return TPT_INVALID;
    *oh = (hp - ws[2]) / sh + 1;
    *ow = (wp - ws[3]) / sw + 1;
    if (!checked_mul(is[0], is[1], &e) || !checked_mul(e, is[2], &e) || !checked_mul(e, is[3], &e))
        return TPT_INVALID;
    if (in_len != e) return set_size_mismatch(ctx, e, in_len);
    if (!checked_mul(ws[0], ws[1], &e) || !checked_mul(e, ws[2], &e) || !checked_mul(e, ws[3], &e))
        return TPT_INVALID;
    if (w_len != e) return set_size_mismatch(ctx, e, w_len);
    if (!checked_mul(is[0], ws[0], &e) || !checked_mul(e, *oh, &e) || !checked_mul(e, *ow, &e))
        return TPT_INVALID;
    if (out_len != e) return set_size_mismatch(ctx, e, out_len);
    return TPT_OK;
}

int tpt_cuda_conv2d(tpt_cuda_ctx *ctx, const float *input, size_t in_len, const size_t in_shape[4],
                    const float *weight, size_t w_len, const size_t w_shape[4], float *out,
                    size_t out_len, size_t stride_h, size_t stride_w, size_t pad_h, size_t pad_w) {
    CHECK_CTX(ctx);
    if (!in_shape || !w_shape) return TPT_INVALID;
    size_t oh, ow;
    TRY(validate_conv2d(ctx, in_len, in_shape, w_len, w_shape, out_len, stride_h, stride_w, pad_h,
                        pad_w, &oh, &ow));
    if (out_len == 0) return TPT_OK;
    Staging st(ctx);
    st.reserve(in_len * 4);
    st.reserve(w_len * 4);
    st.reserve(out_len * 4);
    TRY(st.commit());
    float *di = st.take<float>(in_len), *dw = st.take<float>(w_len), *dc = st.take<float>(out_len);
    TRY(h2d(ctx, di, input, in_len * 4));
    TRY(h2d(ctx, dw, weight, w_len * 4));
    TRY(launch_conv2d_f32(ctx, di, dw, dc, in_shape, w_shape, oh, ow, stride_h, stride_w, pad_h, pad_w));
    TRY(d2h(ctx, out, dc, out_len * 4));
    return sync_and_check(ctx);
}

int tpt_cuda_conv2d_dev(tpt_cuda_ctx *ctx, const float *input, const size_t in_shape[4],
                        const float *weight, const size_t w_shape[4], float *out, size_t stride_h,
                        size_t stride_w, size_t pad_h, size_t pad_w) {
    CHECK_CTX(ctx);
    if (!in_shape || !w_shape) return TPT_INVALID;
    if (in_shape[1] != w_shape[1]) return TPT_SHAPE_MISMATCH;
    if (w_shape[2] == 0 || w_shape[3] == 0 || stride_h == 0 || stride_w == 0) return TPT_INVALID;
    if (in_shape[2] + 2 * pad_h < w_shape[2] || in_shape[3] + 2 * pad_w < w_shape[3]) return TPT_INVALID;
    size_t oh = (in_shape[2] + 2 * pad_h - w_shape[2]) / stride_h + 1;
    size_t ow = (in_shape[3] + 2 * pad_w - w_shape[3]) / stride_w + 1;
    if (in_shape[0] * w_shape[0] * oh * ow == 0) return TPT_OK;
    return launch_conv2d_f32(ctx, input, weight, out, in_shape, w_shape, oh, ow, stride_h, stride_w,
                             pad_h, pad_w);
}

// ------------------------------------------------------------------ element ops
static int unary_host(tpt_cuda_ctx *ctx, int op, const float *a, size_t a_len, float *out,
                      size_t out_len) {
    CHECK_CTX(ctx);
    // validate_unary (backend.rs:201-209)
    if (out_len != a_len) return set_size_mismatch(ctx, a_len, out_len);
    if (a_len == 0) return TPT_OK;
    Staging st(ctx);
    st.reserve(a_len * 4);
    st.reserve(a_len * 4);
    TRY(st.commit());
    float *da = st.take<float>(a_len), *dc = st.take<float>(a_len);
    TRY(h2d(ctx, da, a, a_len * 4));
    TRY(launch_unary(ctx, op, da, dc, a_len));
    TRY(d2h(ctx, out, dc, a_len * 4));
    return sync_and_check(ctx);
}

int tpt_cuda_relu(tpt_cuda_ctx *ctx, const float *a, size_t a_len, float *out, size_t out_len) {
    return unary_host(ctx, 1, a, a_len, out, out_len);
}
int tpt_cuda_sigmoid(tpt_cuda_ctx *ctx, const float *a, size_t a_len, float *out, size_t out_len) {
    return unary_host(ctx, 2, a, a_len, out, out_len);
}
int tpt_cuda_gelu(tpt_cuda_ctx *ctx, const float *a, size_t a_len, float *out, size_t out_len) {
    return unary_host(ctx, 3, a, a_len, out, out_len);
}

int tpt_cuda_elementwise_add(tpt_cuda_ctx *ctx, const float *a, size_t a_len, const float *b,
                             size_t b_len, float *out, size_t out_len) {
    CHECK_CTX(ctx);
    // validate_binary (backend.rs:185-199)
    if (a_len != b_len) return set_size_mismatch(ctx, a_len, b_len);
    if (out_len != a_len) return set_size_mismatch(ctx, a_len, out_len);
    if (a_len == 0) return TPT_OK;
    Staging st(ctx);
    st.reserve(a_len * 4);
    st.reserve(a_len * 4);
    st.reserve(a_len * 4);
    TRY(st.commit());
    float *da = st.take<float>(a_len), *db = st.take<float>(a_len), *dc = st.take<float>(a_len);
    TRY(h2d(ctx, da, a, a_len * 4));
    TRY(h2d(ctx, db, b, a_len * 4));
    TRY(launch_add(ctx, da, db, dc, a_len));
    TRY(d2h(ctx, out, dc, a_len * 4));
    return sync_and_check(ctx);
}

int tpt_cuda_softmax(tpt_cuda_ctx *ctx, const float *a, size_t a_len, float *out, size_t out_len,
                     size_t row_len) {
    CHECK_CTX(ctx);
    // validate_softmax (backend.rs:211-217)
    if (out_len != a_len) return set_size_mismatch(ctx, a_len, out_len);
    if (row_len == 0 || a_len % row_len != 0) return TPT_INVALID;
    if (a_len == 0) return TPT_OK;
    Staging st(ctx);
    st.reserve(a_len * 4);
    st.reserve(a_len * 4);
    TRY(st.commit());
    float *da = st.take<float>(a_len), *dc = st.take<float>(a_len);
    TRY(h2d(ctx, da, a, a_len * 4));
    TRY(launch_softmax(ctx, da, dc, a_len / row_len, row_len));
    TRY(d2h(ctx, out, dc, a_len * 4));
    return sync_and_check(ctx);
}

int tpt_cuda_elementwise_add_dev(tpt_cuda_ctx *ctx, const float *a, const float *b, float *out, size_t n) {
    CHECK_CTX(ctx);
    return n ? launch_add(ctx, a, b, out, n) : TPT_OK;
}
int tpt_cuda_relu_dev(tpt_cuda_ctx *ctx, const float *a, float *out, size_t n) {
    CHECK_CTX(ctx);
    return n ? launch_unary(ctx, 1, a, out, n) : TPT_OK;
}
int tpt_cuda_sigmoid_dev(tpt_cuda_ctx *ctx, const float *a, float *out, size_t n) {
    CHECK_CTX(ctx);
    return n ? launch_unary(ctx, 2, a, out, n) : TPT_OK;
}
int tpt_cuda_gelu_dev(tpt_cuda_ctx *ctx, const float *a, float *out, size_t n) {
    CHECK_CTX(ctx);
    return n ? launch_unary(ctx, 3, a, out, n) : TPT_OK;
}
int tpt_cuda_softmax_dev(tpt_cuda_ctx *ctx, const float *a, float *out, size_t n, size_t row_len) {
    CHECK_CTX(ctx);
    if (row_len == 0 || n % row_len != 0) return TPT_INVALID;
    return n ? launch_softmax(ctx, a, out, n / row_len, row_len) : TPT_OK;
}

}  // extern "C"

extern "C" int tpt_cuda_ctx_set_wait_limit(tpt_cuda_ctx *ctx, uint32_t cycles) {
    if (!ctx) return TPT_INVALID;
    if (ctx->capturing) return refuse_in_capture(ctx, "setting the wait limit");
    cudaSetDevice(ctx->device);
    cudaError_t e = cudaMemcpyAsync(ctx->d_flags + TPT_FLAG_WAIT_LIMIT, &cycles, sizeof cycles, cudaMemcpyHostToDevice,
                                    ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    return e == cudaSuccess ? TPT_OK : cuda_fail(ctx, e, "wait limit");
}
