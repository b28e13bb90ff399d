// plan.cu -- device-resident execution plans: the device counterpart of
// tpt-infer's execute_graph (crates/tpt-infer-runtime/src/exec.rs:570-635).
//
// The reference lays every non-input node's activation out at a disjoint
// offset of one arena slice in topological order (assign_offsets,
// exec.rs:276-294; one alloc_slice, exec.rs:595), runs the nodes in that order
// and copies the marked outputs out at the end. A plan does the same on the
// device: tensors get disjoint 256-byte-aligned offsets in ONE device
// allocation made at finalize, constants (f32 weights, biases, LayerNorm
// parameters) are uploaded once, ops run in order on the context's stream, and
// host<->device copies happen only at graph inputs and outputs.
//
// INT8 activation quantization points carry a per-tensor scale. A plan in
// calibration mode measures max|x| at every quantization point on each run
// (the quantize_i8_symmetric rule, quant.rs:25-31, applied to the running
// max); tpt_cuda_plan_freeze_scales turns the maxima into static scales.
#include <string.h>

#include <algorithm>
#include <new>
#include <vector>

#include "common.cuh"

namespace tpt {
int launch_layernorm(tpt_cuda_ctx *ctx, const float *x, const float *g, const float *b, float *y, size_t rows,
                     size_t cols, float eps, int8_t *q = nullptr, float qs = 0.0f, const float *res = nullptr);
int launch_attention(tpt_cuda_ctx *ctx, const float *qkv, float *out, int B, int S, int H, int D, float scale,
                     int8_t *q = nullptr, float qs = 0.0f);
int launch_bias_act(tpt_cuda_ctx *ctx, const float *x, const float *bias, float *y, size_t rows, size_t cols, int act);
int launch_add_act(tpt_cuda_ctx *ctx, const float *a, const float *b, float *y, size_t n, int act,
                   int8_t *q = nullptr, float qs = 0.0f);
int launch_nchw_to_nhwc_q8(tpt_cuda_ctx *ctx, const float *x, int8_t *q, int N, int C, int HW, int W, int Cp, int s2d,
                           float scale);
int launch_im2col(tpt_cuda_ctx *ctx, const int8_t *x, int8_t *col, int N, int H, int W, int C, int KH, int KW, int sh,
                  int sw, int ph, int pw, int OH, int OW, int Kp);
int launch_maxpool_nhwc(tpt_cuda_ctx *ctx, const float *x, float *y, int N, int H, int W, int C, int KH, int KW, int sh,
                        int sw, int ph, int pw, int OH, int OW, int8_t *q = nullptr,
                        float qs = 0.0f);
int launch_gap_nhwc(tpt_cuda_ctx *ctx, const float *x, float *y, int N, int HW, int C);
int launch_absmax_acc(tpt_cuda_ctx *ctx, const float *x, size_t n, unsigned *cell);
int launch_panels_to_rows(tpt_cuda_ctx *ctx, const int8_t *in, int8_t *out, int P, size_t T, int C);
int comm_all_gather(tpt_cuda_comm *c, const void *in, void *out, size_t bytes_per_rank);
int launch_conv_w8a8(tpt_cuda_ctx *ctx, const int8_t *x, int N, int H, int W, int C, int KH, int KW, int sh, int sw,
                     int ph, int pw, int OH, int OW, const tpt_cuda_weights *w, float a_scale, const float *bias,
                     int act, float *y, bool *handled, Requant rq, Residual res = Residual());
int launch_stem_pool(tpt_cuda_ctx *ctx, const int8_t *x, int N, int H, int W, int C, int KH, int KW, int sh, int sw,
                     int ph, int pw, int OH, int OW, const tpt_cuda_weights *w, float a_scale, const float *bias,
                     int act, int PH, int PW, float *P, int8_t *Q, float q_scale, bool *handled);
int comm_max_u32(tpt_cuda_comm *c, unsigned *words, size_t n);
int ensure_copy_streams(tpt_cuda_ctx *ctx);
int launch_binary(tpt_cuda_ctx *ctx, const float *a, const float *b, float *out, const size_t od[8], unsigned amask,
                  unsigned bmask, int op, size_t n);
int launch_pool_nchw(tpt_cuda_ctx *ctx, const float *x, float *y, int avg, size_t NC, int H, int W, int KH, int KW,
                     int sh, int sw, int ph, int pw, int OH, int OW);
int launch_batchnorm(tpt_cuda_ctx *ctx, const float *x, const float *prm, float *y, size_t n, size_t plen, size_t hw,
                     int channel_mode, float eps);
int launch_transpose(tpt_cuda_ctx *ctx, const float *x, float *y, const size_t xd[8], const size_t perm[8], size_t n);
int launch_concat_copy(tpt_cuda_ctx *ctx, const float *src, float *dst, size_t outer, size_t src_block,
                       size_t out_block, size_t offset);
int launch_bmm(tpt_cuda_ctx *ctx, const float *a, const float *b, float *c, const size_t bd[6], unsigned amask,
               unsigned bmask, size_t m, size_t k, size_t n);
}  // namespace tpt

using namespace tpt;

struct PlanTensor {
    int dtype = TPT_DT_F32;
    size_t numel = 0;
    size_t offset = 0;      // arena offset (activations)
    void *ptr = nullptr;    // device pointer (set at finalize / for constants)
    bool is_const = false;
    float scale = 0.0f;     // INT8 tensors: the per-tensor scale in effect
    int readers = 0;        // ops reading this tensor (set at finalize)
};

struct PlanOp {
    tpt_plan_op op;
    int cell = -1;          // calibration cell index (quantization points)
    float frozen = 0.0f;    // static scale once frozen (or given)
};

struct tpt_cuda_plan {
    tpt_cuda_ctx *ctx = nullptr;
    tpt_cuda_comm *comm = nullptr;  // multi-GPU plans: ALLGATHER and rank-global scales
    int device = 0;  // destroying needs only the device: the context may be gone
    std::vector<PlanTensor> tensors;
    std::vector<PlanOp> ops;
    char *arena = nullptr;
    size_t arena_bytes = 0;
    unsigned *cells = nullptr;  // device: one max-abs word per quantization point
    std::vector<float> cal_max; // host: running max per quantization point
    int n_cells = 0;
    bool finalized = false;
    bool calibrating = false;
    // liveness-based arena (tpt_cuda_plan_reuse_arena): only `keep` tensors and
    // graph inputs (before their last reader) may be fetched
    bool reuse = false;
    std::vector<char> keep;
    // tpt_cuda_plan_run_batches: two device staging buffers for the inputs and the
    // events that order them between the copy stream and the compute stream
    char *stage = nullptr;
    size_t stage_bytes = 0;
    cudaEvent_t ev_in[2] = {nullptr, nullptr}, ev_free[2] = {nullptr, nullptr};
    // recorded replay of run_ops (tpt_cuda_plan_set_graph) and the output set it was recorded for
    bool use_graph = false;
    tpt_cuda_graph *graph = nullptr;
    std::vector<int> graph_out;
};

namespace {

size_t dt_size(int dt) { return dt == TPT_DT_I8 ? 1 : 4; }

void drop_graph(tpt_cuda_plan *p) {
    if (p->graph) tpt_cuda_graph_destroy(p->graph);
    p->graph = nullptr;
    p->graph_out.clear();
}

bool valid_id(tpt_cuda_plan *p, int id) { return id >= 0 && (size_t)id < p->tensors.size(); }

float *F(tpt_cuda_plan *p, int id) { return id < 0 ? nullptr : static_cast<float *>(p->tensors[id].ptr); }
int8_t *Q(tpt_cuda_plan *p, int id) { return id < 0 ? nullptr : static_cast<int8_t *>(p->tensors[id].ptr); }

// Scale for a quantization point: frozen/static, or (calibrating) measured now.
// A rank-global point (a column-sharded tensor that is all-gathered next)
// takes the max over the plan's communicator, so every rank quantizes its
// shard with the scale of the whole tensor.
int point_scale(tpt_cuda_plan *p, PlanOp &po, const float *x, size_t n, float *scale, bool global = false) {
    if (!p->calibrating) {
        if (!(po.frozen > 0.0f)) return TPT_INVALID;  // not calibrated and no static scale given
        *scale = po.frozen;
        return TPT_OK;
    }
    tpt_cuda_ctx *ctx = p->ctx;
    unsigned *cell = p->cells + po.cell;
    cudaError_t e = cudaMemsetAsync(cell, 0, 4, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "calibration cell clear");
    int st = launch_absmax_acc(ctx, x, n, cell);
    if (st) return st;
    if (global) {
        if (!p->comm) return TPT_INVALID;
        st = comm_max_u32(p->comm, cell, 1);
        if (st) return st;
    }
    unsigned bits = 0;
    st = d2h(ctx, &bits, cell, 4);
    if (st) return st;
    st = sync_and_check(ctx);
    if (st) return st;
    float m;
    memcpy(&m, &bits, 4);
    if (m > p->cal_max[po.cell]) p->cal_max[po.cell] = m;
    // quantize_i8_symmetric's rule (quant.rs:27-31) on this run's max
    *scale = m == 0.0f ? 1.0f : m / 127.0f;
    return TPT_OK;
}

int run_op(tpt_cuda_plan *p, PlanOp &po) {
    tpt_cuda_ctx *ctx = p->ctx;
    const tpt_plan_op &o = po.op;
    const size_t *d = o.dims;
    int st = TPT_OK;
    switch (o.kind) {
        case TPT_OP_QUANTIZE: {  // f32 [n] -> i8 [n], per-tensor scale (d1 != 0: rank-global)
            float s;
            st = point_scale(p, po, F(p, o.in0), d[0], &s, d[1] != 0);
            if (st) return st;
            p->tensors[o.out].scale = s;
            return launch_quant_i8_static(ctx, F(p, o.in0), d[0], s, Q(p, o.out));
        }
        case TPT_OP_NCHW_TO_NHWC_Q8: {  // f32 NCHW [N,C,HW] -> i8 NHWC with d3 (>= C, or 0 = C) channels;
                                        // d4 = W, d5 = 2: space-to-depth 2x2
            float s;
            st = point_scale(p, po, F(p, o.in0), d[0] * d[1] * d[2], &s);
            if (st) return st;
            p->tensors[o.out].scale = s;
            const int cp = d[3] > d[1] ? (int)d[3] : (int)d[1];
            return launch_nchw_to_nhwc_q8(ctx, F(p, o.in0), Q(p, o.out), (int)d[0], (int)d[1], (int)d[2], (int)d[4], cp,
                                          (int)d[5], s);
        }
        case TPT_OP_LINEAR_W8A8: {  // i8 [rows, K] x W^T -> f32 [rows, N] (+bias, act)
            const float sa = p->tensors[o.in0].scale;
            return launch_w8a8(ctx, Q(p, o.in0), d[0], o.w->k, o.w, sa, F(p, o.in1), o.act, F(p, o.out), nullptr);
        }
        case TPT_OP_MATMUL_F32: {  // [m,k] x [k,n] (+bias, act)
            return launch_matmul_f32_epi(ctx, F(p, o.in0), F(p, o.in1), o.in2 < 0 ? nullptr : F(p, o.in2), o.act,
                                         F(p, o.out), d[0], d[1], d[2]);
        }
        case TPT_OP_BIAS_ACT:
            return launch_bias_act(ctx, F(p, o.in0), F(p, o.in1), F(p, o.out), d[0], d[1], o.act);
        case TPT_OP_ADD_ACT:
            return launch_add_act(ctx, F(p, o.in0), F(p, o.in1), F(p, o.out), d[0], o.act);
        case TPT_OP_SOFTMAX:
            return launch_softmax(ctx, F(p, o.in0), F(p, o.out), d[0], d[1]);
        case TPT_OP_ALLGATHER: {  // in0 [d0 elements] on every rank -> out [world * d0], rank order
            if (!p->comm) return TPT_INVALID;
            p->tensors[o.out].scale = p->tensors[o.in0].scale;
            return comm_all_gather(p->comm, p->tensors[o.in0].ptr, p->tensors[o.out].ptr,
                                   d[0] * dt_size(p->tensors[o.in0].dtype));
        }
        case TPT_OP_GEMM_F32: {  // ONNX Gemm, beta folded into the constant C
            const int c_mode = o.in2 < 0 ? 0 : (p->tensors[o.in2].numel == d[2] ? 1 : 2);
            return launch_gemm_onnx(ctx, F(p, o.in0), F(p, o.in1), F(p, o.in2), c_mode, o.f0, 1.0f, F(p, o.out), d[0],
                                    d[1], d[2], d[3] != 0, d[4] != 0);
        }
        case TPT_OP_PANELS_TO_ROWS:  // i8 [d0 = P][d1 = T][d2 = C] -> i8 [T][P * C]
            p->tensors[o.out].scale = p->tensors[o.in0].scale;
            return launch_panels_to_rows(ctx, Q(p, o.in0), Q(p, o.out), (int)d[0], d[1], (int)d[2]);
        case TPT_OP_LAYERNORM:
            return launch_layernorm(ctx, F(p, o.in0), F(p, o.in1), F(p, o.in2), F(p, o.out), d[0], d[1], o.f0);
        case TPT_OP_ATTENTION:
            return launch_attention(ctx, F(p, o.in0), F(p, o.out), (int)d[0], (int)d[1], (int)d[2], (int)d[3], o.f0);
        case TPT_OP_IM2COL:  // dims: N,H,W,C,KH,KW,sh,sw,ph,pw,OH,OW,Kp
            p->tensors[o.out].scale = p->tensors[o.in0].scale;
            return launch_im2col(ctx, Q(p, o.in0), Q(p, o.out), (int)d[0], (int)d[1], (int)d[2], (int)d[3], (int)d[4],
                                 (int)d[5], (int)d[6], (int)d[7], (int)d[8], (int)d[9], (int)d[10], (int)d[11],
                                 (int)d[12]);
        case TPT_OP_MAXPOOL_NHWC:
            return launch_maxpool_nhwc(ctx, F(p, o.in0), F(p, o.out), (int)d[0], (int)d[1], (int)d[2], (int)d[3],
                                       (int)d[4], (int)d[5], (int)d[6], (int)d[7], (int)d[8], (int)d[9], (int)d[10],
                                       (int)d[11]);
        case TPT_OP_GAP_NHWC:
            return launch_gap_nhwc(ctx, F(p, o.in0), F(p, o.out), (int)d[0], (int)d[1], (int)d[2]);
        case TPT_OP_BINARY: {
            size_t n = 1;
            for (int i = 0; i < 8; i++) n *= d[i];
            return launch_binary(ctx, F(p, o.in0), F(p, o.in1), F(p, o.out), d, (unsigned)d[8], (unsigned)d[9], o.act,
                                 n);
        }
        case TPT_OP_UNARY:
            return launch_unary(ctx, o.act, F(p, o.in0), F(p, o.out), d[0]);
        case TPT_OP_POOL_NCHW:
            return launch_pool_nchw(ctx, F(p, o.in0), F(p, o.out), o.act, d[0] * d[1], (int)d[2], (int)d[3],
                                    (int)d[4], (int)d[5], (int)d[6], (int)d[7], (int)d[8], (int)d[9], (int)d[10],
                                    (int)d[11]);
        case TPT_OP_BATCHNORM:
            return launch_batchnorm(ctx, F(p, o.in0), F(p, o.in1), F(p, o.out), d[0], d[1], d[3], (int)d[2], o.f0);
        case TPT_OP_TRANSPOSE:
            return launch_transpose(ctx, F(p, o.in0), F(p, o.out), d, d + 8, p->tensors[o.in0].numel);
        case TPT_OP_CONCAT_COPY:
            return launch_concat_copy(ctx, F(p, o.in0), F(p, o.out), d[0], d[1], d[2], d[3]);
        case TPT_OP_CONV2D_F32: {
            const size_t is[4] = {d[0], d[1], d[2], d[3]}, ws[4] = {d[4], d[1], d[5], d[6]};
            const size_t oh = (d[2] + 2 * d[9] - d[5]) / d[7] + 1, ow = (d[3] + 2 * d[10] - d[6]) / d[8] + 1;
            return launch_conv2d_f32(ctx, F(p, o.in0), F(p, o.in1), F(p, o.out), is, ws, oh, ow, d[7], d[8], d[9],
                                     d[10]);
        }
        case TPT_OP_BATCHED_MATMUL:
            return launch_bmm(ctx, F(p, o.in0), F(p, o.in1), F(p, o.out), d, (unsigned)d[6], (unsigned)d[7], d[8],
                              d[9], d[10]);
        default:
            return TPT_UNSUPPORTED;
    }
}

}  // namespace

namespace {
// Sizes of the graph-level ops checked against their tensors at add time, so a
// launch can never index outside a tensor. Invalid geometry (a zero stride, a
// non-permutation, a shape that does not broadcast) is TPT_INVALID.
size_t numel_of(tpt_cuda_plan *p, int id) { return p->tensors[id].numel; }
bool prod_ok(const size_t *d, int n, size_t *out) {
    size_t r = 1;
    for (int i = 0; i < n; i++)
        if (!checked_mul(r, d[i], &r)) return false;
    *out = r;
    return true;
}
int validate_graph_op(tpt_cuda_plan *p, const tpt_plan_op &o) {
    const size_t *d = o.dims;
    const bool f32 = p->tensors[o.in0].dtype == TPT_DT_F32 && p->tensors[o.out].dtype == TPT_DT_F32 &&
                     (o.in1 < 0 || p->tensors[o.in1].dtype == TPT_DT_F32);
    if (!f32) return TPT_INVALID;
    switch (o.kind) {
        case TPT_OP_BINARY: {
            if (o.in1 < 0 || o.act < 0 || o.act > 3 || d[8] > 255 || d[9] > 255) return TPT_INVALID;
            size_t n, na = 1, nb = 1;
            if (!prod_ok(d, 8, &n) || n != numel_of(p, o.out)) return TPT_INVALID;
            for (int i = 0; i < 8; i++) {
                if (!(d[8] >> i & 1)) na *= d[i];
                if (!(d[9] >> i & 1)) nb *= d[i];
            }
            return na == numel_of(p, o.in0) && nb == numel_of(p, o.in1) ? TPT_OK : TPT_INVALID;
        }
        case TPT_OP_UNARY:
            return o.act >= 1 && o.act <= 3 && d[0] <= numel_of(p, o.in0) && d[0] <= numel_of(p, o.out) ? TPT_OK
                                                                                                      : TPT_INVALID;
        case TPT_OP_POOL_NCHW: {
            size_t a, b;
            const size_t in_d[4] = {d[0], d[1], d[2], d[3]}, out_d[4] = {d[0], d[1], d[10], d[11]};
            if (o.act < 0 || o.act > 1 || d[4] == 0 || d[5] == 0 || d[6] == 0 || d[7] == 0) return TPT_INVALID;
            for (int i = 2; i < 12; i++)
                if (d[i] > INT32_MAX) return TPT_INVALID;
            if (!prod_ok(in_d, 4, &a) || !prod_ok(out_d, 4, &b)) return TPT_INVALID;
            return a == numel_of(p, o.in0) && b == numel_of(p, o.out) ? TPT_OK : TPT_INVALID;
        }
        case TPT_OP_BATCHNORM: {
            size_t four;
            if (o.in1 < 0 || d[1] == 0 || !checked_mul(d[1], 4, &four) || four != numel_of(p, o.in1)) return TPT_INVALID;
            if (d[0] != numel_of(p, o.in0) || d[0] != numel_of(p, o.out)) return TPT_INVALID;
            if (d[2]) return d[3] && d[0] % (d[1] * d[3]) == 0 ? TPT_OK : TPT_INVALID;
            return d[1] == d[0] ? TPT_OK : TPT_INVALID;
        }
        case TPT_OP_TRANSPOSE: {
            size_t n;
            unsigned seen = 0;
            for (int i = 0; i < 8; i++) {
                if (d[8 + i] > 7 || (seen >> d[8 + i] & 1)) return TPT_INVALID;
                seen |= 1u << d[8 + i];
            }
            if (!prod_ok(d, 8, &n)) return TPT_INVALID;
            return n == numel_of(p, o.in0) && n == numel_of(p, o.out) ? TPT_OK : TPT_INVALID;
        }
        case TPT_OP_CONCAT_COPY: {
            size_t n, last;
            if (d[0] == 0 || d[1] == 0) return TPT_INVALID;
            if (!checked_mul(d[0], d[1], &n) || n > numel_of(p, o.in0)) return TPT_INVALID;
            if (!checked_mul(d[0] - 1, d[2], &last) || d[3] + d[1] > d[2]) return TPT_INVALID;
            return last + d[2] <= numel_of(p, o.out) ? TPT_OK : TPT_INVALID;
        }
        case TPT_OP_CONV2D_F32: {
            size_t a, w, y;
            if (o.in1 < 0 || d[7] == 0 || d[8] == 0) return TPT_INVALID;
            if (d[2] + 2 * d[9] < d[5] || d[3] + 2 * d[10] < d[6]) return TPT_INVALID;
            const size_t oh = (d[2] + 2 * d[9] - d[5]) / d[7] + 1, ow = (d[3] + 2 * d[10] - d[6]) / d[8] + 1;
            const size_t xd[4] = {d[0], d[1], d[2], d[3]}, wd[4] = {d[4], d[1], d[5], d[6]}, yd[4] = {d[0], d[4], oh, ow};
            if (!prod_ok(xd, 4, &a) || !prod_ok(wd, 4, &w) || !prod_ok(yd, 4, &y)) return TPT_INVALID;
            return a == numel_of(p, o.in0) && w == numel_of(p, o.in1) && y == numel_of(p, o.out) ? TPT_OK
                                                                                                 : TPT_INVALID;
        }
        case TPT_OP_BATCHED_MATMUL: {
            if (o.in1 < 0 || d[6] > 63 || d[7] > 63) return TPT_INVALID;
            size_t bo, ba = 1, bb = 1, mk, kn, mn, t;
            if (!prod_ok(d, 6, &bo)) return TPT_INVALID;
            for (int i = 0; i < 6; i++) {
                if (!(d[6] >> i & 1)) ba *= d[i];
                if (!(d[7] >> i & 1)) bb *= d[i];
            }
            if (!checked_mul(d[8], d[9], &mk) || !checked_mul(d[9], d[10], &kn) || !checked_mul(d[8], d[10], &mn))
                return TPT_INVALID;
            if (!checked_mul(ba, mk, &t) || t != numel_of(p, o.in0)) return TPT_INVALID;
            if (!checked_mul(bb, kn, &t) || t != numel_of(p, o.in1)) return TPT_INVALID;
            return checked_mul(bo, mn, &t) && t == numel_of(p, o.out) ? TPT_OK : TPT_INVALID;
        }
    }
    return TPT_OK;
}
}  // namespace

#define CHECK_PLAN(pl)                                  \
    do {                                                \
        if (!(pl) || !(pl)->ctx) return TPT_INVALID;    \
        cudaSetDevice((pl)->ctx->device);               \
    } while (0)

extern "C" {

int tpt_cuda_plan_create(tpt_cuda_ctx *ctx, tpt_cuda_plan **out) {
    if (!ctx || !out) return TPT_INVALID;
    tpt_cuda_plan *p = new (std::nothrow) tpt_cuda_plan();
    if (!p) return TPT_OUT_OF_MEMORY;
    p->ctx = ctx;
    p->device = ctx->device;
    *out = p;
    return TPT_OK;
}

// cudaFree waits for work using the memory, so the context is not touched and
// a plan may outlive it.
int tpt_cuda_plan_destroy(tpt_cuda_plan *p) {
    if (!p) return TPT_INVALID;
    cudaSetDevice(p->device);
    drop_graph(p);
    if (p->stage) cudaFree(p->stage);
    for (int i = 0; i < 2; i++) {
        if (p->ev_in[i]) cudaEventDestroy(p->ev_in[i]);
        if (p->ev_free[i]) cudaEventDestroy(p->ev_free[i]);
    }
    if (p->arena) cudaFree(p->arena);
    if (p->cells) cudaFree(p->cells);
    for (auto &t : p->tensors)
        if (t.is_const && t.ptr) cudaFree(t.ptr);
    delete p;
    return TPT_OK;
}

int tpt_cuda_plan_add_tensor(tpt_cuda_plan *p, int dtype, size_t numel, int *id) {
    CHECK_PLAN(p);
    if (p->finalized || !id || (dtype != TPT_DT_F32 && dtype != TPT_DT_I8)) return TPT_INVALID;
    PlanTensor t;
    t.dtype = dtype;
    t.numel = numel;
    p->tensors.push_back(t);
    *id = (int)p->tensors.size() - 1;
    return TPT_OK;
}

int tpt_cuda_plan_add_const(tpt_cuda_plan *p, const float *host, size_t numel, int *id) {
    CHECK_PLAN(p);
    if (!id || (!host && numel)) return TPT_INVALID;
    PlanTensor t;
    t.numel = numel;
    t.is_const = true;
    cudaError_t e = cudaMalloc(&t.ptr, numel ? numel * 4 : 4);
    if (e == cudaSuccess && numel) e = cudaMemcpy(t.ptr, host, numel * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaGetLastError();
        if (t.ptr) cudaFree(t.ptr);
        return cuda_fail(p->ctx, e, "plan constant upload");
    }
    p->tensors.push_back(t);
    *id = (int)p->tensors.size() - 1;
    return TPT_OK;
}

int tpt_cuda_plan_add_op(tpt_cuda_plan *p, const tpt_plan_op *op) {
    CHECK_PLAN(p);
    if (!op || p->finalized) return TPT_INVALID;
    if (!valid_id(p, op->in0) || !valid_id(p, op->out)) return TPT_INVALID;
    if ((op->in1 >= 0 && !valid_id(p, op->in1)) || (op->in2 >= 0 && !valid_id(p, op->in2))) return TPT_INVALID;
    if (op->kind == TPT_OP_LINEAR_W8A8 && (!op->w || op->w->kind != 8)) return TPT_INVALID;
    if (op->kind < TPT_OP_QUANTIZE || op->kind > TPT_OP_BATCHED_MATMUL) return TPT_UNSUPPORTED;
    if (op->kind >= TPT_OP_BINARY) {
        const int st = validate_graph_op(p, *op);
        if (st) return st;
    }
    if (op->kind == TPT_OP_GEMM_F32) {
        size_t mk = 0, kn = 0, mn = 0;
        const size_t m = op->dims[0], k = op->dims[1], n = op->dims[2];
        if (!checked_mul(m, k, &mk) || !checked_mul(k, n, &kn) || !checked_mul(m, n, &mn) ||
            p->tensors[op->in0].numel != mk || p->tensors[op->in1].numel != kn || p->tensors[op->out].numel != mn)
            return TPT_INVALID;
        if (op->in2 >= 0 && p->tensors[op->in2].numel != n && p->tensors[op->in2].numel != mn) return TPT_INVALID;
    }
    if (op->kind == TPT_OP_ALLGATHER) {
        const PlanTensor &a = p->tensors[op->in0], &b = p->tensors[op->out];
        if (a.dtype != b.dtype || op->dims[0] > a.numel) return TPT_INVALID;
    }
    if (op->kind == TPT_OP_PANELS_TO_ROWS) {
        const PlanTensor &a = p->tensors[op->in0], &b = p->tensors[op->out];
        size_t n = 0;
        if (a.dtype != TPT_DT_I8 || b.dtype != TPT_DT_I8 || op->dims[0] == 0 || op->dims[2] == 0 ||
            !checked_mul(op->dims[0] * op->dims[2], op->dims[1], &n) || n > a.numel || n > b.numel)
            return TPT_INVALID;
    }
    PlanOp po;
    po.op = *op;
    if (op->kind == TPT_OP_QUANTIZE || op->kind == TPT_OP_NCHW_TO_NHWC_Q8) {
        po.cell = p->n_cells++;
        po.frozen = op->f0;  // > 0: a static scale given by the caller
    }
    p->ops.push_back(po);
    return TPT_OK;
}

// Arena offsets by liveness. A tensor lives from its first writer (less the
// span of the longest run-time fusion, 3 ops: a fused launch at op i writes
// the outputs of ops i+1 .. i+3) to its last reader; graph inputs (no writer)
// from before the first op; kept tensors to the end. Tensors whose lifetimes
// are disjoint share bytes; every placement is the lowest 256-byte aligned
// offset free over the tensor's whole lifetime.
static size_t liveness_layout(tpt_cuda_plan *p) {
    const int nt = (int)p->tensors.size(), no = (int)p->ops.size();
    std::vector<int> first_w(nt, INT32_MAX), last_use(nt, -1);
    for (int i = 0; i < no; i++) {
        const tpt_plan_op &o = p->ops[i].op;
        if (o.out >= 0) {
            first_w[o.out] = std::min(first_w[o.out], i);
            last_use[o.out] = std::max(last_use[o.out], i);
        }
        for (int id : {o.in0, o.in1, o.in2})
            if (id >= 0) last_use[id] = std::max(last_use[id], i);
    }
    struct Iv {
        int t, start, end;
        size_t size, off;
    };
    std::vector<Iv> iv;
    for (int t = 0; t < nt; t++) {
        const PlanTensor &T = p->tensors[t];
        if (T.is_const) continue;
        Iv v;
        v.t = t;
        v.start = first_w[t] == INT32_MAX ? -4 : first_w[t] - 3;
        v.end = p->keep[t] ? INT32_MAX : std::max(last_use[t], v.start);
        v.size = (T.numel * dt_size(T.dtype) + 255) & ~size_t(255);
        v.off = 0;
        iv.push_back(v);
    }
    std::vector<Iv *> placed;
    size_t top = 0;
    for (auto &v : iv) {
        std::vector<std::pair<size_t, size_t>> busy;  // [off, off + size) of overlapping lifetimes
        for (Iv *u : placed)
            if (!(u->end < v.start || v.end < u->start)) busy.push_back({u->off, u->off + u->size});
        std::sort(busy.begin(), busy.end());
        size_t off = 0;
        for (auto &b : busy) {
            if (off + v.size <= b.first) break;
            off = std::max(off, b.second);
        }
        v.off = off;
        top = std::max(top, off + v.size);
        placed.push_back(&v);
    }
    for (auto &v : iv) p->tensors[v.t].offset = v.off;
    return top;
}

int tpt_cuda_plan_finalize(tpt_cuda_plan *p) {
    CHECK_PLAN(p);
    if (p->finalized) return TPT_INVALID;
    size_t off = 0;
    if (p->reuse) {
        p->keep.resize(p->tensors.size(), 0);
        off = liveness_layout(p);
    } else {
        for (auto &t : p->tensors) {
            if (t.is_const) continue;
            t.offset = off;
            off += (t.numel * dt_size(t.dtype) + 255) & ~size_t(255);
        }
    }
    p->arena_bytes = off;
    cudaError_t e = cudaMalloc(&p->arena, off ? off : 256);
    if (e == cudaSuccess) e = cudaMalloc(&p->cells, (size_t)(p->n_cells ? p->n_cells : 1) * 4);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_fail(p->ctx, e, "plan arena");
    }
    for (auto &t : p->tensors)
        if (!t.is_const) t.ptr = p->arena + t.offset;
    p->cal_max.assign(p->n_cells, 0.0f);
    for (auto &t : p->tensors) t.readers = 0;
    for (auto &po : p->ops) {
        const tpt_plan_op &o = po.op;
        for (int id : {o.in0, o.in1, o.in2})
            if (id >= 0) p->tensors[id].readers++;
    }
    p->finalized = true;
    return TPT_OK;
}

int tpt_cuda_plan_reuse_arena(tpt_cuda_plan *p, const int *keep_ids, size_t n_keep) {
    CHECK_PLAN(p);
    if (p->finalized || (n_keep && !keep_ids)) return TPT_INVALID;
    p->keep.assign(p->tensors.size(), 0);
    for (size_t i = 0; i < n_keep; i++) {
        if (!valid_id(p, keep_ids[i])) return TPT_INVALID;
        p->keep[keep_ids[i]] = 1;
    }
    p->reuse = true;
    return TPT_OK;
}

int tpt_cuda_plan_set_comm(tpt_cuda_plan *p, tpt_cuda_comm *comm) {
    CHECK_PLAN(p);
    drop_graph(p);
    p->comm = comm;
    return TPT_OK;
}

int tpt_cuda_plan_arena_bytes(tpt_cuda_plan *p, size_t *bytes) {
    if (!p || !bytes) return TPT_INVALID;
    *bytes = p->arena_bytes;
    return TPT_OK;
}

int tpt_cuda_plan_tensor_ptr(tpt_cuda_plan *p, int id, void **dev) {
    CHECK_PLAN(p);
    if (!p->finalized || !valid_id(p, id) || !dev) return TPT_INVALID;
    *dev = p->tensors[id].ptr;
    return TPT_OK;
}

int tpt_cuda_plan_set_calibration(tpt_cuda_plan *p, int on) {
    CHECK_PLAN(p);
    drop_graph(p);
    p->calibrating = on != 0;
    return TPT_OK;
}

int tpt_cuda_plan_set_graph(tpt_cuda_plan *p, int on) {
    CHECK_PLAN(p);
    drop_graph(p);
    p->use_graph = on != 0;
    return TPT_OK;
}

int tpt_cuda_plan_freeze_scales(tpt_cuda_plan *p) {
    CHECK_PLAN(p);
    for (auto &po : p->ops)
        if (po.cell >= 0 && !(po.op.f0 > 0.0f)) {
            const float m = p->cal_max[po.cell];
            po.frozen = m == 0.0f ? 1.0f : m / 127.0f;
        }
    drop_graph(p);
    p->calibrating = false;
    return TPT_OK;
}

int tpt_cuda_plan_get_scales(tpt_cuda_plan *p, float *scales, size_t n, size_t *count) {
    CHECK_PLAN(p);
    size_t c = 0;
    for (auto &po : p->ops)
        if (po.cell >= 0) {
            if (scales && c < n) scales[c] = po.frozen;
            c++;
        }
    if (count) *count = c;
    return TPT_OK;
}

int tpt_cuda_plan_set_scales(tpt_cuda_plan *p, const float *scales, size_t n) {
    CHECK_PLAN(p);
    if (!scales || n != (size_t)p->n_cells) return TPT_INVALID;
    for (size_t i = 0; i < n; i++)
        if (!(scales[i] > 0.0f)) return TPT_INVALID;
    size_t c = 0;
    for (auto &po : p->ops)
        if (po.cell >= 0) po.frozen = scales[c++];
    drop_graph(p);
    p->calibrating = false;
    return TPT_OK;
}

namespace {
bool is_output(const int *out_ids, size_t n_out, int id) {
    for (size_t i = 0; i < n_out; i++)
        if (out_ids[i] == id) return true;
    return false;
}

// With frozen scales, LINEAR_W8A8 -> QUANTIZE of its f32 output (read by no
// other op and not fetched by the caller) runs as one launch whose epilogue
// writes the int8 tensor (clamp(roundf(y / s)), the QUANTIZE op's arithmetic):
// the f32 tensor is neither written nor read back.
int run_ops(tpt_cuda_plan *p, const int *out_ids, size_t n_out) {
    for (size_t i = 0; i < p->ops.size(); i++) {
        PlanOp &po = p->ops[i];
        const tpt_plan_op &o = po.op;
        // IM2COL -> LINEAR_W8A8 of its rows (read by no other op, not fetched):
        // one implicit-GEMM convolution launch gathers the rows from the NHWC
        // tensor instead of writing and re-reading them; a QUANTIZE of the f32
        // result folds into its epilogue as for a plain LINEAR. An ADD_ACT of
        // the result (read by nothing else) and another tensor (a residual)
        // folds in too: the epilogue adds the residual, applies the activation
        // and writes the sum (and, with a QUANTIZE of the sum after it, also
        // its int8 copy), so the conv output is neither written nor read back.
        // IM2COL -> LINEAR_W8A8 (+ReLU) -> MAXPOOL 3x3/2/1 of the conv output (the
        // conv rows and the conv output read by nothing else, neither fetched):
        // the ResNet stem in its 16-channel 4x4 form runs fused with its pool, so
        // the conv output is never written; a QUANTIZE of the pooled tensor folds
        // in (its f32 copy is still written: a residual reads it).
        if (o.kind == TPT_OP_IM2COL && i + 2 < p->ops.size()) {
            const tpt_plan_op &l = p->ops[i + 1].op, &mp = p->ops[i + 2].op;
            const PlanTensor &col = p->tensors[o.out], &yt = p->tensors[l.out];
            const size_t *d = o.dims, *md = mp.dims;
            if (l.kind == TPT_OP_LINEAR_W8A8 && l.in0 == o.out && col.readers == 1 &&
                !is_output(out_ids, n_out, o.out) && mp.kind == TPT_OP_MAXPOOL_NHWC && mp.in0 == l.out &&
                yt.readers == 1 && !is_output(out_ids, n_out, l.out) && md[0] == d[0] && md[1] == d[10] &&
                md[2] == d[11] && md[3] == l.w->n && md[4] == 3 && md[5] == 3 && md[6] == 2 && md[7] == 2 &&
                md[8] == 1 && md[9] == 1) {
                const float sa = p->tensors[o.in0].scale;
                p->tensors[o.out].scale = sa;
                int8_t *qo = nullptr;
                float qs = 0.0f;
                size_t fused = 2;
                if (!p->calibrating && i + 3 < p->ops.size()) {
                    PlanOp &nq = p->ops[i + 3];
                    const tpt_plan_op &q = nq.op;
                    if (q.kind == TPT_OP_QUANTIZE && q.in0 == mp.out && q.dims[1] == 0 && nq.frozen > 0.0f &&
                        q.dims[0] == p->tensors[mp.out].numel) {
                        qo = Q(p, q.out);
                        qs = nq.frozen;
                        fused = 3;
                    }
                }
                bool handled = false;
                int st = launch_stem_pool(p->ctx, Q(p, o.in0), (int)d[0], (int)d[1], (int)d[2], (int)d[3], (int)d[4],
                                          (int)d[5], (int)d[6], (int)d[7], (int)d[8], (int)d[9], (int)d[10],
                                          (int)d[11], l.w, sa, F(p, l.in1), l.act, (int)md[10], (int)md[11],
                                          F(p, mp.out), qo, qs, &handled);
                if (st) return st;
                if (handled) {
                    if (qo) p->tensors[p->ops[i + 3].op.out].scale = qs;
                    i += fused;
                    continue;
                }
            }
        }
        if (o.kind == TPT_OP_IM2COL && i + 1 < p->ops.size()) {
            const tpt_plan_op &l = p->ops[i + 1].op;
            const PlanTensor &col = p->tensors[o.out];
            if (l.kind == TPT_OP_LINEAR_W8A8 && l.in0 == o.out && col.readers == 1 &&
                !is_output(out_ids, n_out, o.out)) {
                const float sa = p->tensors[o.in0].scale;
                p->tensors[o.out].scale = sa;
                Requant rq;
                Residual res;
                float *y = F(p, l.out);
                int q_op = -1;
                size_t fused = 1;
                const PlanTensor &t = p->tensors[l.out];
                const bool private_out = t.readers == 1 && !is_output(out_ids, n_out, l.out);
                if (private_out && i + 2 < p->ops.size()) {
                    const tpt_plan_op &a = p->ops[i + 2].op;
                    if (a.kind == TPT_OP_ADD_ACT && (a.in0 == l.out) != (a.in1 == l.out) && a.dims[0] == t.numel) {
                        res.r = F(p, a.in0 == l.out ? a.in1 : a.in0);
                        res.act = a.act;
                        y = F(p, a.out);
                        fused = 2;
                    }
                }
                const size_t qi = i + 1 + fused;  // the op after the conv (and its residual add)
                if (!p->calibrating && qi < p->ops.size()) {
                    PlanOp &nq = p->ops[qi];
                    const tpt_plan_op &q = nq.op;
                    const int src = fused == 2 ? p->ops[i + 2].op.out : l.out;
                    // without a residual the f32 output is dropped, so it must be private;
                    // the residual sum is still written (a later op reads it)
                    if (q.kind == TPT_OP_QUANTIZE && q.in0 == src && q.dims[1] == 0 && nq.frozen > 0.0f &&
                        q.dims[0] == p->tensors[src].numel && (fused == 2 || private_out)) {
                        rq.q = Q(p, q.out);
                        rq.scale = nq.frozen;
                        if (fused == 1) y = nullptr;
                        q_op = (int)qi;
                        fused++;
                    }
                }
                const size_t *d = o.dims;
                bool handled = false;
                int st = launch_conv_w8a8(p->ctx, Q(p, o.in0), (int)d[0], (int)d[1], (int)d[2], (int)d[3], (int)d[4],
                                          (int)d[5], (int)d[6], (int)d[7], (int)d[8], (int)d[9], (int)d[10],
                                          (int)d[11], l.w, sa, F(p, l.in1), l.act, y, &handled, rq, res);
                if (st) return st;
                if (handled) {
                    if (q_op >= 0) p->tensors[p->ops[q_op].op.out].scale = rq.scale;
                    i += fused;
                    continue;
                }
            }
        }
        if (!p->calibrating && o.kind == TPT_OP_LINEAR_W8A8 && i + 1 < p->ops.size()) {
            PlanOp &nq = p->ops[i + 1];
            const tpt_plan_op &q = nq.op;
            const PlanTensor &t = p->tensors[o.out];
            if (q.kind == TPT_OP_QUANTIZE && q.in0 == o.out && q.dims[1] == 0 && nq.frozen > 0.0f &&
                t.readers == 1 && q.dims[0] == t.numel && !is_output(out_ids, n_out, o.out)) {
                Requant rq;
                rq.q = Q(p, q.out);
                rq.scale = nq.frozen;
                p->tensors[q.out].scale = nq.frozen;
                int st = launch_w8a8(p->ctx, Q(p, o.in0), o.dims[0], o.w->k, o.w, p->tensors[o.in0].scale,
                                     F(p, o.in1), o.act, nullptr, nullptr, rq);
                if (st) return st;
                i++;
                continue;
            }
        }
        // MATMUL_F32 -> SOFTMAX of its rows (at most 16 wide): one launch writes
        // both tensors (the matmul's output is still written, for its other
        // readers or the caller); the softmax has k_softmax_warp's arithmetic
        if (o.kind == TPT_OP_MATMUL_F32 && i + 1 < p->ops.size()) {
            const tpt_plan_op &sm = p->ops[i + 1].op;
            if (sm.kind == TPT_OP_SOFTMAX && sm.in0 == o.out && sm.dims[0] == o.dims[0] && sm.dims[1] == o.dims[2] &&
                o.dims[2] <= 16) {
                bool handled = false;
                int st = launch_matmul_f32_softmax(p->ctx, F(p, o.in0), F(p, o.in1), F(p, o.in2), o.act, F(p, o.out),
                                                   F(p, sm.out), o.dims[0], o.dims[1], o.dims[2], &handled);
                if (st) return st;
                if (handled) {
                    i++;
                    continue;
                }
            }
        }
        // ATTENTION -> QUANTIZE of a context read by nothing else: int8 straight from the kernel
        if (!p->calibrating && o.kind == TPT_OP_ATTENTION && i + 1 < p->ops.size()) {
            PlanOp &nq = p->ops[i + 1];
            const tpt_plan_op &q = nq.op;
            const PlanTensor &t = p->tensors[o.out];
            if (q.kind == TPT_OP_QUANTIZE && q.in0 == o.out && q.dims[1] == 0 && nq.frozen > 0.0f &&
                t.readers == 1 && q.dims[0] == t.numel && !is_output(out_ids, n_out, o.out)) {
                p->tensors[q.out].scale = nq.frozen;
                int st = launch_attention(p->ctx, F(p, o.in0), F(p, o.out), (int)o.dims[0], (int)o.dims[1],
                                          (int)o.dims[2], (int)o.dims[3], o.f0, Q(p, q.out), nq.frozen);
                if (st) return st;
                i++;
                continue;
            }
        }
        // ADD_ACT (no activation) -> LAYERNORM of the sum (read by no other op,
        // not fetched): the layernorm adds its two inputs itself (the same f32
        // add), so the sum is neither written nor read back; a QUANTIZE of the
        // layernorm's output folds in as below.
        if (o.kind == TPT_OP_ADD_ACT && o.act == 0 && i + 1 < p->ops.size()) {
            const tpt_plan_op &l = p->ops[i + 1].op;
            const PlanTensor &t = p->tensors[o.out];
            if (l.kind == TPT_OP_LAYERNORM && l.in0 == o.out && t.readers == 1 && !is_output(out_ids, n_out, o.out) &&
                l.dims[0] * l.dims[1] == o.dims[0]) {
                int8_t *qo = nullptr;
                float qs = 0.0f;
                size_t fused = 1;
                if (!p->calibrating && i + 2 < p->ops.size()) {
                    PlanOp &nq = p->ops[i + 2];
                    const tpt_plan_op &q = nq.op;
                    if (q.kind == TPT_OP_QUANTIZE && q.in0 == l.out && q.dims[1] == 0 && nq.frozen > 0.0f &&
                        q.dims[0] == p->tensors[l.out].numel) {
                        qo = Q(p, q.out);
                        qs = nq.frozen;
                        p->tensors[q.out].scale = qs;
                        fused = 2;
                    }
                }
                int st = launch_layernorm(p->ctx, F(p, o.in0), F(p, l.in1), F(p, l.in2), F(p, l.out), l.dims[0],
                                          l.dims[1], l.f0, qo, qs, F(p, o.in1));
                if (st) return st;
                i += fused;
                continue;
            }
        }
        // ADD_ACT / LAYERNORM / MAXPOOL -> QUANTIZE of its output: one pass writes
        // the f32 tensor (still read later, e.g. by a residual) and its int8 copy
        if (!p->calibrating &&
            (o.kind == TPT_OP_ADD_ACT || o.kind == TPT_OP_LAYERNORM ||
             (o.kind == TPT_OP_MAXPOOL_NHWC && o.dims[3] % 4 == 0)) &&
            i + 1 < p->ops.size()) {
            PlanOp &nq = p->ops[i + 1];
            const tpt_plan_op &q = nq.op;
            const PlanTensor &t = p->tensors[o.out];
            if (q.kind == TPT_OP_QUANTIZE && q.in0 == o.out && q.dims[1] == 0 && nq.frozen > 0.0f &&
                q.dims[0] == t.numel) {
                p->tensors[q.out].scale = nq.frozen;
                const size_t *d = o.dims;
                int st = o.kind == TPT_OP_ADD_ACT
                             ? launch_add_act(p->ctx, F(p, o.in0), F(p, o.in1), F(p, o.out), d[0], o.act,
                                              Q(p, q.out), nq.frozen)
                         : o.kind == TPT_OP_LAYERNORM
                             ? launch_layernorm(p->ctx, F(p, o.in0), F(p, o.in1), F(p, o.in2), F(p, o.out), d[0], d[1],
                                                o.f0, Q(p, q.out), nq.frozen)
                             : launch_maxpool_nhwc(p->ctx, F(p, o.in0), F(p, o.out), (int)d[0], (int)d[1], (int)d[2],
                                                   (int)d[3], (int)d[4], (int)d[5], (int)d[6], (int)d[7], (int)d[8],
                                                   (int)d[9], (int)d[10], (int)d[11], Q(p, q.out), nq.frozen);
                if (st) return st;
                i++;
                continue;
            }
        }
        int st = run_op(p, po);
        if (st) return st;
    }
    return TPT_OK;
}

// run_ops, or its recorded replay. The first run after a change goes direct
// (sizing every workspace the ops use), then the same sequence is recorded;
// later runs launch the recording.
int run_plan(tpt_cuda_plan *p, const int *out_ids, size_t n_out) {
    // a plan with a communicator records its all-gathers too (NCCL collectives
    // are captured as graph nodes); calibration, whose scales are agreed by an
    // all-reduce read back on the host, always runs direct
    if (!p->use_graph || p->calibrating) return run_ops(p, out_ids, n_out);
    tpt_cuda_ctx *ctx = p->ctx;
    const std::vector<int> key(out_ids, out_ids + n_out);
    if (p->graph && key == p->graph_out) {
        if (tpt_cuda_graph_launch(ctx, p->graph) == TPT_OK) return TPT_OK;
        drop_graph(p);  // a workspace moved: record again below
    }
    drop_graph(p);
    int st = run_ops(p, out_ids, n_out);
    if (st) return st;
    st = tpt_cuda_capture_begin(ctx);
    if (st) return st;
    const int st_ops = run_ops(p, out_ids, n_out);
    tpt_cuda_graph *g = nullptr;
    st = tpt_cuda_capture_end(ctx, &g);
    if (st_ops) {
        if (g) tpt_cuda_graph_destroy(g);
        return st_ops;
    }
    if (st) return st;
    p->graph = g;
    p->graph_out = key;
    return TPT_OK;
}
}  // namespace

int tpt_cuda_plan_run_device(tpt_cuda_plan *p) {
    CHECK_PLAN(p);
    if (!p->finalized) return TPT_INVALID;
    return run_plan(p, nullptr, 0);
}

int tpt_cuda_plan_run(tpt_cuda_plan *p, const int *in_ids, const float *const *inputs, size_t n_in,
                      const int *out_ids, float *const *outputs, size_t n_out) {
    CHECK_PLAN(p);
    if (!p->finalized) return TPT_INVALID;
    for (size_t i = 0; i < n_in; i++) {
        if (!valid_id(p, in_ids[i])) return TPT_INVALID;
        const PlanTensor &t = p->tensors[in_ids[i]];
        int st = h2d(p->ctx, t.ptr, inputs[i], t.numel * dt_size(t.dtype));
        if (st) return st;
    }
    for (size_t i = 0; i < n_out; i++)
        if (!valid_id(p, out_ids[i]) || (p->reuse && !p->keep[out_ids[i]])) return TPT_INVALID;
    int st = run_plan(p, out_ids, n_out);
    if (st) return st;
    for (size_t i = 0; i < n_out; i++) {
        if (!valid_id(p, out_ids[i])) return TPT_INVALID;
        const PlanTensor &t = p->tensors[out_ids[i]];
        st = d2h(p->ctx, outputs[i], t.ptr, t.numel * dt_size(t.dtype));
        if (st) return st;
    }
    return sync_and_check(p->ctx);
}

// n_steps forward passes, step s reading inputs[s * n_in + i] and writing
// outputs[s * n_out + j]. Step s + 1's inputs travel host -> device on the
// context's copy stream into one of two staging buffers while step s computes;
// at the start of its step the compute stream waits for them and moves them
// into the input tensors (device to device); outputs return on the compute
// stream. With page-locked host buffers the H2D of the next batch overlaps the
// whole forward pass of the current one.
int tpt_cuda_plan_run_batches(tpt_cuda_plan *p, const int *in_ids, const float *const *inputs, size_t n_in,
                              const int *out_ids, float *const *outputs, size_t n_out, size_t n_steps) {
    CHECK_PLAN(p);
    if (!p->finalized || (n_in && (!in_ids || !inputs)) || (n_out && (!out_ids || !outputs))) return TPT_INVALID;
    size_t in_bytes = 0;
    std::vector<size_t> off(n_in);
    for (size_t i = 0; i < n_in; i++) {
        if (!valid_id(p, in_ids[i]) || p->tensors[in_ids[i]].is_const) return TPT_INVALID;
        const PlanTensor &t = p->tensors[in_ids[i]];
        off[i] = in_bytes;
        in_bytes += (t.numel * dt_size(t.dtype) + 255) & ~size_t(255);
    }
    for (size_t i = 0; i < n_out; i++)
        if (!valid_id(p, out_ids[i]) || (p->reuse && !p->keep[out_ids[i]])) return TPT_INVALID;
    if (n_steps == 0) return TPT_OK;
    tpt_cuda_ctx *ctx = p->ctx;
    int st = ensure_copy_streams(ctx);
    if (st) return st;
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < 2 && e == cudaSuccess; i++) {
        if (!p->ev_in[i]) e = cudaEventCreateWithFlags(&p->ev_in[i], cudaEventDisableTiming);
        if (e == cudaSuccess && !p->ev_free[i]) e = cudaEventCreateWithFlags(&p->ev_free[i], cudaEventDisableTiming);
    }
    if (e == cudaSuccess && p->stage_bytes < 2 * in_bytes) {
        if (p->stage) cudaFree(p->stage);
        p->stage = nullptr;
        p->stage_bytes = 0;
        e = cudaMalloc(&p->stage, 2 * in_bytes);
        if (e == cudaSuccess) p->stage_bytes = 2 * in_bytes;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cuda_fail(ctx, e, "batch pipeline set-up");
    }
    // the staging buffers may still be read by an earlier call's last step
    e = cudaStreamWaitEvent(ctx->copy_in, p->ev_free[0], 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(ctx->copy_in, p->ev_free[1], 0);
    auto upload = [&](size_t s) -> cudaError_t {
        char *dst = p->stage + (s & 1) * in_bytes;
        for (size_t i = 0; i < n_in; i++) {
            const PlanTensor &t = p->tensors[in_ids[i]];
            cudaError_t r = cudaMemcpyAsync(dst + off[i], inputs[s * n_in + i], t.numel * dt_size(t.dtype),
                                            cudaMemcpyHostToDevice, ctx->copy_in);
            if (r != cudaSuccess) return r;
        }
        return cudaEventRecord(p->ev_in[s & 1], ctx->copy_in);
    };
    if (e == cudaSuccess) e = upload(0);
    for (size_t s = 0; s < n_steps && e == cudaSuccess; s++) {
        const int b = (int)(s & 1);
        if (s + 1 < n_steps) {  // the next batch's inputs, once its buffer is free again
            e = cudaStreamWaitEvent(ctx->copy_in, p->ev_free[b ^ 1], 0);
            if (e == cudaSuccess) e = upload(s + 1);
            if (e != cudaSuccess) break;
        }
        e = cudaStreamWaitEvent(ctx->stream, p->ev_in[b], 0);
        for (size_t i = 0; i < n_in && e == cudaSuccess; i++) {
            const PlanTensor &t = p->tensors[in_ids[i]];
            e = cudaMemcpyAsync(t.ptr, p->stage + b * in_bytes + off[i], t.numel * dt_size(t.dtype),
                                cudaMemcpyDeviceToDevice, ctx->stream);
        }
        if (e == cudaSuccess) e = cudaEventRecord(p->ev_free[b], ctx->stream);
        if (e != cudaSuccess) break;
        st = run_plan(p, out_ids, n_out);
        if (st) {
            cudaStreamSynchronize(ctx->copy_in);
            return st;
        }
        for (size_t j = 0; j < n_out && e == cudaSuccess; j++) {
            const PlanTensor &t = p->tensors[out_ids[j]];
            e = cudaMemcpyAsync(outputs[s * n_out + j], t.ptr, t.numel * dt_size(t.dtype), cudaMemcpyDeviceToHost,
                                ctx->stream);
        }
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        cudaStreamSynchronize(ctx->copy_in);
        cudaStreamSynchronize(ctx->stream);
        return cuda_fail(ctx, e, "batch pipeline");
    }
    return sync_and_check(ctx);
}

}  // extern "C"
