// graph_ops.cu -- the remaining operators of the reference runtime's dispatch
// table (crates/tpt-infer-runtime/src/exec.rs:347-533) as device kernels, so a
// whole ComputationGraph lowers onto a plan with no host round trip:
//
//   BINARY         Add / Sub / Mul / Div with numpy broadcasting (kernels.rs:92-137)
//   POOL_NCHW      MaxPool2d / AveragePool2d over NCHW (kernels.rs:271-390)
//   BATCHNORM      inference BatchNorm, channel or element mode (kernels.rs:425-476)
//   TRANSPOSE      dimension permutation up to rank 8 (kernels.rs:484-532)
//   CONCAT_COPY    one input's slab of a Concat (kernels.rs:548-588, exec.rs:471-513)
//   BATCHED_MATMUL rank-3/4 MatMul with broadcast batch dimensions (the shape rule of
//                  crates/tpt-infer-onnx/src/shapes.rs:163-186; the reference runtime
//                  rejects rank != 2, exec.rs:360-362)
//
// Every kernel performs the reference's arithmetic per element in the
// reference's order (separately rounded operations, no contraction), so the
// results are bit-identical to the reference's CPU kernels. All index math is
// 64-bit; grids are grid-stride loops sized to the SM count.
#include "common.cuh"

namespace tpt {
namespace {

constexpr int GR = 8;  // MAX_RANK (crates/tpt-infer-core/src/shape.rs:4)

struct Dims8 {
    size_t d[GR];
};

// out[i] = a[ai] op b[bi]; dims padded to rank 8 with leading 1s, an operand's
// dimension either equals the output's or is 1 (bit set in its mask), the
// map_coord rule of kernels.rs:60-66.
__global__ void k_binary(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ out,
                         Dims8 od, unsigned amask, unsigned bmask, int op, size_t n) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        size_t rem = i, ai = 0, bi = 0, as = 1, bs = 1;
#pragma unroll
        for (int d = GR - 1; d >= 0; d--) {
            const size_t c = rem % od.d[d];
            rem /= od.d[d];
            if (!(amask >> d & 1)) {
                ai += c * as;
                as *= od.d[d];
            }
            if (!(bmask >> d & 1)) {
                bi += c * bs;
                bs *= od.d[d];
            }
        }
        const float x = a[ai], y = b[bi];
        float r;
        if (op == 0)
            r = __fadd_rn(x, y);
        else if (op == 1)
            r = __fsub_rn(x, y);
        else if (op == 2)
            r = __fmul_rn(x, y);
        else
            r = __fdiv_rn(x, y);
        out[i] = r;
    }
}

// NCHW pooling, one thread per output. Max: -inf start, window taps in ky, kx
// order, padding skipped, a tap replaces the running best only when it is
// strictly greater (kernels.rs:271-325), so NaN taps are ignored and the first
// of equal taps (e.g. -0 before +0) is kept. Average: the in-bounds taps summed in ky, kx order,
// divided by their count (count_include_pad = 0; 0 when no tap is in bounds).
__global__ void k_pool_nchw(const float *__restrict__ x, float *__restrict__ y, int avg, size_t NC, int H, int W,
                            int KH, int KW, int sh, int sw, int ph, int pw, int OH, int OW) {
    pdl_wait();
    pdl_trigger();
    const size_t n = NC * OH * OW;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int ox = (int)(i % OW);
        const int oy = (int)(i / OW % OH);
        const size_t nc = i / ((size_t)OW * OH);
        const float *xp = x + nc * H * W;
        float acc = avg ? 0.0f : -INFINITY;
        int count = 0;
        for (int ky = 0; ky < KH; ky++) {
            const int yy = oy * sh + ky - ph;
            if (yy < 0 || yy >= H) continue;
            for (int kx = 0; kx < KW; kx++) {
                const int xx = ox * sw + kx - pw;
                if (xx < 0 || xx >= W) continue;
                const float v = xp[(size_t)yy * W + xx];
                if (avg) {
                    acc = __fadd_rn(acc, v);
                    count++;
                } else if (v > acc) {  // a strict comparison, as the reference's
                    acc = v;
                }
            }
        }
        y[i] = avg ? (count == 0 ? 0.0f : __fdiv_rn(acc, (float)count)) : acc;
    }
}

// The reference's own square root (kernels.rs:397-411): the exponent halved
// through the bit pattern, then four Newton steps y = 0.5 (y + x / y), each
// operation rounded separately. Not IEEE sqrt; restated so BatchNorm matches.
__device__ __forceinline__ float sqrt_ref(float x) {
    if (isnan(x) || x < 0.0f) return __int_as_float(0x7fc00000);
    if (x == 0.0f || isinf(x)) return x;
    float y = __uint_as_float((__float_as_uint(x) >> 1) + (1u << 29));
#pragma unroll
    for (int i = 0; i < 4; i++) y = __fmul_rn(0.5f, __fadd_rn(y, __fdiv_rn(x, y)));
    return y;
}

// BatchNorm (kernels.rs:425-476). params = [scale | bias | mean | var], plen
// each. Channel mode (x rank 4, plen = C): f = scale[c] / sqrt(var[c] + eps)
// (as 1 / sqrt, then a multiply), g = bias[c] - mean[c] * f, out = x * f + g.
// Element mode (plen = numel): out = (x - mean) * f + bias.
__global__ void k_batchnorm(const float *__restrict__ x, const float *__restrict__ prm, float *__restrict__ y,
                            size_t n, size_t plen, size_t hw, int channel_mode, float eps) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t c = channel_mode ? (i / hw) % plen : i;
        const float inv = __fdiv_rn(1.0f, sqrt_ref(__fadd_rn(prm[3 * plen + c], eps)));
        const float f = __fmul_rn(prm[c], inv);
        if (channel_mode) {
            const float g = __fsub_rn(prm[plen + c], __fmul_rn(prm[2 * plen + c], f));
            y[i] = __fadd_rn(__fmul_rn(x[i], f), g);
        } else {
            y[i] = __fadd_rn(__fmul_rn(__fsub_rn(x[i], prm[2 * plen + c]), f), prm[plen + c]);
        }
    }
}

// Transpose (kernels.rs:484-532): out dims od, input dims xd, both padded to
// rank 8 (leading 1s, identity for the padded axes), out axis d reads input
// axis perm[d].
__global__ void k_transpose(const float *__restrict__ x, float *__restrict__ y, Dims8 od, Dims8 xstride_of_out,
                            size_t n) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        size_t rem = i, xi = 0;
#pragma unroll
        for (int d = GR - 1; d >= 0; d--) {
            const size_t c = rem % od.d[d];
            rem /= od.d[d];
            xi += c * xstride_of_out.d[d];
        }
        y[i] = x[xi];
    }
}

// One Concat input (concat_copy_one, kernels.rs:548-588): `outer` slabs of
// src_block values land at o * out_block + offset.
__global__ void k_concat_copy(const float *__restrict__ src, float *__restrict__ dst, size_t outer, size_t src_block,
                              size_t out_block, size_t offset) {
    pdl_wait();
    pdl_trigger();
    const size_t n = outer * src_block;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t o = i / src_block, r = i - o * src_block;
        dst[o * out_block + offset + r] = src[i];
    }
}

// Batched MatMul: for each batch index z (over the output's batch dims bd,
// padded to rank 6), C_z [m, n] = A_z [m, k] x B_z [k, n], A_z / B_z the
// broadcast batch slices (mask bit set: that batch dim is 1 in the operand).
// Per output one sequential k chain with a separately rounded multiply and
// add, the naive.rs:13-33 arithmetic, so each batch equals Backend::matmul of
// its slices bit for bit. 16x16 outputs per 256-thread CTA, k-slices of 32.
struct BatchMap {
    size_t bd[6];
    unsigned amask, bmask;
};
constexpr int BB = 16, BKS = 32;
__global__ void __launch_bounds__(256) k_bmm(const float *__restrict__ A, const float *__restrict__ B,
                                            float *__restrict__ Cout, int M, int N, int K, BatchMap bm) {
    pdl_wait();
    pdl_trigger();
    __shared__ float As[BKS][BB + 1];
    __shared__ float Bs[BKS][BB + 1];
    size_t rem = blockIdx.z, ao = 0, bo = 0, as = 1, bs = 1;
#pragma unroll
    for (int d = 5; d >= 0; d--) {
        const size_t c = rem % bm.bd[d];
        rem /= bm.bd[d];
        if (!(bm.amask >> d & 1)) {
            ao += c * as;
            as *= bm.bd[d];
        }
        if (!(bm.bmask >> d & 1)) {
            bo += c * bs;
            bs *= bm.bd[d];
        }
    }
    A += ao * (size_t)M * K;
    B += bo * (size_t)K * N;
    Cout += (size_t)blockIdx.z * M * N;
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BB, n0 = blockIdx.x * BB;
    float acc = 0.0f;
    for (int k0 = 0; k0 < K; k0 += BKS) {
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int e = tid + 256 * i;
            const int ar = e >> 5, ac = e & 31;
            const int m = m0 + ar, ka = k0 + ac;
            As[ac][ar] = (m < M && ka < K) ? A[(size_t)m * K + ka] : 0.0f;
            const int br = e >> 4, bc = e & 15;
            const int kb = k0 + br, n = n0 + bc;
            Bs[br][bc] = (kb < K && n < N) ? B[(size_t)kb * N + n] : 0.0f;
        }
        __syncthreads();
        const int kn = K - k0 < BKS ? K - k0 : BKS;
        for (int kk = 0; kk < kn; kk++) acc = __fadd_rn(acc, __fmul_rn(As[kk][ty], Bs[kk][tx]));
        __syncthreads();
    }
    const int m = m0 + ty, n = n0 + tx;
    if (m < M && n < N) Cout[(size_t)m * N + n] = acc;
}

}  // namespace
}  // namespace tpt

namespace tpt {

static unsigned go_grid(tpt_cuda_ctx *ctx, size_t n) { return grid_1d(n, 256, (unsigned)ctx->sm_count * 8); }

int launch_binary(tpt_cuda_ctx *ctx, const float *a, const float *b, float *out, const size_t od[8], unsigned amask,
                  unsigned bmask, int op, size_t n) {
    if (n == 0) return TPT_OK;
    Dims8 d;
    for (int i = 0; i < GR; i++) d.d[i] = od[i] ? od[i] : 1;
    launch_pdl(k_binary, go_grid(ctx, n), 256, 0, ctx->stream, a, b, out, d, amask, bmask, op, n);
    return after_launch(ctx, "binary");
}

int launch_pool_nchw(tpt_cuda_ctx *ctx, const float *x, float *y, int avg, size_t NC, int H, int W, int KH, int KW,
                     int sh, int sw, int ph, int pw, int OH, int OW) {
    const size_t n = NC * (size_t)OH * OW;
    if (n == 0) return TPT_OK;
    launch_pdl(k_pool_nchw, go_grid(ctx, n), 256, 0, ctx->stream, x, y, avg, NC, H, W, KH, KW, sh, sw, ph, pw, OH,
               OW);
    return after_launch(ctx, avg ? "average_pool2d" : "max_pool2d");
}

int launch_batchnorm(tpt_cuda_ctx *ctx, const float *x, const float *prm, float *y, size_t n, size_t plen, size_t hw,
                     int channel_mode, float eps) {
    if (n == 0) return TPT_OK;
    launch_pdl(k_batchnorm, go_grid(ctx, n), 256, 0, ctx->stream, x, prm, y, n, plen, hw ? hw : 1, channel_mode, eps);
    return after_launch(ctx, "batch_norm");
}

// xd: input dims padded to rank 8 (leading 1s); perm: out axis d reads input
// axis perm[d] (identity on the padded axes).
int launch_transpose(tpt_cuda_ctx *ctx, const float *x, float *y, const size_t xd[8], const size_t perm[8], size_t n) {
    if (n == 0) return TPT_OK;
    size_t xs[GR];
    size_t s = 1;
    for (int d = GR - 1; d >= 0; d--) {
        xs[d] = s;
        s *= xd[d];
    }
    Dims8 od, st;
    for (int d = 0; d < GR; d++) {
        od.d[d] = xd[perm[d]];
        st.d[d] = xs[perm[d]];
    }
    launch_pdl(k_transpose, go_grid(ctx, n), 256, 0, ctx->stream, x, y, od, st, n);
    return after_launch(ctx, "transpose");
}

int launch_concat_copy(tpt_cuda_ctx *ctx, const float *src, float *dst, size_t outer, size_t src_block,
                       size_t out_block, size_t offset) {
    const size_t n = outer * src_block;
    if (n == 0) return TPT_OK;
    launch_pdl(k_concat_copy, go_grid(ctx, n), 256, 0, ctx->stream, src, dst, outer, src_block, out_block, offset);
    return after_launch(ctx, "concat");
}

int launch_bmm(tpt_cuda_ctx *ctx, const float *a, const float *b, float *c, const size_t bd[6], unsigned amask,
               unsigned bmask, size_t m, size_t k, size_t n) {
    if (m > INT32_MAX || n > INT32_MAX || k > INT32_MAX) return TPT_UNSUPPORTED;
    BatchMap bm;
    size_t batch = 1;
    for (int i = 0; i < 6; i++) {
        bm.bd[i] = bd[i] ? bd[i] : 1;
        batch *= bm.bd[i];
    }
    bm.amask = amask;
    bm.bmask = bmask;
    if (batch == 0 || m == 0 || n == 0) return TPT_OK;
    if (k == 0) {
        cudaError_t e = cudaMemsetAsync(c, 0, batch * m * n * 4, ctx->stream);
        return e == cudaSuccess ? TPT_OK : cuda_fail(ctx, e, "batched matmul k=0 memset");
    }
    dim3 g((unsigned)((n + BB - 1) / BB), (unsigned)((m + BB - 1) / BB), (unsigned)batch);
    if (g.y > 65535 || batch > 65535) return TPT_UNSUPPORTED;
    launch_pdl(k_bmm, g, 256, 0, ctx->stream, a, b, c, (int)m, (int)n, (int)k, bm);
    return after_launch(ctx, "batched_matmul");
}

}  // namespace tpt
