// model_ops.cu -- device ops the model plans need besides the GEMMs:
// LayerNorm, fused attention, bias/residual adds, NHWC INT8 conv plumbing
// (layout change + quantize, im2col), pooling, per-tensor max-abs.
//
// Layout inside a plan: activations are row-major [rows, channels] (NHWC for
// images), so a conv's im2col rows and a GEMM's output rows are both
// [N*H*W, C] and no transposes are needed between layers.
#include <float.h>

#include "common.cuh"

namespace tpt {
namespace {

// ---------------------------------------------------------------- LayerNorm
// ONNX LayerNormalization over the last axis (the reference runtime lacks it:
// crates/tpt-infer-onnx/src/registry.rs:62 maps it to Custom): mean, biased
// variance, y = (x - mean) / sqrt(var + eps) * gamma + beta. One warp per row,
// the row held in registers (cols <= 32 * LN_MAX).
constexpr int LN_MAX = 32;
__global__ void k_layernorm(const float *__restrict__ x, const float *__restrict__ g, const float *__restrict__ b,
                            float *__restrict__ y, int rows, int cols, float eps) {
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    for (int r = warp; r < rows; r += nwarps) {
        const float *xr = x + (size_t)r * cols;
        float v[LN_MAX];
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < LN_MAX; i++) {
            const int c = lane + 32 * i;
            v[i] = c < cols ? xr[c] : 0.0f;
            s += v[i];
        }
        const float mean = __fdiv_rn(warp_sum(s), (float)cols);
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < LN_MAX; i++) {
            const int c = lane + 32 * i;
            const float d = c < cols ? v[i] - mean : 0.0f;
            q += d * d;
        }
        const float var = __fdiv_rn(warp_sum(q), (float)cols);
        const float inv = __fdiv_rn(1.0f, sqrtf(var + eps));
#pragma unroll
        for (int i = 0; i < LN_MAX; i++) {
            const int c = lane + 32 * i;
            if (c < cols) y[(size_t)r * cols + c] = (v[i] - mean) * inv * __ldg(g + c) + __ldg(b + c);
        }
    }
}

// ---------------------------------------------------------------- attention
// Fused softmax(Q K^T * scale) V per (batch, head) on f32, reading Q, K, V from
// the packed projection output qkv [B*S, 3*H*D] (Q | K | V along columns) and
// writing ctx [B*S, H*D]. One CTA per (batch, head, 64-query block); K and V of
// the head are staged in shared memory; each thread owns one query row and
// runs an online (streaming) softmax over key blocks of 16.
constexpr int AT_D = 64;    // head dimension
constexpr int AT_Q = 64;    // queries per CTA
constexpr int AT_KB = 16;   // keys per online-softmax block
__global__ void __launch_bounds__(AT_Q) k_attention(const float *__restrict__ qkv, float *__restrict__ out, int S,
                                                    int H, float scale) {
    extern __shared__ float sm[];
    float *Ks = sm;                 // [S][AT_D]
    float *Vs = sm + (size_t)S * AT_D;
    const int b = blockIdx.z, h = blockIdx.y, q0 = blockIdx.x * AT_Q;
    const int ld = 3 * H * AT_D;
    const float *base = qkv + (size_t)b * S * ld;
    for (int i = threadIdx.x; i < S * (AT_D / 4); i += blockDim.x) {
        const int j = i / (AT_D / 4), c4 = i - j * (AT_D / 4);
        const float4 kv = *reinterpret_cast<const float4 *>(base + (size_t)j * ld + H * AT_D + h * AT_D + 4 * c4);
        const float4 vv = *reinterpret_cast<const float4 *>(base + (size_t)j * ld + 2 * H * AT_D + h * AT_D + 4 * c4);
        *reinterpret_cast<float4 *>(Ks + j * AT_D + 4 * c4) = kv;
        *reinterpret_cast<float4 *>(Vs + j * AT_D + 4 * c4) = vv;
    }
    __syncthreads();
    const int qi = q0 + threadIdx.x;
    if (qi >= S) return;
    float q[AT_D], o[AT_D];
    const float *qr = base + (size_t)qi * ld + h * AT_D;
#pragma unroll
    for (int d = 0; d < AT_D; d += 4) {
        const float4 t = *reinterpret_cast<const float4 *>(qr + d);
        q[d] = t.x * scale;
        q[d + 1] = t.y * scale;
        q[d + 2] = t.z * scale;
        q[d + 3] = t.w * scale;
    }
#pragma unroll
    for (int d = 0; d < AT_D; d++) o[d] = 0.0f;
    float mrun = -INFINITY, lrun = 0.0f;
    for (int j0 = 0; j0 < S; j0 += AT_KB) {
        float sc[AT_KB];
        float bm = -INFINITY;
#pragma unroll
        for (int jj = 0; jj < AT_KB; jj++) {
            float a = -INFINITY;
            if (j0 + jj < S) {
                const float *kr = Ks + (j0 + jj) * AT_D;
                a = 0.0f;
#pragma unroll
                for (int d = 0; d < AT_D; d++) a = fmaf(q[d], kr[d], a);
            }
            sc[jj] = a;
            bm = fmaxf(bm, a);
        }
        const float mnew = fmaxf(mrun, bm);
        const float corr = expf(mrun - mnew);
        lrun *= corr;
#pragma unroll
        for (int d = 0; d < AT_D; d++) o[d] *= corr;
#pragma unroll
        for (int jj = 0; jj < AT_KB; jj++) {
            if (j0 + jj < S) {
                const float p = expf(sc[jj] - mnew);
                lrun += p;
                const float *vr = Vs + (j0 + jj) * AT_D;
#pragma unroll
                for (int d = 0; d < AT_D; d++) o[d] = fmaf(p, vr[d], o[d]);
            }
        }
        mrun = mnew;
    }
    const float inv = __fdiv_rn(1.0f, lrun);
    float *orow = out + ((size_t)b * S + qi) * (H * AT_D) + h * AT_D;
#pragma unroll
    for (int d = 0; d < AT_D; d += 4)
        *reinterpret_cast<float4 *>(orow + d) = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
}

// ---------------------------------------------------------------- adds
// y[r, c] = act(x[r, c] + bias[c]) (the runtime's broadcast bias add,
// crates/tpt-infer-runtime/src/kernels.rs:150-178, plus a fused activation)
__global__ void k_bias_act(const float *__restrict__ x, const float *__restrict__ bias, float *__restrict__ y,
                           size_t rows, int cols, int act) {
    const size_t n = rows * (size_t)cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v = x[i];
        if (bias) v = v + bias[i % cols];
        y[i] = apply_act(v, act);
    }
}

// y = act(a + b) element-wise (residual adds)
__global__ void k_add_act(const float4 *__restrict__ a, const float4 *__restrict__ b, float4 *__restrict__ y, size_t n4,
                          int act) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 x = a[i], z = b[i];
        y[i] = make_float4(apply_act(x.x + z.x, act), apply_act(x.y + z.y, act), apply_act(x.z + z.z, act),
                           apply_act(x.w + z.w, act));
    }
}

// ---------------------------------------------------------------- images
// NCHW f32 -> NHWC int8 with a static per-tensor scale:
// q = clamp(round(x / scale), -127, 127) (quant.rs:35-36)
__global__ void k_nchw_to_nhwc_q8(const float *__restrict__ x, int8_t *__restrict__ q, int N, int C, int HW,
                                  float scale) {
    const size_t total = (size_t)N * C * HW;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        // i indexes the NHWC output
        const int c = (int)(i % C);
        const size_t p = i / C;  // n*HW + hw
        const size_t n = p / HW, hw = p - n * HW;
        q[i] = round_clamp_i8(__fdiv_rn(x[(n * C + c) * HW + hw], scale), -127.0f, 127.0f);
    }
}

// im2col of an NHWC int8 tensor: row m = (n, oy, ox), column (ky, kx, c),
// zero for padded taps and for columns in [K, Kp).
__global__ void k_im2col_nhwc(const int8_t *__restrict__ x, int8_t *__restrict__ col, int N, int H, int W, int C,
                              int KH, int KW, int sh, int sw, int ph, int pw, int OH, int OW, int Kp) {
    const int K = KH * KW * C;
    if ((C & 15) == 0) {
        // 16-byte chunks: one chunk = 16 channels of one tap
        const int chunks = Kp >> 4;
        const size_t total = (size_t)N * OH * OW * chunks;
        for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
            const int ch = (int)(i % chunks);
            const size_t m = i / chunks;
            const int kk = ch << 4;
            int4 v = make_int4(0, 0, 0, 0);
            if (kk < K) {
                const int tap = kk / C, c = kk - tap * C;
                const int ky = tap / KW, kx = tap - ky * KW;
                const int ox = (int)(m % OW);
                const size_t t2 = m / OW;
                const int oy = (int)(t2 % OH);
                const int n = (int)(t2 / OH);
                const int iy = oy * sh + ky - ph, ix = ox * sw + kx - pw;
                if (iy >= 0 && iy < H && ix >= 0 && ix < W)
                    v = *reinterpret_cast<const int4 *>(x + (((size_t)n * H + iy) * W + ix) * C + c);
            }
            *reinterpret_cast<int4 *>(col + m * Kp + kk) = v;
        }
    } else {
        const size_t total = (size_t)N * OH * OW * Kp;
        for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
            const int kk = (int)(i % Kp);
            const size_t m = i / Kp;
            int8_t v = 0;
            if (kk < K) {
                const int tap = kk / C, c = kk - tap * C;
                const int ky = tap / KW, kx = tap - ky * KW;
                const int ox = (int)(m % OW);
                const size_t t2 = m / OW;
                const int oy = (int)(t2 % OH);
                const int n = (int)(t2 / OH);
                const int iy = oy * sh + ky - ph, ix = ox * sw + kx - pw;
                if (iy >= 0 && iy < H && ix >= 0 && ix < W) v = x[(((size_t)n * H + iy) * W + ix) * C + c];
            }
            col[i] = v;
        }
    }
}

// max pool on NHWC f32, padding as -inf (kernels.rs:271-325)
__global__ void k_maxpool_nhwc(const float *__restrict__ x, float *__restrict__ y, int N, int H, int W, int C, int KH,
                               int KW, int sh, int sw, int ph, int pw, int OH, int OW) {
    const size_t total = (size_t)N * OH * OW * C;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % C);
        size_t t = i / C;
        const int ox = (int)(t % OW);
        t /= OW;
        const int oy = (int)(t % OH);
        const int n = (int)(t / OH);
        float best = -INFINITY;
        for (int ky = 0; ky < KH; ky++) {
            const int iy = oy * sh + ky - ph;
            if (iy < 0 || iy >= H) continue;
            for (int kx = 0; kx < KW; kx++) {
                const int ix = ox * sw + kx - pw;
                if (ix < 0 || ix >= W) continue;
                const float v = x[(((size_t)n * H + iy) * W + ix) * C + c];
                if (v > best) best = v;
            }
        }
        y[i] = best;
    }
}

// global average pool NHWC f32 [N, HW, C] -> [N, C]: sequential sum over the
// window, then divide by the count (kernels.rs:335-390 with kernel = spatial)
__global__ void k_gap_nhwc(const float *__restrict__ x, float *__restrict__ y, int N, int HW, int C) {
    const size_t total = (size_t)N * C;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % C);
        const size_t n = i / C;
        float acc = 0.0f;
        for (int p = 0; p < HW; p++) acc += x[(n * HW + p) * C + c];
        y[i] = __fdiv_rn(acc, (float)HW);
    }
}

// max |x| folded into *cell (non-negative float bits; atomicMax), used to
// calibrate static activation scales
__global__ void k_absmax_acc(const float *__restrict__ x, size_t n, unsigned *cell) {
    float m = 0.0f;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(x[i]));
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) atomicMax(cell, __float_as_uint(m));
}

}  // namespace

int launch_layernorm(tpt_cuda_ctx *ctx, const float *x, const float *g, const float *b, float *y, size_t rows,
                     size_t cols, float eps) {
    if (cols > 32 * LN_MAX || rows > INT32_MAX) return TPT_UNSUPPORTED;
    k_layernorm<<<grid_1d(rows * 32, 256, (unsigned)ctx->sm_count * 16), 256, 0, ctx->stream>>>(x, g, b, y, (int)rows,
                                                                                              (int)cols, eps);
    return after_launch(ctx, "layernorm");
}

int launch_attention(tpt_cuda_ctx *ctx, const float *qkv, float *out, int B, int S, int H, int D, float scale) {
    if (D != AT_D || S <= 0 || S > 256) return TPT_UNSUPPORTED;
    const size_t smem = (size_t)2 * S * AT_D * sizeof(float);
    static bool attr[64] = {};
    if (!attr[ctx->device & 63]) {
        cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 256 * AT_D * 4);
        attr[ctx->device & 63] = true;
    }
    dim3 grid((unsigned)((S + AT_Q - 1) / AT_Q), (unsigned)H, (unsigned)B);
    k_attention<<<grid, AT_Q, smem, ctx->stream>>>(qkv, out, S, H, scale);
    return after_launch(ctx, "attention");
}

int launch_bias_act(tpt_cuda_ctx *ctx, const float *x, const float *bias, float *y, size_t rows, size_t cols, int act) {
    k_bias_act<<<grid_1d(rows * cols, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream>>>(x, bias, y, rows,
                                                                                              (int)cols, act);
    return after_launch(ctx, "bias_act");
}

int launch_add_act(tpt_cuda_ctx *ctx, const float *a, const float *b, float *y, size_t n, int act) {
    if (n % 4) return TPT_UNSUPPORTED;
    k_add_act<<<grid_1d(n / 4, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream>>>(
        (const float4 *)a, (const float4 *)b, (float4 *)y, n / 4, act);
    return after_launch(ctx, "add_act");
}

int launch_nchw_to_nhwc_q8(tpt_cuda_ctx *ctx, const float *x, int8_t *q, int N, int C, int HW, float scale) {
    k_nchw_to_nhwc_q8<<<grid_1d((size_t)N * C * HW, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream>>>(
        x, q, N, C, HW, scale);
    return after_launch(ctx, "nchw_to_nhwc_q8");
}

int launch_im2col(tpt_cuda_ctx *ctx, const int8_t *x, int8_t *col, int N, int H, int W, int C, int KH, int KW, int sh,
                  int sw, int ph, int pw, int OH, int OW, int Kp) {
    const size_t work = (size_t)N * OH * OW * ((C & 15) == 0 ? Kp / 16 : Kp);
    k_im2col_nhwc<<<grid_1d(work, 256, (unsigned)ctx->sm_count * 16), 256, 0, ctx->stream>>>(x, col, N, H, W, C, KH, KW,
                                                                                           sh, sw, ph, pw, OH, OW, Kp);
    return after_launch(ctx, "im2col");
}

int launch_maxpool_nhwc(tpt_cuda_ctx *ctx, const float *x, float *y, int N, int H, int W, int C, int KH, int KW, int sh,
                        int sw, int ph, int pw, int OH, int OW) {
    k_maxpool_nhwc<<<grid_1d((size_t)N * OH * OW * C, 256, (unsigned)ctx->sm_count * 16), 256, 0, ctx->stream>>>(
        x, y, N, H, W, C, KH, KW, sh, sw, ph, pw, OH, OW);
    return after_launch(ctx, "maxpool");
}

int launch_gap_nhwc(tpt_cuda_ctx *ctx, const float *x, float *y, int N, int HW, int C) {
    k_gap_nhwc<<<grid_1d((size_t)N * C, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream>>>(x, y, N, HW, C);
    return after_launch(ctx, "global_avgpool");
}

namespace {
// [P][T][C] int8 panels (the all-gathered column shards) -> [T][P*C] rows, the
// K-contiguous A operand of the next GEMM; 16 bytes per thread (C % 16 == 0).
__global__ void k_panels_to_rows16(const int4 *__restrict__ in, int4 *__restrict__ out, int P, size_t T, int C16) {
    const size_t total = (size_t)P * T * C16;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % C16);
        const size_t pt = i / C16;
        const size_t t = pt % T;
        const int pp = (int)(pt / T);
        out[(t * P + pp) * C16 + c] = __ldcs(in + i);
    }
}
__global__ void k_panels_to_rows1(const int8_t *__restrict__ in, int8_t *__restrict__ out, int P, size_t T, int C) {
    const size_t total = (size_t)P * T * C;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % C);
        const size_t pt = i / C;
        const size_t t = pt % T;
        const int pp = (int)(pt / T);
        out[(t * P + pp) * C + c] = in[i];
    }
}
}  // namespace

int launch_panels_to_rows(tpt_cuda_ctx *ctx, const int8_t *in, int8_t *out, int P, size_t T, int C) {
    const size_t total = (size_t)P * T * C;
    if (C % 16 == 0 && ((uintptr_t)in & 15) == 0 && ((uintptr_t)out & 15) == 0) {
        k_panels_to_rows16<<<grid_1d(total / 16, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream>>>(
            reinterpret_cast<const int4 *>(in), reinterpret_cast<int4 *>(out), P, T, C / 16);
    } else {
        k_panels_to_rows1<<<grid_1d(total, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream>>>(in, out, P, T, C);
    }
    return after_launch(ctx, "panels_to_rows");
}

int launch_absmax_acc(tpt_cuda_ctx *ctx, const float *x, size_t n, unsigned *cell) {
    k_absmax_acc<<<grid_1d(n, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream>>>(x, n, cell);
    return after_launch(ctx, "absmax");
}

}  // namespace tpt
