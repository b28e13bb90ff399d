// model_ops.cu -- device ops the model plans need besides the GEMMs:
// LayerNorm, bias/residual adds, NHWC INT8 conv plumbing (layout change +
// quantize, im2col), pooling, per-tensor max-abs. The fused attention is in
// attention_i8.cu.
//
// Layout inside a plan: activations are row-major [rows, channels] (NHWC for
// images), so a conv's im2col rows and a GEMM's output rows are both
// [N*H*W, C] and no transposes are needed between layers.
#include <float.h>

#include <type_traits>

#include "common.cuh"

namespace tpt {
namespace {

// ---------------------------------------------------------------- LayerNorm
// ONNX LayerNormalization over the last axis (the reference runtime lacks it:
// crates/tpt-infer-onnx/src/registry.rs:62 maps it to Custom): mean, biased
// variance, y = (x - mean) / sqrt(var + eps) * gamma + beta. One warp per row,
// the row held in registers (cols <= 32 * LN_MAX).
//
// The evaluation order is fixed, every operation explicitly rounded, so a CPU
// restatement reproduces the bits:
//   lane l holds columns c = l + 32 i (k_layernorm) or the float4 groups
//   4 (l + 32 i) .. +3 (k_layernorm4, 768 columns); x = in (+ residual, one add);
//   partial sum: s = s + x_c over its columns in increasing i (in k_layernorm4
//   s = s + (((x0 + x1) + x2) + x3) per group); lanes combined by the xor
//   butterfly s = s + s[l ^ o], o = 16, 8, 4, 2, 1; mean = s / cols;
//   partial variance q = fmaf(d, d, q), d = x - mean, in the same order (a
//   group's four in order), the same butterfly; var = q / cols;
//   inv = 1 / sqrtf(var + eps); y = fmaf((x - mean) * inv, gamma, beta).
// Columns past cols contribute +0 to both sums.
constexpr int LN_MAX = 32;
__device__ __forceinline__ float ln_butterfly(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__global__ void k_layernorm(const float *__restrict__ x, const float *__restrict__ g, const float *__restrict__ b,
                            float *__restrict__ y, int rows, int cols, float eps, int8_t *__restrict__ qout, float qs,
                            const float *__restrict__ res) {
    pdl_wait();
    pdl_trigger();
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
            v[i] = c < cols ? (res ? __fadd_rn(xr[c], res[(size_t)r * cols + c]) : xr[c]) : 0.0f;
            s = __fadd_rn(s, v[i]);
        }
        const float mean = __fdiv_rn(ln_butterfly(s), (float)cols);
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < LN_MAX; i++) {
            const int c = lane + 32 * i;
            const float d = c < cols ? __fsub_rn(v[i], mean) : 0.0f;
            q = __fmaf_rn(d, d, q);
        }
        const float var = __fdiv_rn(ln_butterfly(q), (float)cols);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
        for (int i = 0; i < LN_MAX; i++) {
            const int c = lane + 32 * i;
            if (c < cols) {
                const float o = __fmaf_rn(__fmul_rn(__fsub_rn(v[i], mean), inv), __ldg(g + c), __ldg(b + c));
                y[(size_t)r * cols + c] = o;
                if (qout) qout[(size_t)r * cols + c] = requant_i8(o, qs);  // the next QUANTIZE, fused
            }
        }
    }
}

// Same definition, cols = 128 G (each lane owns float4 groups 4 (lane + 32 i)):
// 16-byte loads and stores and a 4-byte store of the int8 copy.
template <int G>
__global__ void k_layernorm4(const float4 *__restrict__ x, const float4 *__restrict__ g, const float4 *__restrict__ b,
                             float4 *__restrict__ y, int rows, float eps, uint32_t *__restrict__ qout, float qs,
                             const float4 *__restrict__ res) {
    pdl_wait();
    pdl_trigger();
    const int lane = threadIdx.x & 31;
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    constexpr int cols4 = 32 * G;
    const float n = (float)(4 * cols4);
    for (int r = warp; r < rows; r += nwarps) {
        const float4 *xr = x + (size_t)r * cols4;
        float4 v[G];
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < G; i++) {
            v[i] = xr[lane + 32 * i];
            if (res) {  // LayerNorm(x + res): the residual add of the ADD_ACT it replaces, same rounding
                const float4 z = res[(size_t)r * cols4 + lane + 32 * i];
                v[i] = make_float4(__fadd_rn(v[i].x, z.x), __fadd_rn(v[i].y, z.y), __fadd_rn(v[i].z, z.z),
                                   __fadd_rn(v[i].w, z.w));
            }
            s = __fadd_rn(s, __fadd_rn(__fadd_rn(__fadd_rn(v[i].x, v[i].y), v[i].z), v[i].w));
        }
        const float mean = __fdiv_rn(ln_butterfly(s), n);
        float q = 0.0f;
#pragma unroll
        for (int i = 0; i < G; i++) {
            const float dx = __fsub_rn(v[i].x, mean), dy = __fsub_rn(v[i].y, mean), dz = __fsub_rn(v[i].z, mean),
                        dw = __fsub_rn(v[i].w, mean);
            q = __fmaf_rn(dx, dx, q);
            q = __fmaf_rn(dy, dy, q);
            q = __fmaf_rn(dz, dz, q);
            q = __fmaf_rn(dw, dw, q);
        }
        const float var = __fdiv_rn(ln_butterfly(q), n);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
        for (int i = 0; i < G; i++) {
            const int c = lane + 32 * i;
            const float4 gg = __ldg(g + c), bb = __ldg(b + c);
            const float4 o = make_float4(__fmaf_rn(__fmul_rn(__fsub_rn(v[i].x, mean), inv), gg.x, bb.x),
                                         __fmaf_rn(__fmul_rn(__fsub_rn(v[i].y, mean), inv), gg.y, bb.y),
                                         __fmaf_rn(__fmul_rn(__fsub_rn(v[i].z, mean), inv), gg.z, bb.z),
                                         __fmaf_rn(__fmul_rn(__fsub_rn(v[i].w, mean), inv), gg.w, bb.w));
            y[(size_t)r * cols4 + c] = o;
            if (qout)
                qout[(size_t)r * cols4 + c] = (uint32_t)(uint8_t)requant_i8(o.x, qs) |
                                             ((uint32_t)(uint8_t)requant_i8(o.y, qs) << 8) |
                                             ((uint32_t)(uint8_t)requant_i8(o.z, qs) << 16) |
                                             ((uint32_t)(uint8_t)requant_i8(o.w, qs) << 24);
        }
    }
}

// ---------------------------------------------------------------- adds
// y[r, c] = act(x[r, c] + bias[c]) (the runtime's broadcast bias add,
// crates/tpt-infer-runtime/src/kernels.rs:150-178, plus a fused activation)
__global__ void k_bias_act(const float *__restrict__ x, const float *__restrict__ bias, float *__restrict__ y,
                           size_t rows, int cols, int act) {
    pdl_wait();
    pdl_trigger();
    const size_t n = rows * (size_t)cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v = x[i];
        if (bias) v = v + bias[i % cols];
        y[i] = apply_act(v, act);
    }
}

// y = act(a + b) element-wise (residual adds)
// out = act(a + b); with q, also its int8 copy at the next quantization
// point's scale (the following QUANTIZE op, fused)
__global__ void k_add_act(const float4 *__restrict__ a, const float4 *__restrict__ b, float4 *__restrict__ y, size_t n4,
                          int act, uint32_t *__restrict__ q, float qs) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 x = a[i], z = b[i];
        const float4 o = make_float4(apply_act(x.x + z.x, act), apply_act(x.y + z.y, act), apply_act(x.z + z.z, act),
                                     apply_act(x.w + z.w, act));
        y[i] = o;
        if (q)
            q[i] = (uint32_t)(uint8_t)requant_i8(o.x, qs) | ((uint32_t)(uint8_t)requant_i8(o.y, qs) << 8) |
                   ((uint32_t)(uint8_t)requant_i8(o.z, qs) << 16) | ((uint32_t)(uint8_t)requant_i8(o.w, qs) << 24);
    }
}

// ---------------------------------------------------------------- images
// NCHW f32 -> NHWC int8 with a static per-tensor scale:
// q = clamp(round(x / scale), -127, 127) (quant.rs:35-36), Cp >= C channels
// per pixel (channels [C, Cp) are zero). With s2d = 2 the pixels are also
// regrouped space-to-depth: output pixel (y, x) of an [H/2, W/2] grid holds the
// 2x2 input pixels (2y + dy, 2x + dx) as channels ((dy * 2 + dx) * Cp + c). A
// stride-2 convolution then runs as a stride-1 one on 16-byte pixels (a
// 3-channel image padded to 4: the stem's gathers move 16-byte chunks).
__global__ void k_nchw_to_nhwc_q8(const float *__restrict__ x, int8_t *__restrict__ q, int N, int C, int HW, int W,
                                  int Cp, int s2d, float scale) {
    pdl_wait();
    pdl_trigger();
    const size_t total = (size_t)N * Cp * HW;
    const int cpp = Cp * s2d * s2d;  // output channels per pixel
    const int Wo = W / s2d;
    const size_t HWo = (size_t)HW / ((size_t)s2d * s2d);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        // i indexes the output
        const int oc = (int)(i % cpp);
        const size_t p = i / cpp;  // n * HWo + output pixel
        const size_t n = p / HWo, hwo = p - n * HWo;
        const int sub = oc / Cp, c = oc - sub * Cp;
        const int oy = (int)(hwo / Wo), ox = (int)(hwo - (size_t)oy * Wo);
        const size_t hw = (size_t)(oy * s2d + sub / s2d) * W + (ox * s2d + sub % s2d);
        q[i] = c < C ? round_clamp_i8(__fdiv_rn(x[(n * C + c) * HW + hw], scale), -127.0f, 127.0f) : (int8_t)0;
    }
}

// The ResNet stem's form of the same conversion (2x2 space-to-depth, C <= 4
// channels padded to Cp = 4): one thread per output pixel, its 16 bytes as one
// 16-byte store; the 2 x 2 input pixels of each channel are two 8-byte loads
// (x even, W even), consecutive threads reading consecutive pairs.
__global__ void k_nchw_to_nhwc_q8_s2d4(const float *__restrict__ x, uint4 *__restrict__ q, int N, int C, int H, int W,
                                       float scale) {
    pdl_wait();
    pdl_trigger();
    const int Ho = H >> 1, Wo = W >> 1;
    const int total = N * Ho * Wo;
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < total; p += gridDim.x * blockDim.x) {
        const int n = p / (Ho * Wo), r = p - n * (Ho * Wo), oy = r / Wo, ox = r - oy * Wo;
        uint32_t w[4] = {0u, 0u, 0u, 0u};  // word sub = dy * 2 + dx, byte c
#pragma unroll
        for (int c = 0; c < 4; c++) {
            if (c >= C) break;
#pragma unroll
            for (int dy = 0; dy < 2; dy++) {
                const float2 v = __ldg(reinterpret_cast<const float2 *>(
                    x + (((size_t)n * C + c) * H + 2 * oy + dy) * W + 2 * ox));
                const uint32_t b0 = (uint8_t)round_clamp_i8(__fdiv_rn(v.x, scale), -127.0f, 127.0f);
                const uint32_t b1 = (uint8_t)round_clamp_i8(__fdiv_rn(v.y, scale), -127.0f, 127.0f);
                w[2 * dy] |= b0 << (8 * c);
                w[2 * dy + 1] |= b1 << (8 * c);
            }
        }
        q[p] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// im2col of an NHWC int8 tensor: row m = (n, oy, ox), column (ky, kx, c),
// zero for padded taps and for columns in [K, Kp). One warp per output row:
// the row's pixel is decoded once (32-bit index math), lanes walk the row's
// 16-byte (C % 16 == 0), 4-byte (C % 4 == 0) or 1-byte chunks, so loads of a
// tap are contiguous channels and the row is written with coalesced stores.
template <int VB>
__global__ void __launch_bounds__(256) k_im2col_nhwc(const int8_t *__restrict__ x, int8_t *__restrict__ col, int N,
                                                     int H, int W, int C, int KH, int KW, int sh, int sw, int ph,
                                                     int pw, int OH, int OW, int Kp) {
    pdl_wait();
    pdl_trigger();
    using V = typename std::conditional<VB == 16, int4, typename std::conditional<VB == 4, int, int8_t>::type>::type;
    const int lane = threadIdx.x & 31;
    const int rows = N * OH * OW, K = KH * KW * C, chunks = Kp / VB;
    const int warp = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
    const int nwarps = (int)((gridDim.x * (size_t)blockDim.x) >> 5);
    for (int m = warp; m < rows; m += nwarps) {
        const int ox = m % OW, t = m / OW, oy = t % OH, n = t / OH;
        const int iy0 = oy * sh - ph, ix0 = ox * sw - pw;
        const int8_t *img = x + (size_t)n * H * W * C;
        V *dst = reinterpret_cast<V *>(col + (size_t)m * Kp);
        for (int ch = lane; ch < chunks; ch += 32) {
            const int kk = ch * VB;
            V v{};
            if (kk < K) {
                const int tap = kk / C, c = kk - tap * C;
                const int ky = tap / KW, kx = tap - ky * KW;
                const int iy = iy0 + ky, ix = ix0 + kx;
                if (iy >= 0 && iy < H && ix >= 0 && ix < W)
                    v = *reinterpret_cast<const V *>(img + ((size_t)iy * W + ix) * C + c);
            }
            dst[ch] = v;
        }
    }
}

// im2col for small, unaligned C (the 3-channel stem): lanes gather whole taps
// (C bytes each) into a shared-memory copy of the row, which the warp then
// writes with 16-byte stores. Kp <= IM2COL_ROW_MAX, Kp % 16 == 0.
constexpr int IM2COL_ROW_MAX = 1024;
__global__ void __launch_bounds__(256) k_im2col_nhwc_taps(const int8_t *__restrict__ x, int8_t *__restrict__ col,
                                                          int N, int H, int W, int C, int KH, int KW, int sh, int sw,
                                                          int ph, int pw, int OH, int OW, int Kp) {
    pdl_wait();
    pdl_trigger();
    __shared__ __align__(16) int8_t rowbuf[8][IM2COL_ROW_MAX];
    const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
    int8_t *rb = rowbuf[wib];
    const int rows = N * OH * OW, taps = KH * KW, K = taps * C;
    const int warp = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
    const int nwarps = (int)((gridDim.x * (size_t)blockDim.x) >> 5);
    for (int kk = K + lane; kk < Kp; kk += 32) rb[kk] = 0;
    for (int m = warp; m < rows; m += nwarps) {
        const int ox = m % OW, t = m / OW, oy = t % OH, n = t / OH;
        const int iy0 = oy * sh - ph, ix0 = ox * sw - pw;
        const int8_t *img = x + (size_t)n * H * W * C;
        for (int tap = lane; tap < taps; tap += 32) {
            const int ky = tap / KW, kx = tap - ky * KW;
            const int iy = iy0 + ky, ix = ix0 + kx;
            const bool in = iy >= 0 && iy < H && ix >= 0 && ix < W;
            const int8_t *src = img + ((size_t)iy * W + ix) * C;
            for (int c = 0; c < C; c++) rb[tap * C + c] = in ? src[c] : (int8_t)0;
        }
        __syncwarp();
        int4 *dst = reinterpret_cast<int4 *>(col + (size_t)m * Kp);
        for (int ch = lane; ch < Kp / 16; ch += 32) dst[ch] = reinterpret_cast<const int4 *>(rb)[ch];
        __syncwarp();
    }
}

// max pool on NHWC f32, padding as -inf (kernels.rs:271-325)
__global__ void k_maxpool_nhwc(const float *__restrict__ x, float *__restrict__ y, int N, int H, int W, int C, int KH,
                               int KW, int sh, int sw, int ph, int pw, int OH, int OW) {
    pdl_wait();
    pdl_trigger();
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

// Same, 4 channels per thread (C % 4 == 0, 16-byte aligned), 32-bit index math.
// KT > 0: a KT x KT window known at compile time, so its loads are issued
// together; taps outside the input are skipped as in the generic loop, and
// the taps are compared in the same order (row by row), so ties between
// signed zeros and NaN inputs resolve the same way.
// q != nullptr: also the int8 copy of the output, clamp(roundf(y / qs)) (the
// QUANTIZE op's rule), 4 bytes per thread.
template <int KT>
__global__ void k_maxpool_nhwc4(const float4 *__restrict__ x, float4 *__restrict__ y, int N, int H, int W, int C4,
                                int KH, int KW, int sh, int sw, int ph, int pw, int OH, int OW,
                                uint32_t *__restrict__ q, float qs) {
    pdl_wait();
    pdl_trigger();
    if (KT > 0) KH = KW = KT;
    const int total = N * OH * OW * C4;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int c = i % C4, t = i / C4, ox = t % OW, t2 = t / OW, oy = t2 % OH, n = t2 / OH;
        float4 best = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
#pragma unroll
        for (int ky = 0; ky < (KT > 0 ? KT : KH); ky++) {
            const int iy = oy * sh + ky - ph;
#pragma unroll
            for (int kx = 0; kx < (KT > 0 ? KT : KW); kx++) {
                const int ix = ox * sw + kx - pw;
                if (iy < 0 || iy >= H || ix < 0 || ix >= W) continue;
                const float4 v = __ldg(x + ((n * H + iy) * W + ix) * C4 + c);
                if (v.x > best.x) best.x = v.x;
                if (v.y > best.y) best.y = v.y;
                if (v.z > best.z) best.z = v.z;
                if (v.w > best.w) best.w = v.w;
            }
        }
        y[i] = best;
        if (q) {
            const bool fast = requant_fast_ok(qs);
            const float rs = __frcp_rn(qs);
            auto rq = [&](float v) { return (uint32_t)(uint8_t)(fast ? requant_i8_fast(v, qs, rs) : requant_i8(v, qs)); };
            q[i] = rq(best.x) | (rq(best.y) << 8) | (rq(best.z) << 16) | (rq(best.w) << 24);
        }
    }
}

// global average pool NHWC f32 [N, HW, C] -> [N, C]: sequential sum over the
// window, then divide by the count (kernels.rs:335-390 with kernel = spatial)
__global__ void k_gap_nhwc(const float *__restrict__ x, float *__restrict__ y, int N, int HW, int C) {
    pdl_wait();
    pdl_trigger();
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
    pdl_wait();
    pdl_trigger();
    float m = 0.0f;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(x[i]));
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) atomicMax(cell, __float_as_uint(m));
}

}  // namespace

int launch_layernorm(tpt_cuda_ctx *ctx, const float *x, const float *g, const float *b, float *y, size_t rows,
                     size_t cols, float eps, int8_t *q, float qs, const float *res) {
    if (cols > 32 * LN_MAX || rows > INT32_MAX) return TPT_UNSUPPORTED;
    const unsigned grid = grid_1d(rows * 32, 256, (unsigned)ctx->sm_count * 16);
    const bool a16 = ((((uintptr_t)x | (uintptr_t)g | (uintptr_t)b | (uintptr_t)y | (uintptr_t)res) & 15) == 0) &&
                     ((uintptr_t)q & 3) == 0;
    if (a16 && cols == 768) {  // the BERT hidden size
        launch_pdl(k_layernorm4<6>, grid, 256, 0, ctx->stream, (const float4 *)x, (const float4 *)g, (const float4 *)b,
                                                       (float4 *)y, (int)rows, eps, (uint32_t *)q, qs,
                   (const float4 *)res);
        return after_launch(ctx, "layernorm");
    }
    launch_pdl(k_layernorm, grid, 256, 0, ctx->stream, x, g, b, y, (int)rows, (int)cols, eps, q, qs, res);
    return after_launch(ctx, "layernorm");
}

int launch_attention_i8(tpt_cuda_ctx *ctx, const float *qkv, float *out, int B, int S, int H, int D, float scale,
                        int8_t *q, float qs);

int launch_attention(tpt_cuda_ctx *ctx, const float *qkv, float *out, int B, int S, int H, int D, float scale,
                     int8_t *q, float qs) {
    return launch_attention_i8(ctx, qkv, out, B, S, H, D, scale, q, qs);
}

int launch_bias_act(tpt_cuda_ctx *ctx, const float *x, const float *bias, float *y, size_t rows, size_t cols, int act) {
    launch_pdl(k_bias_act, grid_1d(rows * cols, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream, x, bias, y, rows,
                                                                                              (int)cols, act);
    return after_launch(ctx, "bias_act");
}

int launch_add_act(tpt_cuda_ctx *ctx, const float *a, const float *b, float *y, size_t n, int act, int8_t *q,
                   float qs) {
    if (n % 4 || ((uintptr_t)q & 3)) return TPT_UNSUPPORTED;
    launch_pdl(k_add_act, grid_1d(n / 4, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream, (const float4 *)a, (const float4 *)b, (float4 *)y, n / 4, act, reinterpret_cast<uint32_t *>(q), qs);
    return after_launch(ctx, "add_act");
}

int launch_nchw_to_nhwc_q8(tpt_cuda_ctx *ctx, const float *x, int8_t *q, int N, int C, int HW, int W, int Cp, int s2d,
                           float scale) {
    if (s2d < 1) s2d = 1;
    if (W <= 0) W = HW;  // no width given: only s2d = 1 is possible
    if (s2d > 2 || HW % W || (W % s2d) || ((HW / W) % s2d)) return TPT_UNSUPPORTED;
    if (s2d == 2 && Cp == 4 && C <= 4 && ((uintptr_t)x & 7) == 0 && ((uintptr_t)q & 15) == 0 &&
        (size_t)N * HW / 4 < 0x7fffffff) {
        launch_pdl(k_nchw_to_nhwc_q8_s2d4, grid_1d((size_t)N * HW / 4, 256, (unsigned)ctx->sm_count * 8), 256, 0,
                   ctx->stream, x, reinterpret_cast<uint4 *>(q), N, C, HW / W, W, scale);
        return after_launch(ctx, "nchw_to_nhwc_q8");
    }
    launch_pdl(k_nchw_to_nhwc_q8, grid_1d((size_t)N * Cp * HW, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream,
               x, q, N, C, HW, W, Cp, s2d, scale);
    return after_launch(ctx, "nchw_to_nhwc_q8");
}

int launch_im2col(tpt_cuda_ctx *ctx, const int8_t *x, int8_t *col, int N, int H, int W, int C, int KH, int KW, int sh,
                  int sw, int ph, int pw, int OH, int OW, int Kp) {
    const size_t rows = (size_t)N * OH * OW;
    if (rows > 0x7fffffff || (size_t)H * W * C > 0x7fffffff) return TPT_UNSUPPORTED;
    const unsigned g = grid_1d(rows * 32, 256, (unsigned)ctx->sm_count * 16);
    const bool a16 = ((uintptr_t)x & 15) == 0 && ((uintptr_t)col & 15) == 0;
    if ((C & 15) == 0 && (Kp & 15) == 0 && a16)
        launch_pdl(k_im2col_nhwc<16>, g, 256, 0, ctx->stream, x, col, N, H, W, C, KH, KW, sh, sw, ph, pw, OH, OW, Kp);
    else if ((C & 3) == 0 && (Kp & 3) == 0 && a16)
        launch_pdl(k_im2col_nhwc<4>, g, 256, 0, ctx->stream, x, col, N, H, W, C, KH, KW, sh, sw, ph, pw, OH, OW, Kp);
    else if ((Kp & 15) == 0 && Kp <= IM2COL_ROW_MAX && ((uintptr_t)col & 15) == 0)
        launch_pdl(k_im2col_nhwc_taps, g, 256, 0, ctx->stream, x, col, N, H, W, C, KH, KW, sh, sw, ph, pw, OH, OW, Kp);
    else
        launch_pdl(k_im2col_nhwc<1>, g, 256, 0, ctx->stream, x, col, N, H, W, C, KH, KW, sh, sw, ph, pw, OH, OW, Kp);
    return after_launch(ctx, "im2col");
}

int launch_maxpool_nhwc(tpt_cuda_ctx *ctx, const float *x, float *y, int N, int H, int W, int C, int KH, int KW, int sh,
                        int sw, int ph, int pw, int OH, int OW, int8_t *q, float qs) {
    const size_t total = (size_t)N * OH * OW * C;
    if (C % 4 == 0 && total / 4 < 0x7fffffff && (size_t)N * H * W * C / 4 < 0x7fffffff && ((uintptr_t)x & 15) == 0 &&
        ((uintptr_t)y & 15) == 0 && ((uintptr_t)q & 3) == 0) {
        auto kfn = KH == 3 && KW == 3 ? k_maxpool_nhwc4<3> : k_maxpool_nhwc4<0>;
        launch_pdl(kfn, grid_1d(total / 4, 256, (unsigned)ctx->sm_count * 16), 256, 0, ctx->stream,
                   reinterpret_cast<const float4 *>(x), reinterpret_cast<float4 *>(y), N, H, W, C / 4, KH, KW, sh, sw,
                   ph, pw, OH, OW, reinterpret_cast<uint32_t *>(q), qs);
        return after_launch(ctx, "maxpool");
    }
    if (q) return TPT_UNSUPPORTED;  // the int8 copy needs the 4-channel kernel
    launch_pdl(k_maxpool_nhwc, grid_1d(total, 256, (unsigned)ctx->sm_count * 16), 256, 0, ctx->stream, x, y, N, H, W, C, KH, KW, sh, sw, ph, pw, OH, OW);
    return after_launch(ctx, "maxpool");
}

int launch_gap_nhwc(tpt_cuda_ctx *ctx, const float *x, float *y, int N, int HW, int C) {
    launch_pdl(k_gap_nhwc, grid_1d((size_t)N * C, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream, x, y, N, HW, C);
    return after_launch(ctx, "global_avgpool");
}

namespace {
// [P][T][C] int8 panels (the all-gathered column shards) -> [T][P*C] rows, the
// K-contiguous A operand of the next GEMM; 16 bytes per thread (C % 16 == 0).
__global__ void k_panels_to_rows16(const int4 *__restrict__ in, int4 *__restrict__ out, int P, size_t T, int C16) {
    pdl_wait();
    pdl_trigger();
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
    pdl_wait();
    pdl_trigger();
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
        launch_pdl(k_panels_to_rows16, grid_1d(total / 16, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream, reinterpret_cast<const int4 *>(in), reinterpret_cast<int4 *>(out), P, T, C / 16);
    } else {
        launch_pdl(k_panels_to_rows1, grid_1d(total, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream, in, out, P, T, C);
    }
    return after_launch(ctx, "panels_to_rows");
}

int launch_absmax_acc(tpt_cuda_ctx *ctx, const float *x, size_t n, unsigned *cell) {
    launch_pdl(k_absmax_acc, grid_1d(n, 256, (unsigned)ctx->sm_count * 8), 256, 0, ctx->stream, x, n, cell);
    return after_launch(ctx, "absmax");
}

}  // namespace tpt
