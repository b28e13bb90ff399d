// quant.cu -- device quantizers and (un)packers of tpt-infer-quantize
// (crates/tpt-infer-quantize/src/quant.rs, dequant.rs). All results are
// bit-exact with the reference: max-abs reductions are order-independent,
// x / scale is an IEEE divide (no fast-math anywhere in this library), rounding
// is roundf (half away from zero, Rust's f32::round) and the saturating cast
// maps NaN to 0.
//
// Per-tensor quantizers reduce through one 32-bit cell in device scratch:
// non-negative floats order like their bit patterns, so atomicMax on the bits
// of max|x| (NaN already dropped by fmaxf) is an exact global max.
#include <float.h>

#include "common.cuh"

namespace tpt {
namespace {

// float <-> order-preserving unsigned (for signed min/max through atomics)
__device__ __forceinline__ unsigned f2ord(float f) {
    unsigned u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord2f(unsigned u) {
    return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

template <typename Op>
__device__ __forceinline__ float block_reduce(float v, Op op, float identity) {
    __shared__ float red[32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) red[wid] = v;
    __syncthreads();
    v = lane < nw ? red[lane] : identity;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;  // valid in every thread
}

struct FMax {
    __device__ float operator()(float a, float b) const { return fmaxf(a, b); }
};
struct FMin {
    __device__ float operator()(float a, float b) const { return fminf(a, b); }
};

// max|x| over the whole tensor into *cell (bits of a non-negative float).
__global__ void k_absmax(const float *__restrict__ x, size_t n, unsigned *cell) {
    float m = 0.0f;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(__ldg(x + i)));
    m = block_reduce(m, FMax(), 0.0f);
    if (threadIdx.x == 0) atomicMax(cell, __float_as_uint(m));
}

// quant.rs:27-31: scale = max_abs == 0 ? 1 : max_abs / DIV
__device__ __forceinline__ float sym_scale(unsigned cell, float div) {
    float ma = __uint_as_float(cell);
    return ma == 0.0f ? 1.0f : __fdiv_rn(ma, div);
}

__global__ void k_quant_i8_from_cell(const float *__restrict__ x, size_t n, const unsigned *cell,
                                     int8_t *__restrict__ q, float *scale_out) {
    const float scale = sym_scale(*cell, 127.0f);
    if (blockIdx.x == 0 && threadIdx.x == 0 && scale_out) *scale_out = scale;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        q[i] = round_clamp_i8(__fdiv_rn(x[i], scale), -127.0f, 127.0f);
}

__global__ void k_quant_i8_static(const float *__restrict__ x, size_t n, float scale, int8_t *__restrict__ q) {
    pdl_wait();
    pdl_trigger();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        q[i] = round_clamp_i8(__fdiv_rn(x[i], scale), -127.0f, 127.0f);
}

// Same, 16 elements per thread: four 16-byte loads, one 16-byte store
// (x and q 16-byte aligned, n % 16 == 0).
__global__ void k_quant_i8_static16(const float4 *__restrict__ x, size_t n16, float scale, int4 *__restrict__ q) {
    pdl_wait();
    pdl_trigger();
    const float rs = __frcp_rn(scale);
    const bool fast = requant_fast_ok(scale);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float4 v = __ldcs(x + 4 * i + j);
            const uint32_t b0 = (uint8_t)(fast ? requant_i8_fast(v.x, scale, rs) : requant_i8(v.x, scale));
            const uint32_t b1 = (uint8_t)(fast ? requant_i8_fast(v.y, scale, rs) : requant_i8(v.y, scale));
            const uint32_t b2 = (uint8_t)(fast ? requant_i8_fast(v.z, scale, rs) : requant_i8(v.z, scale));
            const uint32_t b3 = (uint8_t)(fast ? requant_i8_fast(v.w, scale, rs) : requant_i8(v.w, scale));
            w[j] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
        q[i] = make_int4((int)w[0], (int)w[1], (int)w[2], (int)w[3]);
    }
}

// quant.rs:95-107: one CTA per row of [rows, cols]
__global__ void k_quant_i8_rows(const float *__restrict__ x, size_t rows, size_t cols, int8_t *__restrict__ q,
                                float *__restrict__ scales) {
    pdl_wait();
    pdl_trigger();
    for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float *xr = x + r * cols;
        float m = 0.0f;
        for (size_t j = threadIdx.x; j < cols; j += blockDim.x) m = fmaxf(m, fabsf(xr[j]));
        m = block_reduce(m, FMax(), 0.0f);
        const float scale = m == 0.0f ? 1.0f : __fdiv_rn(m, 127.0f);
        if (threadIdx.x == 0) scales[r] = scale;
        for (size_t j = threadIdx.x; j < cols; j += blockDim.x)
            q[r * cols + j] = round_clamp_i8(__fdiv_rn(xr[j], scale), -127.0f, 127.0f);
        __syncthreads();
    }
}

// quant.rs:45-90, phase 0: cells = (ord(+inf), ord(-inf)) for min/max
__global__ void k_minmax_init(unsigned *cells) {
    cells[0] = f2ord(INFINITY);
    cells[1] = f2ord(-INFINITY);
}

// quant.rs:45-90, phase 1: min and max (NaN dropped like f32::min/max).
__global__ void k_minmax(const float *__restrict__ x, size_t n, unsigned *cells) {
    float mn = INFINITY, mx = -INFINITY;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        float v = __ldg(x + i);
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
    }
    mn = block_reduce(mn, FMin(), INFINITY);
    mx = block_reduce(mx, FMax(), -INFINITY);
    if (threadIdx.x == 0) {
        atomicMin(cells + 0, f2ord(mn));
        atomicMax(cells + 1, f2ord(mx));
    }
}

// quant.rs:45-90, phase 2: the scale/zero-point rule, one thread.
__global__ void k_asym_params(const unsigned *cells, float *scale_out, int32_t *zp_out) {
    const float QMIN = -128.0f, QMAX = 127.0f;
    float mn = ord2f(cells[0]), mx = ord2f(cells[1]);
    if (mn > mx || !isfinite(mn) || !isfinite(mx)) {
        mn = 0.0f;
        mx = 0.0f;
    }
    float scale;
    int32_t zp;
    if (fabsf(__fsub_rn(mx, mn)) < FLT_EPSILON) {
        scale = 1.0f;
        zp = 0;
    } else {
        float scale0 = __fdiv_rn(__fsub_rn(mx, mn), __fsub_rn(QMAX, QMIN));
        float zp0 = roundf(__fsub_rn(QMIN, __fdiv_rn(mn, scale0)));
        if (zp0 < QMIN) {
            float s = __fdiv_rn(mx, __fsub_rn(QMAX, QMIN));
            scale = s <= 0.0f ? scale0 : s;
            zp = (int32_t)QMIN;
        } else if (zp0 > QMAX) {
            float s = __fdiv_rn(mn, __fsub_rn(QMIN, QMAX));
            scale = s <= 0.0f ? scale0 : fabsf(s);
            zp = (int32_t)QMAX;
        } else {
            scale = scale0;
            zp = (int32_t)zp0;
        }
    }
    *scale_out = scale;
    *zp_out = zp;
}

__global__ void k_quant_i8_asym(const float *__restrict__ x, size_t n, const float *scale_p, const int32_t *zp_p,
                                int8_t *__restrict__ q) {
    const float scale = *scale_p, zp = (float)*zp_p;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        q[i] = round_clamp_i8(__fadd_rn(__fdiv_rn(x[i], scale), zp), -128.0f, 127.0f);
}

// quant.rs:123-140: byte = (hi & 0xF) << 4 | (lo & 0xF); odd tail hi = 0.
__global__ void k_pack_i4(const int8_t *__restrict__ v, size_t n, uint8_t *__restrict__ out, unsigned *bad) {
    const size_t nb = (n + 1) / 2;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < nb; i += (size_t)gridDim.x * blockDim.x) {
        int lo = v[2 * i];
        int hi = 2 * i + 1 < n ? v[2 * i + 1] : 0;
        if (lo < -8 || lo > 7 || hi < -8 || hi > 7) atomicOr(bad, 1u);
        out[i] = (uint8_t)(((hi & 0x0f) << 4) | (lo & 0x0f));
    }
}

__device__ __forceinline__ int8_t sext4(unsigned nib) { return (int8_t)((int)(nib << 28) >> 28); }

// quant.rs:143-157 (count = number of values to produce)
__global__ void k_unpack_i4(const uint8_t *__restrict__ p, size_t count, int8_t *__restrict__ out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < count; i += (size_t)gridDim.x * blockDim.x) {
        unsigned b = p[i >> 1];
        out[i] = sext4((i & 1) ? (b >> 4) : (b & 0x0f));
    }
}

// quant.rs:171-186 / :192-204: one CTA per row; q in [-7, 7], packed.
__global__ void k_quant_i4_rows(const float *__restrict__ x, size_t rows, size_t cols, uint8_t *__restrict__ p,
                                float *__restrict__ scales) {
    const size_t rb = (cols + 1) / 2;
    for (size_t r = blockIdx.x; r < rows; r += gridDim.x) {
        const float *xr = x + r * cols;
        float m = 0.0f;
        for (size_t j = threadIdx.x; j < cols; j += blockDim.x) m = fmaxf(m, fabsf(xr[j]));
        m = block_reduce(m, FMax(), 0.0f);
        const float scale = m == 0.0f ? 1.0f : __fdiv_rn(m, 7.0f);
        if (threadIdx.x == 0) scales[r] = scale;
        for (size_t j = threadIdx.x; j < rb; j += blockDim.x) {
            int lo = round_clamp_i8(__fdiv_rn(xr[2 * j], scale), -7.0f, 7.0f);
            int hi = 2 * j + 1 < cols ? round_clamp_i8(__fdiv_rn(xr[2 * j + 1], scale), -7.0f, 7.0f) : 0;
            p[r * rb + j] = (uint8_t)(((hi & 0x0f) << 4) | (lo & 0x0f));
        }
        __syncthreads();
    }
}

// Per-tensor INT4 from a max-abs cell.
__global__ void k_quant_i4_from_cell(const float *__restrict__ x, size_t n, const unsigned *cell,
                                     uint8_t *__restrict__ p, float *scale_out) {
    const float scale = sym_scale(*cell, 7.0f);
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = scale;
    const size_t nb = (n + 1) / 2;
    for (size_t j = blockIdx.x * (size_t)blockDim.x + threadIdx.x; j < nb; j += (size_t)gridDim.x * blockDim.x) {
        int lo = round_clamp_i8(__fdiv_rn(x[2 * j], scale), -7.0f, 7.0f);
        int hi = 2 * j + 1 < n ? round_clamp_i8(__fdiv_rn(x[2 * j + 1], scale), -7.0f, 7.0f) : 0;
        p[j] = (uint8_t)(((hi & 0x0f) << 4) | (lo & 0x0f));
    }
}

// dequant.rs:13-15 / :26-37: out = q * scale[row]
__global__ void k_dequant_i8_rows(const int8_t *__restrict__ q, size_t rows, size_t cols,
                                  const float *__restrict__ scales, float *__restrict__ out) {
    const size_t n = rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __fmul_rn((float)q[i], scales[i / cols]);
}

// dequant.rs:18-22: out = (q as f32 - zero_point as f32) * scale (both
// conversions exact, the difference of two small integers exact, one rounding)
__global__ void k_dequant_i8_asym(const int8_t *__restrict__ q, size_t n, float scale, int32_t zp,
                                  float *__restrict__ out) {
    const float z = (float)zp;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __fmul_rn(__fsub_rn((float)q[i], z), scale);
}

// dequant.rs:56-71: rows of ceil(row_elems/2) bytes; values past packed_len absent
__global__ void k_dequant_i4_rows(const uint8_t *__restrict__ p, size_t rows, size_t row_elems, size_t packed_len,
                                  const float *__restrict__ scales, float *__restrict__ out) {
    const size_t n = rows * row_elems, rb = (row_elems + 1) / 2;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        size_t r = i / row_elems, c = i - r * row_elems;
        size_t byte = r * rb + c / 2;
        if (byte >= packed_len) continue;
        unsigned b = p[byte];
        out[i] = __fmul_rn((float)sext4((c & 1) ? (b >> 4) : (b & 0x0f)), scales[r]);
    }
}

}  // namespace

static unsigned cap_grid(tpt_cuda_ctx *ctx) { return (unsigned)ctx->sm_count * 8; }

int launch_quant_i8_sym(tpt_cuda_ctx *ctx, const float *x, size_t n, int8_t *q, float *scale_dev,
                        unsigned *cell) {
    cudaError_t e = cudaMemsetAsync(cell, 0, sizeof(unsigned), ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "absmax cell clear");
    unsigned g = grid_1d(n, 256, cap_grid(ctx));
    k_absmax<<<g, 256, 0, ctx->stream>>>(x, n, cell);
    k_quant_i8_from_cell<<<g, 256, 0, ctx->stream>>>(x, n, cell, q, scale_dev);
    return after_launch(ctx, "quantize_i8_symmetric", 2);
}

int launch_quant_i8_static(tpt_cuda_ctx *ctx, const float *x, size_t n, float scale, int8_t *q) {
    if (n % 16 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)q & 15) == 0) {
        launch_pdl(k_quant_i8_static16, grid_1d(n / 16, 256, cap_grid(ctx)), 256, 0, ctx->stream, reinterpret_cast<const float4 *>(x), n / 16, scale, reinterpret_cast<int4 *>(q));
        return after_launch(ctx, "quantize_i8_static");
    }
    launch_pdl(k_quant_i8_static, grid_1d(n, 256, cap_grid(ctx)), 256, 0, ctx->stream, x, n, scale, q);
    return after_launch(ctx, "quantize_i8_static");
}

int launch_quant_i8_rows(tpt_cuda_ctx *ctx, const float *x, size_t rows, size_t cols, int8_t *q, float *scales) {
    unsigned g = (unsigned)(rows < (size_t)ctx->sm_count * 16 ? rows : (size_t)ctx->sm_count * 16);
    launch_pdl(k_quant_i8_rows, g ? g : 1, 256, 0, ctx->stream, x, rows, cols, q, scales);
    return after_launch(ctx, "quantize_i8_per_channel");
}

int launch_quant_i8_asym(tpt_cuda_ctx *ctx, const float *x, size_t n, int8_t *q, float *scale_dev,
                         int32_t *zp_dev, unsigned *cells) {
    unsigned g = grid_1d(n, 256, cap_grid(ctx));
    k_minmax_init<<<1, 1, 0, ctx->stream>>>(cells);
    k_minmax<<<g, 256, 0, ctx->stream>>>(x, n, cells);
    k_asym_params<<<1, 1, 0, ctx->stream>>>(cells, scale_dev, zp_dev);
    k_quant_i8_asym<<<g, 256, 0, ctx->stream>>>(x, n, scale_dev, zp_dev, q);
    return after_launch(ctx, "quantize_i8_asymmetric", 4);
}

int launch_pack_i4(tpt_cuda_ctx *ctx, const int8_t *v, size_t n, uint8_t *out, unsigned *bad) {
    cudaError_t e = cudaMemsetAsync(bad, 0, sizeof(unsigned), ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "pack flag clear");
    k_pack_i4<<<grid_1d((n + 1) / 2, 256, cap_grid(ctx)), 256, 0, ctx->stream>>>(v, n, out, bad);
    return after_launch(ctx, "pack_i4");
}

int launch_unpack_i4(tpt_cuda_ctx *ctx, const uint8_t *p, size_t count, int8_t *out) {
    k_unpack_i4<<<grid_1d(count, 256, cap_grid(ctx)), 256, 0, ctx->stream>>>(p, count, out);
    return after_launch(ctx, "unpack_i4");
}

int launch_quant_i4_rows(tpt_cuda_ctx *ctx, const float *x, size_t rows, size_t cols, uint8_t *p, float *scales) {
    if (rows == 1) {
        unsigned *cell = ctx->d_reduce;
        cudaError_t e = cudaMemsetAsync(cell, 0, sizeof(unsigned), ctx->stream);
        if (e != cudaSuccess) return cuda_fail(ctx, e, "absmax cell clear");
        unsigned g = grid_1d(cols, 256, cap_grid(ctx));
        k_absmax<<<g, 256, 0, ctx->stream>>>(x, cols, cell);
        k_quant_i4_from_cell<<<g, 256, 0, ctx->stream>>>(x, cols, cell, p, scales);
        return after_launch(ctx, "quantize_i4_symmetric", 2);
    }
    unsigned g = (unsigned)(rows < (size_t)ctx->sm_count * 16 ? rows : (size_t)ctx->sm_count * 16);
    k_quant_i4_rows<<<g, 256, 0, ctx->stream>>>(x, rows, cols, p, scales);
    return after_launch(ctx, "quantize_i4_per_channel");
}

int launch_dequant_i8_rows(tpt_cuda_ctx *ctx, const int8_t *q, size_t rows, size_t cols, const float *scales,
                           float *out) {
    k_dequant_i8_rows<<<grid_1d(rows * cols, 256, cap_grid(ctx)), 256, 0, ctx->stream>>>(q, rows, cols, scales, out);
    return after_launch(ctx, "dequantize_i8");
}

int launch_dequant_i8_asym(tpt_cuda_ctx *ctx, const int8_t *q, size_t n, float scale, int32_t zp, float *out) {
    k_dequant_i8_asym<<<grid_1d(n, 256, cap_grid(ctx)), 256, 0, ctx->stream>>>(q, n, scale, zp, out);
    return after_launch(ctx, "dequantize_i8_asymmetric");
}

int launch_dequant_i4_rows(tpt_cuda_ctx *ctx, const uint8_t *p, size_t rows, size_t row_elems, size_t packed_len,
                           const float *scales, float *out) {
    k_dequant_i4_rows<<<grid_1d(rows * row_elems, 256, cap_grid(ctx)), 256, 0, ctx->stream>>>(
        p, rows, row_elems, packed_len, scales, out);
    return after_launch(ctx, "dequantize_i4");
}

}  // namespace tpt
