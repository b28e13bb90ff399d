// noalloc.cu -- per-tensor symmetric INT8 quantization for callers that must
// not allocate device memory.
//
// tpt_cuda_quantize_i8_symmetric_noalloc produces exactly what
// tpt_cuda_quantize_i8_symmetric_dev produces (the quantize_i8_symmetric rule:
// scale = max|x| / 127, or 1.0 for an all-zero tensor; q = round-half-away(x /
// scale) clamped to [-127, 127]) without a context and without any
// allocation. Some callers cannot allocate at all: code that runs inside
// another runtime's memory budget (a host engine whose allocator owns every
// byte of the GPU), code that runs on a real-time or latency-critical path
// where cudaMalloc's implicit device synchronisation is not acceptable, and
// code that must not fail midway for lack of memory once it has started. For
// them the reduction scratch lives here, in a fixed array that is part of the
// library's device image.
//
// The scratch: g_na_partials, TPT_NOALLOC_PARTIALS 32-bit words (128 KiB),
// aligned to 256 bytes. Every GPU that loads this library holds one copy of it
// until the process exits. Pass 1 writes one partial max|x| per tile of
// NA_TILE elements, pass 2 (one CTA) reduces the partials and writes the
// scale to the caller's output, pass 3 quantizes. A call reads only the
// partials it wrote itself earlier in the same stream order, so nothing in
// the scratch has to start at zero and the last call's leftovers are never
// read. The array is shared by every call on a device: two calls whose
// kernels overlap on the GPU (different streams, no ordering between them)
// race on it and may both produce wrong scales.
#include <mutex>

#include "common.cuh"

namespace tpt {
namespace {

constexpr unsigned NA_TILE = 8192;  // elements reduced by one CTA in pass 1
constexpr unsigned NA_MAX_DEVICES = 64;
static_assert((unsigned long long)NA_TILE * TPT_NOALLOC_PARTIALS == TPT_NOALLOC_QUANT_MAX_ELEMS,
              "maximum size = tile x partials");

// The only scratch the entry point uses. Host code must not pass this name to a
// kernel: on the host it is a stand-in symbol, not a device address. The
// device address comes from cudaGetSymbolAddress (na_scratch below).
static __device__ __align__(256) unsigned g_na_partials[TPT_NOALLOC_PARTIALS];

__device__ __forceinline__ float na_block_max(float v) {
    __shared__ float red[32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[wid] = v;
    __syncthreads();
    v = lane < nw ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Pass 1: partials[b] = max|x| over tile b (NaN ignored, like f32::max).
__global__ void k_na_absmax(const float *__restrict__ x, size_t n, unsigned *__restrict__ partials) {
    const size_t base = (size_t)blockIdx.x * NA_TILE;
    const size_t end = base + NA_TILE < n ? base + NA_TILE : n;
    float m = 0.0f;
    for (size_t i = base + threadIdx.x; i < end; i += blockDim.x) m = fmaxf(m, fabsf(__ldg(x + i)));
    m = na_block_max(m);
    if (threadIdx.x == 0) partials[blockIdx.x] = __float_as_uint(m);
}

// Pass 2 (one CTA): scale = max == 0 ? 1 : max / 127 (quant.rs:27-31).
__global__ void k_na_scale(const unsigned *__restrict__ partials, unsigned count, float *scale_out) {
    float m = 0.0f;
    for (unsigned i = threadIdx.x; i < count; i += blockDim.x) m = fmaxf(m, __uint_as_float(partials[i]));
    m = na_block_max(m);
    if (threadIdx.x == 0) *scale_out = m == 0.0f ? 1.0f : __fdiv_rn(m, 127.0f);
}

// Pass 3: q = clamp(round(x / scale), -127, 127) (quant.rs:32-38).
__global__ void k_na_quant(const float *__restrict__ x, size_t n, const float *scale_p, int8_t *__restrict__ q) {
    const float scale = *scale_p;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        q[i] = round_clamp_i8(__fdiv_rn(x[i], scale), -127.0f, 127.0f);
}

std::mutex g_na_mutex;
unsigned *g_na_addr[NA_MAX_DEVICES];

// Device address of the scratch on the current device, looked up once per
// device (with that device current) and cached.
int na_scratch(int dev, unsigned **out) {
    std::lock_guard<std::mutex> lock(g_na_mutex);
    if (!g_na_addr[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_na_partials);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            return TPT_CUDA_ERROR;
        }
        g_na_addr[dev] = static_cast<unsigned *>(p);
    }
    *out = g_na_addr[dev];
    return TPT_OK;
}

}  // namespace
}  // namespace tpt

extern "C" int tpt_cuda_quantize_i8_symmetric_noalloc(const float *x, size_t n, int8_t *q, float *scale,
                                                      void *stream) {
    using namespace tpt;
    if (!scale || (n && (!x || !q))) return TPT_INVALID;
    if (n > TPT_NOALLOC_QUANT_MAX_ELEMS) return TPT_INVALID;  // more partials than the scratch holds
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= (int)NA_MAX_DEVICES) {
        cudaGetLastError();
        return TPT_UNSUPPORTED;
    }
    unsigned *partials = nullptr;
    int st = na_scratch(dev, &partials);
    if (st) return st;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const unsigned tiles = (unsigned)((n + NA_TILE - 1) / NA_TILE);
    if (tiles) k_na_absmax<<<tiles, 256, 0, s>>>(x, n, partials);
    k_na_scale<<<1, 1024, 0, s>>>(partials, tiles, scale);
    if (n) {
        size_t g = (n + 255) / 256;
        if (g > 148 * 8) g = 148 * 8;
        k_na_quant<<<(unsigned)g, 256, 0, s>>>(x, n, scale, q);
    }
    return cudaGetLastError() == cudaSuccess ? TPT_OK : TPT_CUDA_ERROR;
}
