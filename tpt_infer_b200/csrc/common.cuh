// common.cuh -- shared host/device plumbing of the tpt-infer B200 backend.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include <string>

#include "../../include/tpt_cuda.h"
#include "det_math.cuh"

// Device-side error words (one 32-bit word each), written by kernels whose
// bounded waits ran out or whose own index checks failed. Read and cleared by
// tpt_cuda_ctx_sync / the host-staged entry points.
enum { TPT_FLAG_TIMEOUT = 0, TPT_FLAG_CHECK = 1, TPT_FLAG_WAIT_LIMIT = 2, TPT_FLAG_WORDS = 4 };

struct tpt_cuda_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    bool own_stream = false;
    int sm_count = 0;
    // growable device scratch used by host-staged calls
    char *scratch = nullptr;
    size_t scratch_cap = 0;
    // growable device workspace used inside launches (e.g. split activations);
    // separate from `scratch` so a launch never moves a host-staged buffer
    char *ws = nullptr;
    size_t ws_cap = 0;
    // stream-K reduction workspace (i32/f32 partial tiles + per-tile counters).
    // All-zero between launches: the CTA that finishes a tile zeroes what it
    // read. A launch that timed out may leave it dirty, so sk_dirty makes the
    // next user clear it first.
    char *sk = nullptr;
    size_t sk_cap = 0;
    bool sk_dirty = false;
    // small persistent device words: error flags + reduction cells
    unsigned *d_flags = nullptr;   // TPT_FLAG_WORDS words
    unsigned *d_reduce = nullptr;  // 64 words of reduction scratch
    size_t last_expected = 0, last_actual = 0;
    std::string last_error;
    uint64_t launches = 0;
    // CUDA graph recording: while `capturing`, nothing may allocate or wait.
    // `ws_gen` counts workspace moves; a graph recorded at another generation
    // holds stale workspace addresses and is refused at launch.
    bool capturing = false;
    uint64_t capture_launches0 = 0;
    uint64_t ws_gen = 0;
    // copy streams and events of the pipelined host-buffer calls (created on
    // first use): H2D on copy_in, D2H on copy_out, compute on `stream`
    cudaStream_t copy_in = nullptr, copy_out = nullptr;
    cudaEvent_t pipe_ev[2 * 8 + 2] = {};
};

struct tpt_cuda_weights {
    tpt_cuda_ctx *ctx = nullptr;
    int device = 0;  // freeing needs only the device: the context may be gone
    int kind = 0;          // 8 = int8 [n,k]; 4 = int4 nibbles [n, k/2]
    size_t n = 0, k = 0;
    void *data = nullptr;  // device: packed weight bytes
    float *scales = nullptr;  // device: n per-channel scales
    size_t bytes = 0;
    // TMA descriptors of the int8 weight (CUtensorMap, 128 bytes each), built
    // once: boxes of 128 / 64 / 32 rows x 128 bytes (the small-M kernel's
    // weight tile, and the SM-pair kernel's B half-tiles for tile N = 256 /
    // 128 / 64)
    alignas(64) unsigned char tmaps[4][128];  // int8 weights: TMA boxes of 128 / 64 / 32 / 96 rows x 128 B
    bool tmap_ok = false;
};

namespace tpt {

// Launches `kern` on `st` with programmatic stream serialization (see
// pdl_wait); a launch error is left for after_launch's cudaGetLastError.
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    (void)cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

int set_size_mismatch(tpt_cuda_ctx *ctx, size_t expected, size_t actual);
int cuda_fail(tpt_cuda_ctx *ctx, cudaError_t e, const char *what);
// Ensures the context scratch holds at least `bytes` (grows; never shrinks).
int ensure_scratch(tpt_cuda_ctx *ctx, size_t bytes);
// Same for the launch workspace.
int ensure_ws(tpt_cuda_ctx *ctx, size_t bytes);
// Stream-K workspace layout: TPT_SK_COUNTERS tile counters at offset 0 (a
// fixed region, so kernels with different tile counts never see each other's
// partial tiles as counters), then the partial-tile slots.
constexpr size_t TPT_SK_COUNTERS = 16384;
constexpr size_t TPT_SK_SLOTS_OFFSET = TPT_SK_COUNTERS * sizeof(int);
// Ensures room for `slot_bytes` of slots after the counter region.
int ensure_sk(tpt_cuda_ctx *ctx, size_t slot_bytes);
// Waits for the stream, then reads and clears the device error words.
int sync_and_check(tpt_cuda_ctx *ctx);
// copy streams + events of the pipelined host-buffer calls, created once
int ensure_copy_streams(tpt_cuda_ctx *ctx);
// true when p lies in page-locked (pinned or registered) host memory
bool is_pinned_host(const void *p);
// Returns TPT_CUDA_ERROR if the last launch failed, else TPT_OK; counts launches.
int after_launch(tpt_cuda_ctx *ctx, const char *what, int n = 1);

// Bump allocator over the context scratch for one host-staged call.
struct Staging {
    tpt_cuda_ctx *ctx;
    size_t need = 0;
    size_t off = 0;
    explicit Staging(tpt_cuda_ctx *c) : ctx(c) {}
    static size_t align_up(size_t x) { return (x + 255) & ~size_t(255); }
    // First pass: reserve sizes; second pass: hand out pointers.
    void reserve(size_t bytes) { need += align_up(bytes); }
    int commit() { return ensure_scratch(ctx, need); }
    template <typename T> T *take(size_t count) {
        T *p = reinterpret_cast<T *>(ctx->scratch + off);
        off += align_up(count * sizeof(T));
        return p;
    }
};

int h2d(tpt_cuda_ctx *ctx, void *dst, const void *src, size_t bytes);
int d2h(tpt_cuda_ctx *ctx, void *dst, const void *src, size_t bytes);

inline unsigned grid_1d(size_t n, unsigned block, unsigned cap = 148u * 16u) {
    size_t g = (n + block - 1) / block;
    if (g == 0) g = 1;
    if (g > cap) g = cap;
    return (unsigned)g;
}

bool checked_mul(size_t a, size_t b, size_t *r);

// An int8 output for a W8A8 epilogue: y is requantized with the next
// quantization point's static scale (clamp(roundf(y / scale)), exactly the
// separate QUANTIZE op), so the f32 tensor is never written.
struct Requant {
    int8_t *q = nullptr;
    float scale = 0.0f;
};

// A residual folded into an epilogue: y = act(y + r[row, col]), r f32 with the
// output's shape (the ADD_ACT op's arithmetic)
struct Residual {
    const float *r = nullptr;
    int act = 0;
};

// ---- launchers implemented across the .cu files (device pointers, async) ----
int launch_add(tpt_cuda_ctx *ctx, const float *a, const float *b, float *out, size_t n);
int launch_unary(tpt_cuda_ctx *ctx, int op, const float *a, float *out, size_t n);  // 1 relu 2 sigmoid 3 gelu
int launch_softmax(tpt_cuda_ctx *ctx, const float *a, float *out, size_t rows, size_t row_len);
int launch_matmul_f32(tpt_cuda_ctx *ctx, const float *a, const float *b, float *out, size_t m,
                      size_t k, size_t n);
int launch_matmul_f32_epi(tpt_cuda_ctx *ctx, const float *a, const float *b, const float *bias, int act, float *out,
                          size_t m, size_t k, size_t n);
int launch_matmul_f32_softmax(tpt_cuda_ctx *ctx, const float *a, const float *b, const float *bias, int act,
                              float *out, float *softmax_out, size_t m, size_t k, size_t n, bool *handled);
int launch_bias_act(tpt_cuda_ctx *ctx, const float *x, const float *bias, float *y, size_t rows, size_t cols, int act);
int launch_conv2d_f32(tpt_cuda_ctx *ctx, const float *in, const float *w, float *out, const size_t is[4],
                      const size_t ws[4], size_t oh, size_t ow, size_t sh, size_t sw, size_t ph,
                      size_t pw);
int launch_quant_i8_sym(tpt_cuda_ctx *ctx, const float *x, size_t n, int8_t *q, float *scale_dev,
                        unsigned *cell);
int launch_quant_i8_static(tpt_cuda_ctx *ctx, const float *x, size_t n, float scale, int8_t *q);
int launch_quant_i8_rows(tpt_cuda_ctx *ctx, const float *x, size_t rows, size_t cols, int8_t *q,
                         float *scales);
int launch_quant_i8_asym(tpt_cuda_ctx *ctx, const float *x, size_t n, int8_t *q, float *scale_dev,
                         int32_t *zp_dev, unsigned *cells);
int launch_pack_i4(tpt_cuda_ctx *ctx, const int8_t *v, size_t n, uint8_t *out, unsigned *bad);
int launch_unpack_i4(tpt_cuda_ctx *ctx, const uint8_t *p, size_t count, int8_t *out);
int launch_quant_i4_rows(tpt_cuda_ctx *ctx, const float *x, size_t rows, size_t cols, uint8_t *p,
                         float *scales);
int launch_dequant_i8_rows(tpt_cuda_ctx *ctx, const int8_t *q, size_t rows, size_t cols,
                           const float *scales, float *out);
int launch_dequant_i4_rows(tpt_cuda_ctx *ctx, const uint8_t *p, size_t rows, size_t row_elems,
                           size_t packed_len, const float *scales, float *out);
int launch_dequant_i8_asym(tpt_cuda_ctx *ctx, const int8_t *q, size_t n, float scale, int32_t zp, float *out);
// i8 GEMM: y[m,n] (+bias, act), raw i32 acc when acc != nullptr, or y
// requantized to int8 when rq.q != nullptr; W^T [n,k].
int launch_w8a8(tpt_cuda_ctx *ctx, const int8_t *a, size_t m, size_t k, const tpt_cuda_weights *w,
                float a_scale, const float *bias, int act, float *y, int32_t *acc, Requant rq = Requant{});
// ONNX Gemm: y = alpha * op(a) op(b) + beta * c; c_mode 0 none, 1 [n], 2 [m,n]
int launch_gemm_onnx(tpt_cuda_ctx *ctx, const float *a, const float *b, const float *c, int c_mode, float alpha,
                     float beta, float *y, size_t m, size_t k, size_t n, bool ta, bool tb);
int launch_w4(tpt_cuda_ctx *ctx, const float *x, size_t m, const tpt_cuda_weights *w,
              const float *bias, int act, float *y);

}  // namespace tpt

// ------------------------------------------------------------------ device helpers
#ifdef __CUDACC__
namespace tpt {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// GELU of crates/tpt-infer-ops/src/naive.rs:137-146 (tanh approximation),
// evaluated by gelu_det (det_math.cuh): the same inner term, the tanh through
// exp_det, so every GELU on the device has a bit-exact CPU restatement.
__device__ __forceinline__ float apply_act(float y, int act) {
    if (act == TPT_ACT_RELU) return y > 0.0f ? y : 0.0f;
    if (act == TPT_ACT_GELU) return gelu_det(y);
    return y;
}

// Programmatic dependent launch. A kernel launched with launch_pdl may start
// while the previous kernel on the stream is still finishing: pdl_wait()
// blocks until that kernel has completed and its memory is visible, so every
// read of a predecessor's output (and every write) comes after it; each such
// kernel calls it unconditionally, before any early exit, so it cannot
// complete ahead of its predecessor. pdl_trigger() then lets the next kernel
// be scheduled while this one runs (its own pdl_wait still waits for this
// kernel's completion).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Starts pulling [p, p + bytes) into L2 (the bulk copy unit, no registers, no
// completion to wait for); p 16-byte aligned, bytes a multiple of 16. A hint
// only: L2 is coherent with every write, so this may be issued before
// pdl_wait() for buffers the predecessor could still be writing. Used for
// weights before pdl_wait(), so their HBM stream overlaps the previous kernel.
__device__ __forceinline__ void prefetch_l2_bulk(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <int ACT>
__device__ __forceinline__ float act_t(float y) {
    if constexpr (ACT == TPT_ACT_RELU) return y > 0.0f ? y : 0.0f;
    else if constexpr (ACT == TPT_ACT_GELU) return gelu_det(y);
    else return y;
}

// The channel scales and biases of one 32-column chunk (columns n0 .. n0+31):
// broadcast loads (every lane of a warp passes the same n0), 128-bit when
// aligned and in range, clamped to column N-1 past the edge.
__device__ __forceinline__ void w8a8_load_consts(int n0, int N, const float *ws, const float *bias, float (&sc)[32],
                                                 float (&bi)[32]) {
    if (n0 + 32 <= N && ((reinterpret_cast<uintptr_t>(ws + n0) | reinterpret_cast<uintptr_t>(bias + n0)) & 15) == 0) {
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const float4 w4 = __ldg(reinterpret_cast<const float4 *>(ws + n0) + c);
            sc[4 * c] = w4.x;
            sc[4 * c + 1] = w4.y;
            sc[4 * c + 2] = w4.z;
            sc[4 * c + 3] = w4.w;
            const float4 b4 = bias ? __ldg(reinterpret_cast<const float4 *>(bias + n0) + c) : make_float4(0, 0, 0, 0);
            bi[4 * c] = b4.x;
            bi[4 * c + 1] = b4.y;
            bi[4 * c + 2] = b4.z;
            bi[4 * c + 3] = b4.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; j++) {
            const int n = n0 + j < N ? n0 + j : N - 1;
            sc[j] = __ldg(ws + n);
            bi[j] = bias ? __ldg(bias + n) : 0.0f;
        }
    }
}

// The W8A8 epilogue of one 32-column chunk of one row, in place: i32
// accumulators become the f32 bits of act((float)acc * (a_scale * sc[j]) +
// bi[j]) (the product of the scales first, separately rounded multiply and
// add; no add without a bias, which keeps -0).
template <int ACT>
__device__ __forceinline__ void w8a8_apply32(uint32_t (&v)[32], float a_scale, const float (&sc)[32],
                                             const float (&bi)[32], bool has_bias) {
#pragma unroll
    for (int j = 0; j < 32; j++) {
        float y = __fmul_rn(__int2float_rn((int)v[j]), __fmul_rn(a_scale, sc[j]));
        if (has_bias) y = __fadd_rn(y, bi[j]);
        v[j] = __float_as_uint(act_t<ACT>(y));
    }
}

// w8a8_apply32 on paired f32 operations (two columns per issue; the int ->
// float conversion stays scalar): the same operations in the same order on
// each half, so the same bits. nz from opaque_nz2 (the dequantized product
// feeds the bias add).
template <int ACT>
__device__ __forceinline__ void w8a8_apply32_x2(uint32_t (&v)[32], float a_scale, const float (&sc)[32],
                                                const float (&bi)[32], bool has_bias, uint64_t nz) {
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
        uint64_t y = mulr2(f2pack(__int2float_rn((int)v[j]), __int2float_rn((int)v[j + 1])),
                           mul2(splat2(a_scale), f2pack(sc[j], sc[j + 1])), nz);
        if (has_bias) y = add2(y, f2pack(bi[j], bi[j + 1]));
        float y0, y1;
        f2unpack(y, y0, y1);
        if constexpr (ACT == TPT_ACT_GELU) {
            gelu_det_x2(y0, y1, nz, y0, y1);
        } else {
            y0 = act_t<ACT>(y0);
            y1 = act_t<ACT>(y1);
        }
        v[j] = __float_as_uint(y0);
        v[j + 1] = __float_as_uint(y1);
    }
}

// Both of the above for columns n0 .. n0+31
template <int ACT>
__device__ __forceinline__ void w8a8_epi32(uint32_t (&v)[32], int n0, int N, float a_scale, const float *ws,
                                           const float *bias) {
    float sc[32], bi[32];
    w8a8_load_consts(n0, N, ws, bias, sc, bi);
    w8a8_apply32<ACT>(v, a_scale, sc, bi, bias != nullptr);
}
// The activation of 32 values (f32 bits) in place, for epilogues that keep
// their code small: ReLU as a select, GELU through an out-of-line call.
static __device__ __noinline__ float gelu_outline(float y) { return gelu_det(y); }
__device__ __forceinline__ void act32(uint32_t (&v)[32], int act) {
    if (act == TPT_ACT_RELU) {
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = __float_as_uint(act_t<TPT_ACT_RELU>(__uint_as_float(v[j])));
    } else if (act == TPT_ACT_GELU) {
#pragma unroll
        for (int j = 0; j < 32; j++) v[j] = __float_as_uint(gelu_outline(__uint_as_float(v[j])));
    }
}
__device__ __forceinline__ void w8a8_epi32(uint32_t (&v)[32], int n0, int N, float a_scale, const float *ws,
                                           const float *bias, int act) {
    if (act == TPT_ACT_RELU)
        w8a8_epi32<TPT_ACT_RELU>(v, n0, N, a_scale, ws, bias);
    else if (act == TPT_ACT_GELU)
        w8a8_epi32<TPT_ACT_GELU>(v, n0, N, a_scale, ws, bias);
    else
        w8a8_epi32<TPT_ACT_NONE>(v, n0, N, a_scale, ws, bias);
}

// Rust `f32::round(v).clamp(lo, hi) as i8`: half away from zero (roundf),
// NaN -> 0 (saturating cast).
__device__ __forceinline__ int8_t round_clamp_i8(float v, float lo, float hi) {
    v = roundf(v);
    if (isnan(v)) return 0;
    v = fminf(fmaxf(v, lo), hi);
    return (int8_t)(int)v;
}

// quantize_i8_static's rule for one value: clamp(roundf(y / scale), -127, 127)
__device__ __forceinline__ int8_t requant_i8(float y, float scale) {
    return round_clamp_i8(__fdiv_rn(y, scale), -127.0f, 127.0f);
}

// The same rule without a division, for scales in [2^-40, 2^40] (requant_fast_ok).
// rs = RN(1 / s) (__frcp_rn). q1 = y * rs is within a few ulps of y / s; one
// residual step (r = y - s q by FMA, q += r rs) makes it faithful, and a second
// is Markstein's correction step (P. Markstein, IBM J. Res. Dev. 34(1), 1990),
// which turns a faithful quotient into the correctly rounded one, the IEEE
// quotient, whenever the residual is exact. The residual can be inexact only
// when it underflows, for quotients far below 0.5 that round to 0 either way;
// |y| > 2^80 clamps to +-127 whatever the quotient. Rounding half away from
// zero (roundf): trunc(q + copysign(0.5 - 2^-25, q)) equals roundf(q) for every
// float below 2^31 in magnitude (checked exhaustively), the truncating
// conversion saturates above that and takes NaN to 0, and the integer clamp
// gives [-127, 127]. No branch, so the 32 values of an epilogue chunk interleave.
__device__ __forceinline__ bool requant_fast_ok(float s) { return s >= 0x1p-40f && s <= 0x1p40f; }
__device__ __forceinline__ int8_t requant_i8_fast(float y, float s, float rs) {
    const float q1 = __fmul_rn(y, rs);
    const float q2 = __fmaf_rn(__fmaf_rn(-s, q1, y), rs, q1);
    float q = __fmaf_rn(__fmaf_rn(-s, q2, y), rs, q2);
    q = fabsf(y) <= 0x1p80f ? q : y;
    const float h = __fadd_rn(q, copysignf(0.49999997f, q));
    int n = __float2int_rz(h);  // cvt.rzi.s32.f32: saturating, NaN -> 0
    n = n > 127 ? 127 : (n < -127 ? -127 : n);
    return (int8_t)n;
}
// requant_i8_fast of two values, the quotient steps on paired operations
// (nz from opaque_nz2)
__device__ __forceinline__ void requant_i8_fast_x2(float y0, float y1, float s, float rs, uint64_t nz, int8_t &q0,
                                                   int8_t &q1) {
    const uint64_t Y = f2pack(y0, y1), RS = splat2(rs), NS = splat2(-s);
    const uint64_t qa = mulr2(Y, RS, nz);
    const uint64_t qb = fma2(fma2(NS, qa, Y), RS, qa);
    float a0, a1;
    f2unpack(fma2(fma2(NS, qb, Y), RS, qb), a0, a1);
    a0 = fabsf(y0) <= 0x1p80f ? a0 : y0;
    a1 = fabsf(y1) <= 0x1p80f ? a1 : y1;
    float h0, h1;
    f2unpack(add2(f2pack(a0, a1), f2pack(copysignf(0.49999997f, a0), copysignf(0.49999997f, a1))), h0, h1);
    int n0 = __float2int_rz(h0), n1 = __float2int_rz(h1);  // saturating, NaN -> 0
    n0 = n0 > 127 ? 127 : (n0 < -127 ? -127 : n0);
    n1 = n1 > 127 ? 127 : (n1 < -127 ? -127 : n1);
    q0 = (int8_t)n0;
    q1 = (int8_t)n1;
}
// out of line: the dividing path of the wide epilogues (scales outside the fast range)
static __device__ __noinline__ int8_t requant_i8_outline(float y, float s) { return requant_i8(y, s); }

// requant_pack32 with the fast path on paired operations
__device__ __forceinline__ void requant_pack32_x2(const uint32_t (&v)[32], float s, float rs, bool fast, uint64_t nz,
                                                  uint32_t (&qb)[8]) {
    if (fast) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            int8_t a, b, c, d;
            requant_i8_fast_x2(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), s, rs, nz, a, b);
            requant_i8_fast_x2(__uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]), s, rs, nz, c, d);
            qb[j / 4] = (uint32_t)(uint8_t)a | ((uint32_t)(uint8_t)b << 8) | ((uint32_t)(uint8_t)c << 16) |
                        ((uint32_t)(uint8_t)d << 24);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
            qb[j / 4] = (uint32_t)(uint8_t)requant_i8_outline(__uint_as_float(v[j]), s) |
                        ((uint32_t)(uint8_t)requant_i8_outline(__uint_as_float(v[j + 1]), s) << 8) |
                        ((uint32_t)(uint8_t)requant_i8_outline(__uint_as_float(v[j + 2]), s) << 16) |
                        ((uint32_t)(uint8_t)requant_i8_outline(__uint_as_float(v[j + 3]), s) << 24);
    }
}

// requant_i8 of 32 values (f32 bits) packed 4 to a word, low byte first
__device__ __forceinline__ void requant_pack32(const uint32_t (&v)[32], float s, float rs, bool fast,
                                               uint32_t (&qb)[8]) {
    if (fast) {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
            qb[j / 4] = (uint32_t)(uint8_t)requant_i8_fast(__uint_as_float(v[j]), s, rs) |
                        ((uint32_t)(uint8_t)requant_i8_fast(__uint_as_float(v[j + 1]), s, rs) << 8) |
                        ((uint32_t)(uint8_t)requant_i8_fast(__uint_as_float(v[j + 2]), s, rs) << 16) |
                        ((uint32_t)(uint8_t)requant_i8_fast(__uint_as_float(v[j + 3]), s, rs) << 24);
    } else {
#pragma unroll
        for (int j = 0; j < 32; j += 4)
            qb[j / 4] = (uint32_t)(uint8_t)requant_i8_outline(__uint_as_float(v[j]), s) |
                        ((uint32_t)(uint8_t)requant_i8_outline(__uint_as_float(v[j + 1]), s) << 8) |
                        ((uint32_t)(uint8_t)requant_i8_outline(__uint_as_float(v[j + 2]), s) << 16) |
                        ((uint32_t)(uint8_t)requant_i8_outline(__uint_as_float(v[j + 3]), s) << 24);
    }
}

}  // namespace tpt
#endif
