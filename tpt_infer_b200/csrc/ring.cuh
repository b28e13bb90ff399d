// ring.cuh -- the weight ring shared by the mma.sync decode kernels (W4
// digit-plane GEMV / small batch, W8A8 small batch): 16-row groups of a
// row-major byte matrix moved by one 3-D TMA tensor load each (128B-swizzled,
// no multicast) into a shared-memory ring, and the producer thread that
// streams a CTA's run of groups.
#pragma once

#include "tc_common.cuh"

namespace tpt {

constexpr int WG_ROWS = 16;  // weight rows per group (one ring stage; the MMA's M)

// A row-major byte matrix [n rows, row_bytes] (row_bytes % 128 == 0, at most
// 32768) as the 3-D tensor {128 B, n rows, row_bytes / 128 columns} with box
// {128, 16, row_bytes / 128} and 128B swizzle: one load brings a 16-row group,
// rows past n read as zero, and every address stays inside the matrix.
inline bool make_tmap_rows3d(CUtensorMap *tm, const void *base, uint64_t n, uint64_t row_bytes) {
    auto fn = encode_fn();
    if (!fn || ((uintptr_t)base & 15) || (row_bytes % 128) || row_bytes / 128 > 256) return false;
    cuuint64_t dims[3] = {128, n, row_bytes / 128};
    cuuint64_t strides[2] = {row_bytes, 128};
    cuuint32_t box[3] = {128, (cuuint32_t)WG_ROWS, (cuuint32_t)(row_bytes / 128)};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

namespace ring {
using namespace tc;

// One stage: rows [y, y + 16) x the whole row, as 16-row x 128-byte boxes per
// 128-byte column (3-D view {128 B, rows, columns}), 128B-swizzled.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *tm, uint32_t bar, int y) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(0), "r"(y), "r"(0)
        : "memory");
}

// byte offset of (row, byte b of the row) in a stage: column b / 128 holds 16
// rows of 128 bytes; the 16-byte unit u of row r sits at u ^ (r & 7)
__device__ __forceinline__ uint32_t stage_off(int row, uint32_t b) {
    return (b >> 7) * (WG_ROWS * 128u) + (uint32_t)row * 128u + ((((b >> 4) & 7u) ^ (uint32_t)(row & 7)) << 4) +
           (b & 15u);
}

// ---------------- TMA producer (one thread) ----------------
// The first S groups are requested before the dependency wait: the nibbles are
// constants (written only by host uploads, which a programmatic launch never
// overlaps), so they stream while the previous kernel finishes.
__device__ __forceinline__ void produce(const CUtensorMap &tmW, uint32_t ring, uint32_t stage_bytes, uint32_t bars,
                                        int S, int g0, int g1, volatile int *abort_p, unsigned *gflags) {
    auto full_bar = [&](int s) { return bars + 8u * s; };
    auto empty_bar = [&](int s) { return bars + 8u * (S + s); };
    int s = 0;
    uint32_t ph = 0, issued = 0, last_ph = 0;
    for (int g = g0; g < g1; g++) {
        if (g == g0 + S) {
            pdl_wait();
            pdl_trigger();
        }
        if (!mbar_wait(empty_bar(s), ph ^ 1u, abort_p, gflags, true)) break;
        mbar_arrive_expect_tx(full_bar(s), stage_bytes);  // the whole box, rows past N read as 0
        tma_load_3d(ring + (uint32_t)s * stage_bytes, &tmW, full_bar(s), g * WG_ROWS);
        issued |= 1u << s;
        last_ph = (last_ph & ~(1u << s)) | (ph << s);
        if (++s == S) {
            s = 0;
            ph ^= 1u;
        }
    }
    if (g1 - g0 <= S) {
        pdl_wait();
        pdl_trigger();
    }
    // our copies in flight land before the CTA can exit
    for (int t = 0; t < S; t++)
        if (issued & (1u << t)) mbar_wait(full_bar(t), (last_ph >> t) & 1u, abort_p, gflags, false);
}

}  // namespace ring
}  // namespace tpt
