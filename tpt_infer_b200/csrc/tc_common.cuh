// tc_common.cuh -- device helpers shared by the tcgen05 kernels: mbarriers
// with bounded waits, TMA tile loads/stores, tcgen05 fences/commit/ld, and the
// shared-memory matrix descriptor of 128B-swizzled K-major operand tiles.
// No TMA load here uses cluster multicast.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace tpt {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn();  // null when the driver lacks it

namespace tc {

// Bound of one wait in SM clock cycles: about 1 s at the B200's 1.965 GHz
// boost clock (longer at lower clocks, never unbounded). The SM-local cycle
// counter is read instead of %globaltimer, whose read is slow enough to add a
// visible delay to every wait that does not succeed on its first poll.
constexpr long long TPT_WAIT_CYCLES = 2000000000ll;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// ---- thread-block clusters ----
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank`
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// every thread of every CTA of the cluster (a hardware barrier)
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// arrival on another CTA's mbarrier with the default CTA-scope release
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 4-byte store into another CTA's shared memory (shared::cluster address) that
// counts its bytes on that CTA's mbarrier `bar_cluster`
__device__ __forceinline__ void st_async_b32(uint32_t addr_cluster, uint32_t v, uint32_t bar_cluster) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.b32 [%0], %1, [%2];" ::"r"(addr_cluster), "r"(v),
                 "r"(bar_cluster)
                 : "memory");
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait. Returns false when the CTA is aborting or the wait ran out
// (then the abort is raised and the global timeout flag recorded). The abort
// flag and the clock are checked every 16 polls. Progress waits
// (honour_abort) use the context's wait limit when one is set
// (gflags[TPT_FLAG_WAIT_LIMIT], cycles; tpt_cuda_ctx_set_wait_limit), so a test
// can make a normal launch run out of its waits; the drain waits of an
// aborting CTA (its own copies and MMAs still in flight) always keep the full
// bound, so no CTA exits while the hardware still writes its memory.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

static __device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag, unsigned *gflags,
                                       bool honour_abort) {
    // The context's limit is read through the read-only path, issued before the
    // first poll: it changes only between launches (the host sets it), so after
    // an SM's first read it is an L1 hit, and its latency overlaps the poll
    // instead of adding to every wait that the first poll does not end (a
    // producer waiting on each freed stage would otherwise pay an L2 round
    // trip per stage)
    const unsigned l = (honour_abort && gflags) ? __ldg(gflags + TPT_FLAG_WAIT_LIMIT) : 0u;
    if (mbar_try_wait(bar, parity)) return true;
    long long limit = TPT_WAIT_CYCLES;
    if (honour_abort && gflags) {
        if (l) {  // a limit set by the context: poll without the hardware's suspend, check the clock each time
            const long long t0 = clock64();
            while (!mbar_test_wait(bar, parity)) {
                if (*abort_flag) return false;
                if (clock64() - t0 > (long long)l) {
                    *abort_flag = 1;
                    atomicOr(gflags + TPT_FLAG_TIMEOUT, 1u);
                    return false;
                }
            }
            return true;
        }
    }
    const long long t0 = clock64();
    for (uint32_t i = 1;; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15u) == 0) {
            if (honour_abort && *abort_flag) return false;
            if (clock64() - t0 > limit) {
                *abort_flag = 1;
                if (gflags) atomicOr(gflags + TPT_FLAG_TIMEOUT, 1u);
                return false;
            }
        }
    }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *tm, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(x), "r"(y)
        : "memory");
}

// Pulls the box at {x, y} of the tensor map into L2 (no shared memory, no
// completion); a hint, coherent with every write, so it may run before
// pdl_wait() for constant operands (weights).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap *tm, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(tm)),
                 "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i gets its lane's 32 values.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t *v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major, 128B-swizzled operand tile:
// 8-row x 128-byte swizzle atoms stacked along M/N (stride 1024 B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address, bits 0-13
    d |= (uint64_t)1 << 16;                     // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;           // stride byte offset: 8 rows x 128 B
    d |= (uint64_t)1 << 46;                     // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                     // swizzle mode: 128B
    return d;
}

// 2-D bulk-tensor store of one 32 x 32 (4-byte) block from shared memory.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *tm, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(reinterpret_cast<uint64_t>(tm)), "r"(src), "r"(x), "r"(y)
                 : "memory");
}

// Named barrier over `count` threads (a multiple of 32) that also ANDs a
// predicate across them: every participant gets the same answer.
__device__ __forceinline__ bool bar_and(int id, int count, bool p) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred a, b;\n setp.ne.u32 a, %1, 0;\n bar.red.and.pred b, %2, %3, a;\n selp.u32 %0, 1, 0, b;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)p), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Stream-K grids are at most this many CTAs (one per SM), so a split tile has
// at most this many contributors.
constexpr int TPT_SK_MAX_CTAS = 256;

// The CTA whose stream-K unit range [U*c/G, U*(c+1)/G) holds unit u.
__host__ __device__ inline int sk_cta_of_unit(long long u, long long units, int ctas) {
    return (int)(((u + 1) * ctas + units - 1) / units) - 1;
}
// Partial-tile slot of CTA c for `tile`: only the first and the last segment
// of a CTA's range can be partial, so they own slots 2c and 2c + 1 (the
// workspace is bounded by the grid, not by the tile count). A split tile's
// counter is indexed by its first contributor, which no other split tile has.
__device__ inline int sk_slot(int c, int tile, long long units, int kblocks, int ctas) {
    const long long u0 = units * c / ctas;
    return 2 * c + ((int)(u0 / kblocks) == tile ? 0 : 1);
}

// Stream-K schedule: U = tiles x kblocks units split into gridDim equal
// contiguous ranges; a CTA walks its range as segments (tile, [kb0, kb1)).
struct SkRange {
    long long u, u1;
    int kblocks;
    __device__ SkRange(long long units, int kb, int cta, int ctas)
        : u(units * cta / ctas), u1(units * (cta + 1) / ctas), kblocks(kb) {}
    __device__ bool next(int &tile, int &kb0, int &kb1) {
        if (u >= u1) return false;
        tile = (int)(u / kblocks);
        kb0 = (int)(u - (long long)tile * kblocks);
        const long long left = u1 - u;
        kb1 = left < (long long)(kblocks - kb0) ? kb0 + (int)left : kblocks;
        u += kb1 - kb0;
        return true;
    }
};

}  // namespace tc
}  // namespace tpt
