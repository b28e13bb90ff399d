// selftest.cu -- a check of the device-side failure detection that needs no
// fault: one CTA waits, through the same bounded mbarrier wait every
// tensor-core and TMA-ring kernel uses (tc_common.cuh mbar_wait), on a barrier
// that nothing ever arrives on. The wait runs out after the context's wait
// limit, records the timeout in the context's device flag words, raises the
// CTA's abort and returns; the host reads TPT_TIMEOUT at the next
// synchronising call and the context stays usable.
#include "tc_common.cuh"

namespace tpt {
namespace {
using namespace tc;

__global__ void k_selftest_wait(unsigned *gflags, unsigned *result) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        mbar_init(smem_u32(&bar), 1);  // one arrival completes phase 0; none ever comes
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    volatile int *abort_p = &abort_flag;
    const bool ok = mbar_wait(smem_u32(&bar), 0, abort_p, gflags, true);
    __syncthreads();
    if (threadIdx.x == 0) result[0] = (ok ? 1u : 0u) | ((*abort_p ? 1u : 0u) << 1);
}

}  // namespace
}  // namespace tpt

using namespace tpt;

extern "C" int tpt_cuda_selftest_bounded_wait(tpt_cuda_ctx *ctx, unsigned *outcome) {
    if (!ctx || !outcome) return TPT_INVALID;
    cudaSetDevice(ctx->device);
    unsigned *d = ctx->d_reduce + 63;  // the last word of the context's reduction scratch
    cudaError_t e = cudaMemsetAsync(d, 0xff, sizeof(unsigned), ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "self-test");
    k_selftest_wait<<<1, 32, 0, ctx->stream>>>(ctx->d_flags, d);
    int st = after_launch(ctx, "selftest_wait");
    if (st) return st;
    e = cudaMemcpyAsync(outcome, d, sizeof(unsigned), cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "self-test read");
    return sync_and_check(ctx);  // TPT_TIMEOUT: the wait ran out and was reported
}
