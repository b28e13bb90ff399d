// comm.cu -- the NCCL communicator of the multi-GPU paths (one process per
// GPU, all on one node, NVLink/NVSwitch between them).
//
// tpt-infer itself is single-process; this is the exchange step of the
// column-sharded FFN (each rank computes 1/P of the FFN1 output channels, the
// per-channel quantization axis, and an all-gather reassembles them) and of
// the rank-global activation scale of such a sharded tensor (a max-reduction
// of the calibration max). Every collective is enqueued on the context's
// stream, in the same order on every rank.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, which reuses an
// already-loaded copy, e.g. the one PyTorch ships), so single-GPU users of the
// library never need it. Communicator set-up runs non-blocking and is polled
// with a deadline: a rank that never joins ends in TPT_NCCL_ERROR, not a hang.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <atomic>
#include <chrono>
#include <mutex>
#include <new>
#include <thread>

#include "common.cuh"

struct tpt_cuda_comm {
    tpt_cuda_ctx *ctx = nullptr;
    ncclComm_t comm = nullptr;
    int world = 0, rank = 0;
};

namespace tpt {
namespace {

struct NcclApi {
    bool ok = false;
    ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*commInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    const char *(*getErrorString)(ncclResult_t) = nullptr;
};

NcclApi load_nccl() {
    NcclApi a;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return a;
#define TPT_SYM(field, name) a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, name))
    TPT_SYM(getUniqueId, "ncclGetUniqueId");
    TPT_SYM(commInitRankConfig, "ncclCommInitRankConfig");
    TPT_SYM(commGetAsyncError, "ncclCommGetAsyncError");
    TPT_SYM(commDestroy, "ncclCommDestroy");
    TPT_SYM(commAbort, "ncclCommAbort");
    TPT_SYM(allGather, "ncclAllGather");
    TPT_SYM(allReduce, "ncclAllReduce");
    TPT_SYM(getErrorString, "ncclGetErrorString");
#undef TPT_SYM
    a.ok = a.getUniqueId && a.commInitRankConfig && a.commGetAsyncError && a.commDestroy && a.commAbort &&
           a.allGather && a.allReduce && a.getErrorString;
    return a;
}

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] { api = load_nccl(); });
    return api;
}

constexpr double COMM_TIMEOUT_S = 120.0;
std::atomic<double> g_comm_timeout_s{COMM_TIMEOUT_S};  // tpt_cuda_comm_set_timeout

int nccl_fail(tpt_cuda_ctx *ctx, ncclResult_t r, const char *what) {
    if (ctx) {
        ctx->last_error = std::string(what) + ": " + (nccl().getErrorString ? nccl().getErrorString(r) : "nccl");
    }
    return TPT_NCCL_ERROR;
}

// A non-blocking communicator's call may return ncclInProgress; wait (bounded)
// until the communicator reports completion of the enqueue or an error.
int settle(tpt_cuda_comm *c, ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return TPT_OK;
    if (r != ncclInProgress) return nccl_fail(c->ctx, r, what);
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        ncclResult_t s = ncclInProgress;
        ncclResult_t q = nccl().commGetAsyncError(c->comm, &s);
        if (q != ncclSuccess) return nccl_fail(c->ctx, q, what);
        if (s == ncclSuccess) return TPT_OK;
        if (s != ncclInProgress) return nccl_fail(c->ctx, s, what);
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > g_comm_timeout_s.load())
            return nccl_fail(c->ctx, ncclInProgress, what);
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace

int comm_all_gather(tpt_cuda_comm *c, const void *in, void *out, size_t bytes_per_rank) {
    if (!c || !c->comm) return TPT_INVALID;
    return settle(c, nccl().allGather(in, out, bytes_per_rank, ncclInt8, c->comm, c->ctx->stream), "ncclAllGather");
}

// In-place max over the ranks of `n` 32-bit unsigned words (non-negative
// float bit patterns order like the floats).
int comm_max_u32(tpt_cuda_comm *c, unsigned *words, size_t n) {
    if (!c || !c->comm) return TPT_INVALID;
    return settle(c, nccl().allReduce(words, words, n, ncclUint32, ncclMax, c->comm, c->ctx->stream),
                  "ncclAllReduce");
}

}  // namespace tpt

using namespace tpt;

extern "C" {

int tpt_cuda_comm_unique_id(unsigned char *id, size_t id_bytes) {
    if (!id || id_bytes != sizeof(ncclUniqueId)) return TPT_INVALID;
    if (!nccl().ok) return TPT_UNSUPPORTED;
    ncclUniqueId u;
    ncclResult_t r = nccl().getUniqueId(&u);
    if (r != ncclSuccess) return TPT_NCCL_ERROR;
    memcpy(id, &u, sizeof u);
    return TPT_OK;
}

int tpt_cuda_comm_create(tpt_cuda_ctx *ctx, const unsigned char *id, size_t id_bytes, int world, int rank,
                         tpt_cuda_comm **out) {
    if (!ctx || !id || !out || id_bytes != sizeof(ncclUniqueId) || world < 1 || rank < 0 || rank >= world)
        return TPT_INVALID;
    *out = nullptr;
    if (!nccl().ok) return TPT_UNSUPPORTED;
    cudaSetDevice(ctx->device);
    tpt_cuda_comm *c = new (std::nothrow) tpt_cuda_comm();
    if (!c) return TPT_OUT_OF_MEMORY;
    c->ctx = ctx;
    c->world = world;
    c->rank = rank;
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = nccl().commInitRankConfig(&c->comm, world, u, rank, &cfg);
    int st = TPT_OK;
    if (r != ncclSuccess && r != ncclInProgress) {
        st = nccl_fail(ctx, r, "ncclCommInitRankConfig");
    } else {
        st = settle(c, ncclInProgress, "NCCL communicator set-up");
    }
    if (st) {
        if (c->comm) nccl().commAbort(c->comm);
        delete c;
        return st;
    }
    *out = c;
    return TPT_OK;
}

int tpt_cuda_comm_set_timeout(double seconds) {
    if (!(seconds >= 0.0)) return TPT_INVALID;
    g_comm_timeout_s.store(seconds > 0.0 ? seconds : COMM_TIMEOUT_S);
    return TPT_OK;
}

int tpt_cuda_comm_destroy(tpt_cuda_comm *c) {
    if (!c) return TPT_INVALID;
    if (c->comm) {
        cudaSetDevice(c->ctx->device);
        cudaStreamSynchronize(c->ctx->stream);
        nccl().commDestroy(c->comm);
    }
    delete c;
    return TPT_OK;
}

int tpt_cuda_comm_size(const tpt_cuda_comm *c, int *world, int *rank) {
    if (!c) return TPT_INVALID;
    if (world) *world = c->world;
    if (rank) *rank = c->rank;
    return TPT_OK;
}

int tpt_cuda_all_gather_dev(tpt_cuda_comm *c, const void *in, void *out, size_t bytes_per_rank) {
    if (!c || (!in && bytes_per_rank) || (!out && bytes_per_rank)) return TPT_INVALID;
    cudaSetDevice(c->ctx->device);
    return comm_all_gather(c, in, out, bytes_per_rank);
}

}  // extern "C"
