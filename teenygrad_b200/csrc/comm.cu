// NCCL communicator for the batch-sharded multi-GPU path.
//
// One process per GPU; each rank runs the hot path on its own shard of the
// batch and the only exchange is an all-gather of the final outputs (token
// ids / logits) over NVLink.  NCCL is reached through dlopen of libnccl.so.2
// (in a PyTorch process that is the copy PyTorch already loaded), so the
// library has no link-time NCCL dependency.  The communicator is created
// non-blocking; every host-side wait on it is bounded by the timeout given to
// tb_comm_init, after which the communicator is aborted and TB_ERR_NCCL
// returned.
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>
#include <time.h>

#include <mutex>

#include "tb_internal.h"

namespace tb {

struct NcclApi {
    bool ok = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};

static NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
#define TB_SYM(f) api.f = reinterpret_cast<decltype(api.f)>(dlsym(h, "nccl" #f))
        TB_SYM(GetUniqueId);
        TB_SYM(CommInitRankConfig);
        TB_SYM(AllGather);
        TB_SYM(CommGetAsyncError);
        TB_SYM(CommAbort);
        TB_SYM(CommDestroy);
        TB_SYM(GetErrorString);
#undef TB_SYM
        api.ok = api.GetUniqueId && api.CommInitRankConfig && api.AllGather && api.CommGetAsyncError &&
                 api.CommAbort && api.CommDestroy && api.GetErrorString;
    });
    return api;
}

struct Comm {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0, timeout_ms = 0;
};

static double now_ms() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e3 + ts.tv_nsec * 1e-6;
}

// Polls the communicator until it leaves ncclInProgress; aborts it after the timeout.
static int wait_ready(tb_ctx* ctx, Comm* c, const char* what) {
    NcclApi& api = nccl();
    const double t0 = now_ms();
    while (true) {
        ncclResult_t st = ncclInProgress;
        ncclResult_t r = api.CommGetAsyncError(c->comm, &st);
        if (r != ncclSuccess) st = r;
        if (st == ncclSuccess) return TB_OK;
        if (st != ncclInProgress) {
            api.CommAbort(c->comm);
            c->comm = nullptr;
            return set_error(ctx, TB_ERR_NCCL, "%s: %s", what, api.GetErrorString(st));
        }
        if (now_ms() - t0 > c->timeout_ms) {
            api.CommAbort(c->comm);
            c->comm = nullptr;
            return set_error(ctx, TB_ERR_NCCL, "%s: no progress after %d ms (peer missing?); communicator aborted", what,
                             c->timeout_ms);
        }
        timespec ts{0, 200000};
        nanosleep(&ts, nullptr);
    }
}

}  // namespace tb

using namespace tb;

extern "C" {

int tb_comm_unique_id_bytes(void) { return (int)sizeof(ncclUniqueId); }

int tb_comm_get_unique_id(void* out) {
    if (!out) return TB_ERR_ARG;
    NcclApi& api = nccl();
    if (!api.ok) return TB_ERR_NCCL;
    ncclUniqueId id;
    if (api.GetUniqueId(&id) != ncclSuccess) return TB_ERR_NCCL;
    memcpy(out, &id, sizeof(id));
    return TB_OK;
}

int tb_comm_init(tb_ctx* ctx, const void* unique_id, int nranks, int rank, int timeout_ms) {
    if (!ctx || !unique_id) return TB_ERR_ARG;
    TB_REQUIRE(ctx, nranks >= 1 && rank >= 0 && rank < nranks, TB_ERR_ARG, "comm_init: rank %d of %d", rank, nranks);
    TB_REQUIRE(ctx, timeout_ms > 0, TB_ERR_ARG, "comm_init: timeout_ms must be > 0");
    TB_REQUIRE(ctx, !ctx->comm, TB_ERR_ARG, "comm_init: communicator already initialised");
    NcclApi& api = nccl();
    if (!api.ok) return set_error(ctx, TB_ERR_NCCL, "comm_init: libnccl.so.2 not loadable");
    TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
    Comm* c = new Comm();
    c->nranks = nranks;
    c->rank = rank;
    c->timeout_ms = timeout_ms;
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclUniqueId id;
    memcpy(&id, unique_id, sizeof(id));
    ncclResult_t r = api.CommInitRankConfig(&c->comm, nranks, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        delete c;
        return set_error(ctx, TB_ERR_NCCL, "comm_init: %s", api.GetErrorString(r));
    }
    int rc = wait_ready(ctx, c, "comm_init");
    if (rc) {
        delete c;
        return rc;
    }
    ctx->comm = c;
    return TB_OK;
}

int tb_comm_allgather(tb_ctx* ctx, const void* send, void* recv, size_t bytes_per_rank) {
    if (!ctx || !send || !recv) return TB_ERR_ARG;
    Comm* c = reinterpret_cast<Comm*>(ctx->comm);
    TB_REQUIRE(ctx, c && c->comm, TB_ERR_ARG, "allgather: no communicator (tb_comm_init)");
    NcclApi& api = nccl();
    ncclResult_t r = api.AllGather(send, recv, bytes_per_rank, ncclUint8, c->comm, ctx->stream);
    if (r != ncclSuccess && r != ncclInProgress) return set_error(ctx, TB_ERR_NCCL, "allgather: %s", api.GetErrorString(r));
    return wait_ready(ctx, c, "allgather");
}

int tb_comm_abort(tb_ctx* ctx) {
    if (!ctx) return TB_ERR_ARG;
    Comm* c = reinterpret_cast<Comm*>(ctx->comm);
    if (c) {
        if (c->comm) nccl().CommAbort(c->comm);
        delete c;
        ctx->comm = nullptr;
    }
    return TB_OK;
}

int tb_comm_destroy(tb_ctx* ctx) {
    if (!ctx) return TB_ERR_ARG;
    Comm* c = reinterpret_cast<Comm*>(ctx->comm);
    if (c) {
        if (c->comm) nccl().CommDestroy(c->comm);
        delete c;
        ctx->comm = nullptr;
    }
    return TB_OK;
}

}  // extern "C"
