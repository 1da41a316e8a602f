// Multi-GPU groups: NCCL communicators over the contexts' streams.
//
// The reference is single-GPU (one Vulkan device per process; no collective
// anywhere).  Sharded execution needs one exchange primitive, the in-place
// all-reduce of partial results; this file provides it in the two shapes a
// QuasarML host uses:
//   * one process per GPU (qsml_group_init_rank): every rank passes the same
//     unique id (made by one rank with qsml_group_unique_id and shared by the
//     host, e.g. through torch.distributed or a file);
//   * one process driving several GPUs (qsml_group_init_all): one
//     communicator per context, collectives of several ranks issued from one
//     thread between qsml_group_start / qsml_group_end.
// Communicators are created non-blocking and every wait on NCCL is bounded
// (QSML_NCCL_TIMEOUT_MS, default 60 s): a rank that never joins or a
// collective that never completes ends in QSML_E_TIMEOUT and an aborted
// communicator instead of a hung process.  NCCL is opened with dlopen
// ("libnccl.so.2": the copy a framework already loaded, else the system's).
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <thread>
#include <vector>

#include "qsml_internal.cuh"

struct qsml_group {
    std::vector<ncclComm_t> comms;          // one per local rank
    std::vector<qsml::Context*> ctxs;       // the local ranks' contexts
    int nranks = 0;                         // ranks in the whole group
    bool failed = false;                    // an error or timeout left work behind: abort, do not drain
};

namespace qsml {
namespace {

struct Nccl {
    bool ok = false;
    std::string why;
    ncclResult_t (*get_unique_id)(ncclUniqueId*);
    ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*group_start)();
    ncclResult_t (*group_end)();
    ncclResult_t (*destroy)(ncclComm_t);
    ncclResult_t (*abort)(ncclComm_t);
    ncclResult_t (*async_error)(ncclComm_t, ncclResult_t*);
    const char* (*error_string)(ncclResult_t);
};

template <typename F> bool sym(void* lib, const char* name, F* out) {
    *out = reinterpret_cast<F>(dlsym(lib, name));
    return *out != nullptr;
}

const Nccl& nccl() {
    static Nccl n = [] {
        Nccl t;
        void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) {
            t.why = "libnccl.so.2 not found";
            return t;
        }
        t.ok = sym(lib, "ncclGetUniqueId", &t.get_unique_id) && sym(lib, "ncclCommInitRankConfig", &t.init_rank_config) &&
               sym(lib, "ncclAllReduce", &t.all_reduce) && sym(lib, "ncclGroupStart", &t.group_start) &&
               sym(lib, "ncclGroupEnd", &t.group_end) && sym(lib, "ncclCommDestroy", &t.destroy) &&
               sym(lib, "ncclCommAbort", &t.abort) && sym(lib, "ncclCommGetAsyncError", &t.async_error) &&
               sym(lib, "ncclGetErrorString", &t.error_string);
        if (!t.ok) t.why = "libnccl.so.2 lacks an entry point";
        return t;
    }();
    return n;
}

int64_t timeout_ms() {
    static int64_t t = [] {
        const char* s = std::getenv("QSML_NCCL_TIMEOUT_MS");
        return s ? std::max<int64_t>(1, std::atoll(s)) : int64_t(60000);
    }();
    return t;
}

// Thread-local nesting of qsml_group_start / qsml_group_end, and the
// collectives issued inside the current bracket (settled at its end).
thread_local int g_group_depth = 0;
thread_local std::vector<std::pair<qsml_group*, int>> g_bracket;

qsml_status_t nccl_error(Context* ctx, ncclResult_t r, const char* what) {
    return set_error(ctx, QSML_E_NCCL, std::string(what) + ": " + nccl().error_string(r));
}

// Waits (bounded) until every communicator has left ncclInProgress.
qsml_status_t settle(Context* ctx, const std::vector<ncclComm_t>& comms, const char* what) {
    const Nccl& n = nccl();
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        bool pending = false;
        for (ncclComm_t c : comms) {
            ncclResult_t st = ncclSuccess;
            const ncclResult_t r = n.async_error(c, &st);
            if (r != ncclSuccess) return nccl_error(ctx, r, what);
            if (st == ncclInProgress) pending = true;
            else if (st != ncclSuccess) return nccl_error(ctx, st, what);
        }
        if (!pending) return QSML_OK;
        const auto ms =
            std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
        if (ms > timeout_ms())
            return set_error(ctx, QSML_E_TIMEOUT, std::string(what) + ": no progress within QSML_NCCL_TIMEOUT_MS");
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

ncclConfig_t nonblocking_config() {
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    return cfg;
}

void abort_all(std::vector<ncclComm_t>& comms) {
    for (ncclComm_t c : comms)
        if (c) nccl().abort(c);
    comms.clear();
}

bool map_dtype(int32_t dt, ncclDataType_t* out) {
    switch (dt) {
        case QSML_F32: *out = ncclFloat32; return true;
        case QSML_F16: *out = ncclFloat16; return true;
        case QSML_I32: *out = ncclInt32; return true;
        case QSML_U32: *out = ncclUint32; return true;
        case QSML_I8: *out = ncclInt8; return true;
        case QSML_U8: *out = ncclUint8; return true;
    }
    return false;  // NCCL has no 16-bit integer type
}

bool map_op(int32_t op, ncclRedOp_t* out) {
    switch (op) {
        case QSML_RED_SUM: *out = ncclSum; return true;
        case QSML_RED_MEAN: *out = ncclAvg; return true;
        case QSML_RED_MAX: *out = ncclMax; return true;
        case QSML_RED_MIN: *out = ncclMin; return true;
        case QSML_RED_PROD: *out = ncclProd; return true;
    }
    return false;
}

}  // namespace
}  // namespace qsml

using namespace qsml;

extern "C" {

qsml_status_t qsml_group_unique_id(uint8_t* id) {
    if (!id) return set_error(nullptr, QSML_E_INVALID, "qsml_group_unique_id: null id");
    const Nccl& n = nccl();
    if (!n.ok) return set_error(nullptr, QSML_E_NCCL, "qsml_group_unique_id: " + n.why);
    static_assert(sizeof(ncclUniqueId) == QSML_UNIQUE_ID_BYTES, "unique id size");
    ncclUniqueId uid;
    const ncclResult_t r = n.get_unique_id(&uid);
    if (r != ncclSuccess) return nccl_error(nullptr, r, "ncclGetUniqueId");
    std::memcpy(id, &uid, sizeof(uid));
    return QSML_OK;
}

qsml_status_t qsml_group_init_rank(qsml_ctx* handle, const uint8_t* id, int32_t nranks, int32_t rank,
                                   qsml_group** group) {
    QSML_CTX(handle);
    if (!id || !group || nranks < 1 || rank < 0 || rank >= nranks)
        return set_error(C_, QSML_E_INVALID, "qsml_group_init_rank: bad id, rank or group pointer");
    const Nccl& n = nccl();
    if (!n.ok) return set_error(C_, QSML_E_NCCL, "qsml_group_init_rank: " + n.why);
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclConfig_t cfg = nonblocking_config();
    std::vector<ncclComm_t> comms(1, nullptr);
    ncclResult_t r = n.init_rank_config(&comms[0], nranks, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        abort_all(comms);
        return nccl_error(C_, r, "ncclCommInitRankConfig");
    }
    qsml_status_t st = settle(C_, comms, "qsml_group_init_rank");
    if (st != QSML_OK) {
        abort_all(comms);
        return st;
    }
    auto* g = new qsml_group;
    g->comms = comms;
    g->ctxs = {C_};
    g->nranks = nranks;
    *group = g;
    return QSML_OK;
}

qsml_status_t qsml_group_init_all(qsml_ctx* const* handles, int32_t n_ctx, qsml_group** group) {
    if (!handles || !group || n_ctx < 1) return set_error(nullptr, QSML_E_INVALID, "qsml_group_init_all: bad arguments");
    std::vector<Context*> ctxs(n_ctx);
    for (int i = 0; i < n_ctx; ++i) {
        ctxs[i] = reinterpret_cast<Context*>(handles[i]);
        if (!ctxs[i]) return set_error(nullptr, QSML_E_INVALID, "qsml_group_init_all: null context");
    }
    Context* c0 = ctxs[0];
    const Nccl& n = nccl();
    if (!n.ok) return set_error(c0, QSML_E_NCCL, "qsml_group_init_all: " + n.why);
    ncclUniqueId uid;
    ncclResult_t r = n.get_unique_id(&uid);
    if (r != ncclSuccess) return nccl_error(c0, r, "ncclGetUniqueId");
    std::vector<ncclComm_t> comms(n_ctx, nullptr);
    int prev = 0;
    cudaGetDevice(&prev);
    r = n.group_start();
    for (int i = 0; i < n_ctx && r == ncclSuccess; ++i) {
        ncclConfig_t cfg = nonblocking_config();
        cudaSetDevice(ctxs[i]->device);
        r = n.init_rank_config(&comms[i], n_ctx, uid, i, &cfg);
        if (r == ncclInProgress) r = ncclSuccess;
    }
    ncclResult_t re = n.group_end();
    cudaSetDevice(prev);
    if (r == ncclSuccess && re != ncclSuccess && re != ncclInProgress) r = re;
    if (r != ncclSuccess) {
        abort_all(comms);
        return nccl_error(c0, r, "ncclCommInitRankConfig (group)");
    }
    qsml_status_t st = settle(c0, comms, "qsml_group_init_all");
    if (st != QSML_OK) {
        abort_all(comms);
        return st;
    }
    auto* g = new qsml_group;
    g->comms = comms;
    g->ctxs = ctxs;
    g->nranks = n_ctx;
    *group = g;
    return QSML_OK;
}

qsml_status_t qsml_group_size(qsml_group* g, int32_t* nranks, int32_t* local_ranks) {
    if (!g) return set_error(nullptr, QSML_E_INVALID, "qsml_group_size: null group");
    if (nranks) *nranks = g->nranks;
    if (local_ranks) *local_ranks = static_cast<int32_t>(g->comms.size());
    return QSML_OK;
}

qsml_status_t qsml_group_start(void) {
    const Nccl& n = nccl();
    if (!n.ok) return set_error(nullptr, QSML_E_NCCL, "qsml_group_start: " + n.why);
    const ncclResult_t r = n.group_start();
    if (r != ncclSuccess) return nccl_error(nullptr, r, "ncclGroupStart");
    ++g_group_depth;
    return QSML_OK;
}

qsml_status_t qsml_group_end(void) {
    const Nccl& n = nccl();
    if (!n.ok || g_group_depth == 0) return set_error(nullptr, QSML_E_INVALID, "qsml_group_end without qsml_group_start");
    --g_group_depth;
    const ncclResult_t r = n.group_end();
    if (g_group_depth > 0) return r == ncclSuccess || r == ncclInProgress ? QSML_OK : nccl_error(nullptr, r, "ncclGroupEnd");
    std::vector<std::pair<qsml_group*, int>> issued;
    issued.swap(g_bracket);
    qsml_status_t st = QSML_OK;
    if (r != ncclSuccess && r != ncclInProgress) st = nccl_error(nullptr, r, "ncclGroupEnd");
    // The bracket's collectives are enqueued once their communicators settle.
    for (auto& e : issued) {
        if (st != QSML_OK) {
            e.first->failed = true;
            continue;
        }
        st = settle(e.first->ctxs[e.second], {e.first->comms[e.second]}, "qsml_group_end");
        if (st != QSML_OK) e.first->failed = true;
    }
    return st;
}

qsml_status_t qsml_allreduce(qsml_group* g, int32_t local, void* buf, int64_t count, int32_t dtype, int32_t op) {
    if (!g || local < 0 || local >= static_cast<int32_t>(g->comms.size()))
        return set_error(nullptr, QSML_E_INVALID, "qsml_allreduce: bad group or local rank");
    Context* C_ = g->ctxs[local];
    if (cudaSetDevice(C_->device) != cudaSuccess) return set_error(C_, QSML_E_CUDA, "cudaSetDevice failed");
    if (count < 0 || (count > 0 && !buf)) return set_error(C_, QSML_E_INVALID, "qsml_allreduce: bad buffer");
    ncclDataType_t t;
    ncclRedOp_t o;
    if (!map_dtype(dtype, &t)) return set_error(C_, QSML_E_DTYPE, "qsml_allreduce: no NCCL type for this dtype");
    if (!map_op(op, &o)) return set_error(C_, QSML_E_INVALID, "qsml_allreduce: unknown op");
    const ncclResult_t r =
        nccl().all_reduce(buf, buf, static_cast<size_t>(count), t, o, g->comms[local], C_->stream);
    if (r != ncclSuccess && r != ncclInProgress) {
        g->failed = true;
        return nccl_error(C_, r, "ncclAllReduce");
    }
    // Outside a start/end bracket the call is enqueued once the communicator
    // settles; inside one, qsml_group_end settles it.
    if (g_group_depth > 0) {
        g_bracket.emplace_back(g, local);
        return QSML_OK;
    }
    const qsml_status_t st = settle(C_, {g->comms[local]}, "qsml_allreduce");
    if (st != QSML_OK) g->failed = true;
    return st;
}

qsml_status_t qsml_group_destroy(qsml_group* g) {
    if (!g) return QSML_OK;
    const Nccl& n = nccl();
    qsml_status_t st = QSML_OK;
    for (size_t i = 0; i < g->comms.size(); ++i) {
        cudaSetDevice(g->ctxs[i]->device);
        if (g->failed) {
            // work may never complete: abort it rather than wait for it
            n.abort(g->comms[i]);
            continue;
        }
        cudaStreamSynchronize(g->ctxs[i]->stream);
        if (n.destroy(g->comms[i]) != ncclSuccess) st = QSML_E_NCCL;
    }
    delete g;
    return st;
}

}  // extern "C"
