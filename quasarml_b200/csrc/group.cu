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
// Key decodings of max/min partials combined inside the current bracket:
// they follow the collective, which NCCL enqueues at the bracket's end.
struct PendingDecode {
    Context* ctx;
    void* buf;
    int64_t count;
    int32_t op;
};
thread_local std::vector<PendingDecode> g_decodes;

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
        // A collective is normally enqueued within microseconds: poll without
        // sleeping for the first 2 ms (sleeping would stall the host's launch
        // stream), then back off.
        if (ms < 2)
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

// QSML_NCCL_MAX_CTAS caps the CTAs (channels) each collective of the group
// may occupy: combines that overlap memory-bound kernels take SMs from them.
ncclConfig_t nonblocking_config() {
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    if (const char* s = std::getenv("QSML_NCCL_MAX_CTAS")) {
        const int v = std::atoi(s);
        if (v > 0) {
            cfg.maxCTAs = v;
            cfg.minCTAs = 1;
        }
    }
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

// Max/min partials cross the group as order-preserving unsigned keys, so the
// exchange (an integer max/min) gives exactly what qsml_reduce's max.NaN /
// min.NaN give on one GPU: -0 below +0, and any NaN wins (NaN maps to the
// largest key for max and the smallest for min; it decodes to 0x7fffffff).
// A float max/min in the collective would let a NaN or the sign of zero
// depend on the order of ranks.
__device__ __forceinline__ uint32_t key_of(uint32_t u, bool is_max) {
    if ((u & 0x7fffffffu) > 0x7f800000u) return is_max ? 0xffffffffu : 0u;  // NaN
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ uint32_t value_of(uint32_t k, bool is_max) {
    if (k == (is_max ? 0xffffffffu : 0u)) return 0x7fffffffu;
    return (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
}

__global__ void k_partial_keys(uint32_t* p, int64_t n, int is_max, int decode) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        p[i] = decode ? value_of(p[i], is_max != 0) : key_of(p[i], is_max != 0);
}

// out = partial (times scale for a mean), rounded once to out's dtype.
template <typename OT>
__global__ void k_partial_finish(const float* p, OT* out, int64_t n, float scale, int mul) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float v = mul ? __fmul_rn(p[i], scale) : p[i];
        if constexpr (sizeof(OT) == 2) out[i] = __float2half_rn(v);
        else out[i] = v;
    }
}

unsigned grid_for(const Context* ctx, int64_t n) {
    int64_t g = (n + 255) / 256;
    const int64_t cap = static_cast<int64_t>(ctx->num_sms) * 8;
    if (g > cap) g = cap;
    return static_cast<unsigned>(g < 1 ? 1 : g);
}

qsml_status_t keys_pass(Context* ctx, void* buf, int64_t n, int32_t op, bool decode) {
    if (n == 0) return QSML_OK;
    k_partial_keys<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(static_cast<uint32_t*>(buf), n,
                                                              op == QSML_RED_MAX ? 1 : 0, decode ? 1 : 0);
    return after_launch(ctx, "k_partial_keys");
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
    std::vector<PendingDecode> decodes;
    decodes.swap(g_decodes);
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
    // then the key decodings, in stream order after their collectives
    for (auto& d : decodes) {
        if (st != QSML_OK) break;
        if (cudaSetDevice(d.ctx->device) != cudaSuccess) {
            st = set_error(d.ctx, QSML_E_CUDA, "cudaSetDevice failed");
            break;
        }
        st = keys_pass(d.ctx, d.buf, d.count, d.op, true);
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
    // NCCL's kernel is not one of the library's: the next library kernel on the
    // stream waits for it at its start (no overlap across a collective)
    end_window(C_->stream);
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

qsml_status_t qsml_allreduce_partials(qsml_group* g, int32_t local, int32_t op, void* buf, int64_t count) {
    if (!g || local < 0 || local >= static_cast<int32_t>(g->comms.size()))
        return set_error(nullptr, QSML_E_INVALID, "qsml_allreduce_partials: bad group or local rank");
    Context* C_ = g->ctxs[local];
    if (cudaSetDevice(C_->device) != cudaSuccess) return set_error(C_, QSML_E_CUDA, "cudaSetDevice failed");
    if (op < QSML_RED_SUM || op > QSML_RED_MIN) return set_error(C_, QSML_E_INVALID, "qsml_allreduce_partials: unknown op");
    if (count < 0 || (count > 0 && !buf)) return set_error(C_, QSML_E_INVALID, "qsml_allreduce_partials: bad buffer");
    if (count == 0) return QSML_OK;
    const bool keys = op == QSML_RED_MAX || op == QSML_RED_MIN;
    if (keys) QSML_TRY_STATUS(keys_pass(C_, buf, count, op, false));
    const ncclResult_t r = nccl().all_reduce(buf, buf, static_cast<size_t>(count), keys ? ncclUint32 : ncclFloat32,
                                             op == QSML_RED_MAX ? ncclMax : op == QSML_RED_MIN ? ncclMin : ncclSum,
                                             g->comms[local], C_->stream);
    end_window(C_->stream);  // the next library kernel waits for the collective
    if (r != ncclSuccess && r != ncclInProgress) {
        g->failed = true;
        return nccl_error(C_, r, "ncclAllReduce (partials)");
    }
    if (g_group_depth > 0) {
        // inside a bracket: qsml_group_end settles the collective, then decodes
        g_bracket.emplace_back(g, local);
        if (keys) g_decodes.push_back(PendingDecode{C_, buf, count, op});
        return QSML_OK;
    }
    qsml_status_t st = settle(C_, {g->comms[local]}, "qsml_allreduce_partials");
    if (st != QSML_OK) {
        g->failed = true;
        return st;
    }
    if (keys) QSML_TRY_STATUS(keys_pass(C_, buf, count, op, true));
    return QSML_OK;
}

qsml_status_t qsml_finish_partial(qsml_ctx* handle, int32_t op, const qsml_tdesc* partial, int64_t n,
                                  const qsml_tdesc* out) {
    QSML_CTX(handle);
    QSML_TRY_STATUS(check_desc(C_, partial, "partial"));
    QSML_TRY_STATUS(check_desc(C_, out, "out"));
    if (op < QSML_RED_SUM || op > QSML_RED_MIN) return set_error(C_, QSML_E_INVALID, "qsml_finish_partial: unknown op");
    if (partial->dtype != QSML_F32) return set_error(C_, QSML_E_DTYPE, "qsml_finish_partial: partial must be F32");
    if (out->dtype != QSML_F32 && out->dtype != QSML_F16)
        return set_error(C_, QSML_E_DTYPE, "qsml_finish_partial: out must be F32 or F16");
    if (!is_contiguous(partial) || !is_contiguous(out) || numel(partial) != numel(out))
        return set_error(C_, QSML_E_SHAPE, "qsml_finish_partial: partial and out must be contiguous and equally long");
    if (op == QSML_RED_MEAN && n < 1) return set_error(C_, QSML_E_INVALID, "qsml_finish_partial: mean needs n >= 1");
    const int64_t count = numel(out);
    const bool mul = op == QSML_RED_MEAN;
    if (count == 0 || (!mul && out->dtype == QSML_F32 && out->data == partial->data)) return QSML_OK;
    // the reference's mean: sum * (1.0f / (float)n) (Ops/Reduction.cpp:347-356)
    const float scale = mul ? 1.0f / static_cast<float>(n) : 1.0f;
    const float* p = static_cast<const float*>(partial->data);
    if (out->dtype == QSML_F32)
        k_partial_finish<float><<<grid_for(C_, count), 256, 0, C_->stream>>>(p, static_cast<float*>(out->data), count,
                                                                           scale, mul ? 1 : 0);
    else
        k_partial_finish<__half><<<grid_for(C_, count), 256, 0, C_->stream>>>(p, static_cast<__half*>(out->data),
                                                                             count, scale, mul ? 1 : 0);
    return after_launch(C_, "k_partial_finish");
}

qsml_status_t qsml_reduce_sharded(qsml_group* g, int32_t local, int32_t op, const qsml_tdesc* a, int32_t axis,
                                  int32_t keepdims, const qsml_tdesc* out, int64_t global_rows) {
    if (!g || local < 0 || local >= static_cast<int32_t>(g->comms.size()))
        return set_error(nullptr, QSML_E_INVALID, "qsml_reduce_sharded: bad group or local rank");
    Context* C_ = g->ctxs[local];
    qsml_ctx* h = reinterpret_cast<qsml_ctx*>(C_);
    if (g_group_depth > 0)
        return set_error(C_, QSML_E_INVALID,
                         "qsml_reduce_sharded: not inside qsml_group_start/end (it finishes right after its combine)");
    QSML_TRY_STATUS(check_desc(C_, a, "a"));
    QSML_TRY_STATUS(check_desc(C_, out, "out"));
    if (op < QSML_RED_SUM || op > QSML_RED_MIN) return set_error(C_, QSML_E_INVALID, "qsml_reduce_sharded: unknown op");
    if (a->ndim < 1) return set_error(C_, QSML_E_SHAPE, "qsml_reduce_sharded: a needs a row axis");
    const int ax = axis == QSML_AXIS_ALL ? QSML_AXIS_ALL : (axis < 0 ? axis + a->ndim : axis);
    // Any axis but the row axis: this rank's rows of the result, no exchange.
    if (ax != 0 && ax != QSML_AXIS_ALL) return qsml_reduce(h, op, a, axis, keepdims, out);
    if (global_rows == 0) global_rows = a->shape[0] * g->nranks;
    if (global_rows < a->shape[0]) return set_error(C_, QSML_E_SHAPE, "qsml_reduce_sharded: global_rows below this rank's rows");
    int64_t row_elems = 1;
    for (int i = 1; i < a->ndim; ++i) row_elems *= a->shape[i];
    const int64_t n = ax == 0 ? global_rows : global_rows * row_elems;
    const int64_t count = numel(out);
    // the partial: out itself when it is binary32, else scratch
    void* pbuf = out->data;
    const bool scratch = out->dtype != QSML_F32;
    if (scratch) {
        std::string err;
        qsml_status_t st = C_->allocator->alloc(static_cast<size_t>(count) * 4, &pbuf, &err);
        if (st != QSML_OK) return set_error(C_, st, "qsml_reduce_sharded: " + err);
    }
    qsml_tdesc pd = *out;
    pd.data = pbuf;
    pd.dtype = QSML_F32;
    qsml_status_t st = QSML_OK;
    if (a->shape[0] == 0 && (op == QSML_RED_MAX || op == QSML_RED_MIN)) {
        // no rows here: the identity of max / min
        const float v = op == QSML_RED_MAX ? -INFINITY : INFINITY;
        st = qsml_fill(h, pbuf, &v, 4, count);
    } else {
        st = qsml_reduce(h, op == QSML_RED_MEAN ? QSML_RED_SUM : op, a, axis, keepdims, &pd);
    }
    if (st == QSML_OK) st = qsml_allreduce_partials(g, local, op, pbuf, count);
    if (st == QSML_OK) st = qsml_finish_partial(h, op, &pd, n, out);
    if (scratch) {
        std::string err;
        C_->allocator->free(pbuf, &err);  // reused in stream order
    }
    return st;
}

qsml_status_t qsml_shard_rows(int64_t rows, int32_t nranks, int32_t rank, int64_t* begin, int64_t* count) {
    if (rows < 0 || nranks < 1 || rank < 0 || rank >= nranks || !begin || !count)
        return set_error(nullptr, QSML_E_INVALID, "qsml_shard_rows: bad arguments");
    const int64_t base = rows / nranks, extra = rows % nranks;
    *count = base + (rank < extra ? 1 : 0);
    *begin = rank * base + (rank < extra ? rank : extra);
    return QSML_OK;
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
