// group.cu -- multi-GPU group: NCCL communicators over the GPUs of one node and the gather of
// per-GPU results (detections, logits) to rank 0.
//
// Inference shards by image: every GPU runs the whole network on its slice of the batch and no
// data crosses NVLink inside the network.  The one exchange is the final gather to rank 0
// (the reference has none: TNNet runs on one device, source/nConvolutionLayer.pas:472 marks
// multi-GPU as future work).  Two ways to form a group:
//   * tb_group_init: one process drives every GPU (a context per GPU, ncclCommInitAll);
//   * tb_group_init_rank: one process per GPU (torchrun-style); the caller moves the unique id
//     from rank 0 to the others.  Initialisation is non-blocking with a deadline: a rank that
//     never joins makes every waiting rank return TB_ERR_TIMEOUT after ncclCommAbort instead of
//     hanging.
// NCCL is loaded with dlopen on first use (libnccl.so.2), so the library has no link-time NCCL
// dependency; every wait on NCCL or on the streams it uses is bounded.
#include "common.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <mutex>
#include <thread>
#include <vector>

namespace {

// Types and the config initializer come from nccl.h (compile time only); the functions are
// resolved from libnccl.so.2 at run time.
constexpr ncclResult_t kNcclSuccess = ncclSuccess, kNcclInProgress = ncclInProgress;
constexpr ncclDataType_t kNcclUint8 = ncclUint8;
typedef ncclUniqueId NcclUniqueId;
typedef ncclConfig_t NcclConfig;

struct NcclApi {
    void* handle = nullptr;
    ncclResult_t (*getUniqueId)(NcclUniqueId*) = nullptr;
    ncclResult_t (*commInitAll)(ncclComm_t*, int, const int*) = nullptr;
    ncclResult_t (*commInitRankConfig)(ncclComm_t*, int, NcclUniqueId, int, NcclConfig*) = nullptr;
    ncclResult_t (*commGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*commAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*groupStart)() = nullptr;
    ncclResult_t (*groupEnd)() = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*getErrorString)(ncclResult_t) = nullptr;
    ncclResult_t (*getVersion)(int*) = nullptr;
};

std::mutex g_api_mu;
NcclApi g_api;
bool g_api_tried = false;

const NcclApi* nccl() {
    std::lock_guard<std::mutex> lk(g_api_mu);
    if (g_api_tried) return g_api.handle ? &g_api : nullptr;
    g_api_tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return nullptr;
    NcclApi a;
    a.handle = h;
#define TB_SYM(field, name) a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, name))
    TB_SYM(getUniqueId, "ncclGetUniqueId");
    TB_SYM(commInitAll, "ncclCommInitAll");
    TB_SYM(commInitRankConfig, "ncclCommInitRankConfig");
    TB_SYM(commGetAsyncError, "ncclCommGetAsyncError");
    TB_SYM(commAbort, "ncclCommAbort");
    TB_SYM(commDestroy, "ncclCommDestroy");
    TB_SYM(groupStart, "ncclGroupStart");
    TB_SYM(groupEnd, "ncclGroupEnd");
    TB_SYM(send, "ncclSend");
    TB_SYM(recv, "ncclRecv");
    TB_SYM(getErrorString, "ncclGetErrorString");
    TB_SYM(getVersion, "ncclGetVersion");
#undef TB_SYM
    if (!a.getUniqueId || !a.commInitAll || !a.commInitRankConfig || !a.commGetAsyncError || !a.commAbort ||
        !a.commDestroy || !a.groupStart || !a.groupEnd || !a.send || !a.recv || !a.getErrorString) {
        dlclose(h);
        return nullptr;
    }
    g_api = a;
    return &g_api;
}

int nccl_fail(const NcclApi* api, ncclResult_t r, const char* what) {
    return tbi::fail(TB_ERR_CUDA, "%s: NCCL error %d (%s)", what, r, api->getErrorString ? api->getErrorString(r) : "?");
}

double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

}  // namespace

struct tb_group {
    int nranks = 0;             // ranks of the whole group
    int first_rank = 0;         // global rank of this process's first local GPU
    std::vector<tb_ctx*> ctxs;  // one per local GPU
    std::vector<ncclComm_t> comms;
    bool own_ctxs = false;
    double timeout_s = 30.0;
    bool broken = false;        // a wait ran out and the communicators were aborted
};

namespace {

void abort_all(tb_group* g) {
    const NcclApi* api = nccl();
    for (auto& c : g->comms)
        if (c && api) api->commAbort(c);
    for (auto& c : g->comms) c = nullptr;
    g->broken = true;
}

// Wait until every local communicator has left ncclInProgress (non-blocking communicators) and
// every local stream has drained, or the group's deadline passes (then abort).
int wait_group(tb_group* g, bool streams, const char* what) {
    const NcclApi* api = nccl();
    const double deadline = now_s() + g->timeout_s;
    for (;;) {
        bool pending = false;
        for (size_t i = 0; i < g->comms.size(); ++i) {
            ncclResult_t st = kNcclSuccess;
            ncclResult_t r = api->commGetAsyncError(g->comms[i], &st);
            if (r != kNcclSuccess) return nccl_fail(api, r, what);
            if (st == kNcclInProgress) { pending = true; continue; }
            if (st != kNcclSuccess) {
                int rc = nccl_fail(api, st, what);
                abort_all(g);
                return rc;
            }
            if (streams) {
                cudaSetDevice(g->ctxs[i]->device);
                cudaError_t e = cudaStreamQuery(g->ctxs[i]->stream);
                if (e == cudaErrorNotReady) pending = true;
                else if (e != cudaSuccess) return tbi::cuda_fail(e, what);
            }
        }
        if (!pending) return TB_OK;
        if (now_s() > deadline) {
            abort_all(g);
            return tbi::fail(TB_ERR_TIMEOUT, "%s: no progress within %.1f s (a rank did not take part); the "
                             "group's communicators were aborted", what, g->timeout_s);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace

using namespace tbi;

extern "C" {

int tb_group_available(int64_t* nccl_version) {
    const NcclApi* api = nccl();
    if (!api) return fail(TB_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
    int v = 0;
    if (api->getVersion) api->getVersion(&v);
    if (nccl_version) *nccl_version = v;
    return TB_OK;
}

int tb_group_init(int64_t ngpu, const int64_t* devices, tb_group** out) {
    if (!out || ngpu <= 0 || !devices) return fail(TB_ERR_INVALID, "tb_group_init: bad arguments");
    *out = nullptr;
    const NcclApi* api = nccl();
    if (!api) return fail(TB_ERR_UNSUPPORTED, "tb_group_init: libnccl.so.2 could not be loaded");
    tb_group* g = new tb_group();
    g->nranks = (int)ngpu;
    g->own_ctxs = true;
    std::vector<int> devs((size_t)ngpu);
    for (int64_t i = 0; i < ngpu; ++i) {
        devs[(size_t)i] = (int)devices[i];
        tb_ctx* c = nullptr;
        int r = tb_init(devices[i], nullptr, &c);
        if (r != TB_OK) {
            for (auto* x : g->ctxs) tb_shutdown(x);
            delete g;
            return r;
        }
        g->ctxs.push_back(c);
    }
    g->comms.assign((size_t)ngpu, nullptr);
    ncclResult_t r = api->commInitAll(g->comms.data(), (int)ngpu, devs.data());
    if (r != kNcclSuccess) {
        int rc = nccl_fail(api, r, "ncclCommInitAll");
        for (auto* x : g->ctxs) tb_shutdown(x);
        delete g;
        return rc;
    }
    *out = g;
    return TB_OK;
}

int tb_group_unique_id(void* id_out) {
    if (!id_out) return fail(TB_ERR_INVALID, "tb_group_unique_id: null output");
    const NcclApi* api = nccl();
    if (!api) return fail(TB_ERR_UNSUPPORTED, "tb_group_unique_id: libnccl.so.2 could not be loaded");
    NcclUniqueId id;
    ncclResult_t r = api->getUniqueId(&id);
    if (r != kNcclSuccess) return nccl_fail(api, r, "ncclGetUniqueId");
    memcpy(id_out, &id, sizeof(id));
    return TB_OK;
}

int tb_group_init_rank(tb_ctx* ctx, int64_t nranks, int64_t rank, const void* id, int64_t timeout_ms,
                       tb_group** out) {
    TB_ENTER(ctx);
    if (!out || !id || nranks <= 0 || rank < 0 || rank >= nranks || timeout_ms <= 0)
        return fail(TB_ERR_INVALID, "tb_group_init_rank: bad arguments");
    *out = nullptr;
    const NcclApi* api = nccl();
    if (!api) return fail(TB_ERR_UNSUPPORTED, "tb_group_init_rank: libnccl.so.2 could not be loaded");
    tb_group* g = new tb_group();
    g->nranks = (int)nranks;
    g->first_rank = (int)rank;
    g->ctxs.push_back(ctx);
    g->comms.assign(1, nullptr);
    g->timeout_s = (double)timeout_ms / 1000.0;
    NcclConfig cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // non-blocking: the waits below carry the deadline
    NcclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    ncclResult_t r = api->commInitRankConfig(&g->comms[0], (int)nranks, uid, (int)rank, &cfg);
    if (r != kNcclSuccess && r != kNcclInProgress) {
        int rc = nccl_fail(api, r, "ncclCommInitRankConfig");
        delete g;
        return rc;
    }
    int rc = wait_group(g, false, "tb_group_init_rank");
    if (rc != TB_OK) {
        delete g;
        return rc;
    }
    *out = g;
    return TB_OK;
}

int tb_group_size(tb_group* g, int64_t* nranks, int64_t* first_local_rank, int64_t* local_gpus) {
    if (!g) return fail(TB_ERR_INVALID, "null group");
    if (nranks) *nranks = g->nranks;
    if (first_local_rank) *first_local_rank = g->first_rank;
    if (local_gpus) *local_gpus = (int64_t)g->ctxs.size();
    return TB_OK;
}

int tb_group_context(tb_group* g, int64_t local, tb_ctx** ctx) {
    if (!g || !ctx || local < 0 || local >= (int64_t)g->ctxs.size())
        return fail(TB_ERR_INVALID, "tb_group_context: bad arguments");
    *ctx = g->ctxs[(size_t)local];
    return TB_OK;
}

int tb_group_gather_async(tb_group* g, const void* const* send_local, const int64_t* bytes_per_rank,
                          void* recv_root) {
    if (!g || !send_local || !bytes_per_rank) return fail(TB_ERR_INVALID, "tb_group_gather: bad arguments");
    if (g->broken) return fail(TB_ERR_STATE, "tb_group_gather: the group was aborted after a timeout");
    const NcclApi* api = nccl();
    std::vector<int64_t> off((size_t)g->nranks + 1, 0);
    for (int r = 0; r < g->nranks; ++r) {
        if (bytes_per_rank[r] < 0) return fail(TB_ERR_INVALID, "tb_group_gather: negative size");
        off[(size_t)r + 1] = off[(size_t)r] + bytes_per_rank[r];
    }
    const bool has_root = g->first_rank == 0;
    if (has_root && !recv_root && off[(size_t)g->nranks] > 0)
        return fail(TB_ERR_INVALID, "tb_group_gather: rank 0 needs a receive buffer");
    char* dst = static_cast<char*>(recv_root);
    ncclResult_t r = api->groupStart();
    if (r != kNcclSuccess) return nccl_fail(api, r, "ncclGroupStart");
    int rc = TB_OK;
    for (size_t i = 0; i < g->ctxs.size() && rc == TB_OK; ++i) {
        const int me = g->first_rank + (int)i;
        tb_ctx* c = g->ctxs[i];
        const size_t n = (size_t)bytes_per_rank[me];
        if (me == 0) {  // the root: its own slice by a device copy, then one receive per other rank
            cudaSetDevice(c->device);
            if (n && cudaMemcpyAsync(dst, send_local[i], n, cudaMemcpyDeviceToDevice, c->stream) != cudaSuccess)
                rc = fail(TB_ERR_CUDA, "tb_group_gather: root copy failed");
            for (int q = 1; q < g->nranks && rc == TB_OK; ++q) {
                if (!bytes_per_rank[q]) continue;
                r = api->recv(dst + off[(size_t)q], (size_t)bytes_per_rank[q], kNcclUint8, q, g->comms[i], c->stream);
                if (r != kNcclSuccess && r != kNcclInProgress) rc = nccl_fail(api, r, "ncclRecv");
            }
        } else if (n) {
            r = api->send(send_local[i], n, kNcclUint8, 0, g->comms[i], c->stream);
            if (r != kNcclSuccess && r != kNcclInProgress) rc = nccl_fail(api, r, "ncclSend");
        }
    }
    r = api->groupEnd();
    if (rc != TB_OK) return rc;
    if (r != kNcclSuccess && r != kNcclInProgress) return nccl_fail(api, r, "ncclGroupEnd");
    return wait_group(g, false, "tb_group_gather");  // enqueued (non-blocking communicators)
}

int tb_group_wait(tb_group* g) {
    if (!g) return fail(TB_ERR_INVALID, "null group");
    if (g->broken) return fail(TB_ERR_STATE, "tb_group_wait: the group was aborted after a timeout");
    return wait_group(g, true, "tb_group_wait");
}

int tb_group_gather(tb_group* g, const void* const* send_local, const int64_t* bytes_per_rank, void* recv_root) {
    int r = tb_group_gather_async(g, send_local, bytes_per_rank, recv_root);
    return r != TB_OK ? r : tb_group_wait(g);
}

int tb_group_destroy(tb_group* g) {
    if (!g) return TB_OK;
    const NcclApi* api = nccl();
    for (auto& c : g->comms)
        if (c && api) api->commDestroy(c);
    if (g->own_ctxs)
        for (auto* c : g->ctxs) tb_shutdown(c);
    delete g;
    return TB_OK;
}

}  // extern "C"
