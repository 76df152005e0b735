// fer_comm_* / fer_transformer_broadcast_weights / fer_transformer_shard /
// fer_buffer_row_digests: the host side of the batch-sharded forward over the
// GPUs of one node, one process (or host thread) per GPU, each with its own
// session.
//
// The reference copies a tensor to the other GPUs with a serial
// cudaMemcpyPeer from the source device to each destination, all devices in
// one process (native/core/runtime/modules/hot_multi_gpu_policy_main.inl:221-249,
// gpu_broadcast_tensor). Here each rank owns its GPU; the weights made on the
// root rank reach every rank's weight buffer, in place, by one NCCL broadcast
// over NVLink / NVSwitch on the session stream. Nothing else crosses GPUs: a
// forward runs its rank's contiguous shard of the sequences with no
// collective, and per-sequence digests of the logits let ranks and runs with
// different GPU counts be compared bit for bit.
//
// NCCL is opened at the first fer_comm_* call (FERCUDA_NCCL_LIBRARY, else
// libnccl.so.2, which is the copy already loaded when the process has one),
// so a program that never shards needs no NCCL. Every wait is bounded: the
// communicator is made non-blocking and polled, and a broadcast that does not
// finish within the session's timeout aborts the communicator and returns an
// error instead of hanging the caller.
#include "session.hpp"

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>

extern "C" cudaError_t fer_row_digests(const void* data, uint64_t row_bytes, uint32_t rows, uint64_t* out,
                                       cudaStream_t s);

namespace fer::capi {

namespace {

struct Nccl {
    void* lib = nullptr;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
    ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
    ncclResult_t (*broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*abort)(ncclComm_t) = nullptr;
    ncclResult_t (*finalize)(ncclComm_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

std::mutex g_nccl_mu;
Nccl g_nccl;

template <class F>
bool sym(void* lib, const char* name, F* out) {
    *out = reinterpret_cast<F>(dlsym(lib, name));
    return *out != nullptr;
}

const Nccl* nccl() {
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (g_nccl.ok) return &g_nccl;
    if (!g_nccl.lib) {
        const char* path = std::getenv("FERCUDA_NCCL_LIBRARY");
        g_nccl.lib = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!g_nccl.lib) return nullptr;
    }
    Nccl& n = g_nccl;
    n.ok = sym(n.lib, "ncclGetUniqueId", &n.get_unique_id) && sym(n.lib, "ncclCommInitRankConfig", &n.init_rank_config) &&
           sym(n.lib, "ncclCommGetAsyncError", &n.get_async_error) && sym(n.lib, "ncclBroadcast", &n.broadcast) &&
           sym(n.lib, "ncclCommDestroy", &n.destroy) && sym(n.lib, "ncclCommAbort", &n.abort) &&
           sym(n.lib, "ncclCommFinalize", &n.finalize) && sym(n.lib, "ncclGetErrorString", &n.error_string);
    return n.ok ? &g_nccl : nullptr;
}

using Clock = std::chrono::steady_clock;

// Polls the communicator until its pending operation leaves ncclInProgress
// or the deadline passes (ncclInProgress is then returned).
ncclResult_t settle(const Nccl* n, ncclComm_t c, Clock::time_point deadline) {
    ncclResult_t st = ncclInProgress;
    while (true) {
        if (n->get_async_error(c, &st) != ncclSuccess) return ncclInternalError;
        if (st != ncclInProgress || Clock::now() > deadline) return st;
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace

struct CommState {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    uint32_t timeout_ms = 0;
};

void comm_release(CommState* c) {
    if (!c) return;
    const Nccl* n = nccl();
    if (n && c->comm) {
        // finalize flushes outstanding work; abort if it does not settle in time
        const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
        ncclResult_t st = n->finalize(c->comm);
        if (st == ncclSuccess || st == ncclInProgress) st = settle(n, c->comm, deadline);
        if (st == ncclSuccess) n->destroy(c->comm);
        else n->abort(c->comm);
    }
    delete c;
}

}  // namespace fer::capi

using namespace fer::capi;

extern "C" {

fer_status_t fer_comm_unique_id(uint8_t* out_id) {
    if (!out_id) return invalid("out_id is null");
    static_assert(sizeof(ncclUniqueId) == FER_COMM_UNIQUE_ID_BYTES, "NCCL unique id size");
    const Nccl* n = nccl();
    if (!n) return internal("NCCL library not available");
    ncclUniqueId id;
    if (n->get_unique_id(&id) != ncclSuccess) return internal("ncclGetUniqueId failed");
    std::memcpy(out_id, &id, sizeof(id));
    return ok();
}

fer_status_t fer_comm_init(fer_session_t* session, const uint8_t* id, int32_t rank, int32_t world,
                           uint32_t timeout_ms) {
    if (!session || !id) return invalid("session or id is null");
    if (world < 1 || rank < 0 || rank >= world) return invalid("rank outside world");
    Session& S = session->impl;
    if (S.comm) return invalid("session already has a communicator");
    const Nccl* n = nccl();
    if (!n) return internal("NCCL library not available");
    if (cudaSetDevice(S.device) != cudaSuccess) return internal("cudaSetDevice failed");
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    auto* c = new CommState;
    c->rank = rank;
    c->world = world;
    c->timeout_ms = timeout_ms ? timeout_ms : 120000u;
    const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
    ncclResult_t st = n->init_rank_config(&c->comm, world, uid, rank, &cfg);
    if ((st == ncclSuccess || st == ncclInProgress) && c->comm) st = settle(n, c->comm, deadline);
    if (st != ncclSuccess) {
        if (c->comm) n->abort(c->comm);
        delete c;
        return internal(st == ncclInProgress ? "communicator init timed out (a rank did not join)"
                                             : "ncclCommInitRankConfig failed");
    }
    S.comm = c;
    return ok();
}

fer_status_t fer_comm_destroy(fer_session_t* session) {
    if (!session) return invalid("session is null");
    Session& S = session->impl;
    if (!S.comm) return not_found("session has no communicator");
    comm_release(S.comm);
    S.comm = nullptr;
    return ok();
}

fer_status_t fer_transformer_broadcast_weights(fer_session_t* session, uint64_t model, int32_t root,
                                               uint64_t* out_bytes) {
    if (!session) return invalid("session is null");
    Session& S = session->impl;
    if (!S.comm) return invalid("session has no communicator (fer_comm_init)");
    CommState* c = S.comm;
    if (root < 0 || root >= c->world) return invalid("root outside world");
    uint64_t wid = 0;
    fer_status_t st = fer_transformer_weight_buffer(session, model, &wid);
    if (st.code) return st;
    const Buffer* w = S.find(wid);
    if (!w) return not_found("weight buffer not found");
    const Nccl* n = nccl();
    const auto deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
    // in place on every rank (send == receive buffer), after the work queued so far
    ncclResult_t r = n->broadcast(w->ptr, w->ptr, w->bytes, ncclUint8, root, c->comm, S.stream);
    if (r == ncclInProgress) r = settle(n, c->comm, deadline);
    if (r != ncclSuccess) return internal("ncclBroadcast failed");
    // bounded wait for completion on the session stream
    while (true) {
        const cudaError_t q = cudaStreamQuery(S.stream);
        if (q == cudaSuccess) break;
        if (q != cudaErrorNotReady) return internal("stream error during the weight broadcast");
        ncclResult_t async = ncclSuccess;
        if (n->get_async_error(c->comm, &async) != ncclSuccess || (async != ncclSuccess && async != ncclInProgress)) {
            n->abort(c->comm);
            c->comm = nullptr;
            return internal("communicator failed during the weight broadcast (aborted)");
        }
        if (Clock::now() > deadline) {
            n->abort(c->comm);
            c->comm = nullptr;
            return internal("weight broadcast timed out (communicator aborted)");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
    if (out_bytes) *out_bytes = w->bytes;
    return ok();
}

fer_status_t fer_transformer_shard(uint32_t global_batch, int32_t world, int32_t rank, uint32_t* out_first,
                                   uint32_t* out_count) {
    if (!out_first || !out_count) return invalid("out_first or out_count is null");
    if (world < 1 || rank < 0 || rank >= world) return invalid("rank outside world");
    if (global_batch % static_cast<uint32_t>(world)) return invalid("global batch does not split evenly over the ranks");
    const uint32_t per = global_batch / static_cast<uint32_t>(world);
    *out_first = per * static_cast<uint32_t>(rank);
    *out_count = per;
    return ok();
}

fer_status_t fer_buffer_row_digests(fer_session_t* session, uint64_t buffer, uint64_t row_bytes, uint32_t rows,
                                    uint64_t* out_digests) {
    if (!session || !out_digests) return invalid("session or out_digests is null");
    Session& S = session->impl;
    const Buffer* b = S.find(buffer);
    if (!b) return not_found("buffer id not found");
    if (rows == 0 || row_bytes == 0 || row_bytes % 16) return invalid("row_bytes must be a nonzero multiple of 16");
    if (rows > 65535u) return invalid("at most 65535 rows per call");
    if (row_bytes * rows > b->bytes) return invalid("rows x row_bytes exceeds the buffer");
    if (reinterpret_cast<uintptr_t>(b->ptr) % 16) return invalid("buffer is not 16-byte aligned");
    void* dev = nullptr;
    Temp t{};
    fer_status_t st = S.alloc_temp(static_cast<size_t>(rows) * 8, FER_MEMORY_AUTO, &t);
    if (st.code) return st;
    dev = t.ptr;
    cudaError_t e = fer_row_digests(b->ptr, row_bytes, rows, static_cast<uint64_t*>(dev), S.stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(out_digests, dev, static_cast<size_t>(rows) * 8, cudaMemcpyDeviceToHost, S.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(S.stream);
    S.free_bytes(t.ptr, t.regime, t.tier, t.bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return internal("digest kernel failed");
    }
    return ok();
}

}  // extern "C"
