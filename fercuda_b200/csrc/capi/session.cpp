// Session, regime, buffer, stream and job entry points of the C ABI.
//
// Reference behaviour kept (file:line in the reference):
//   fer_session_create      c_api.cu:140-154, session.cu:62-87 (pool = mutable+immutable, >= 64 MiB)
//   regimes                 regime_manager.cu:15-123 (ids <= 2 builtin, AUTO = default)
//   alloc / import / free   session.cu:132-227 (ids from 1, rank 1..4, nonzero size)
//   upload / download       session.cu:229-272 (exact byte size required)
//   jobs                    job_manager.cu:23-92 (event per job, temps freed when observed done)
// Deliberate differences:
//   - download copies on the session stream and then synchronises it (the
//     reference's blocking cudaMemcpy runs on the legacy stream, which a
//     non-blocking session stream does not order against);
//   - job events come from a recycled pool and are released once a job is
//     observed complete (the reference keeps one live event per job forever).
#include "session.hpp"

#include "jit.hpp"

#include <cuda_runtime_api.h>

#include <algorithm>
#include <new>

namespace fer::capi {

size_t dtype_size(uint32_t dtype) {
    switch (dtype) {
        case FER_DTYPE_F32: case FER_DTYPE_I32: case FER_DTYPE_U32: return 4;
        case FER_DTYPE_F16: case FER_DTYPE_BF16: case FER_DTYPE_I16: case FER_DTYPE_U16: return 2;
        case FER_DTYPE_I8: case FER_DTYPE_U8: return 1;
        case FER_DTYPE_I64: case FER_DTYPE_U64: case FER_DTYPE_F64: return 8;
        default: return 0;
    }
}

fer_status_t check_desc(const fer_buffer_desc_t& d, size_t* numel, size_t* bytes) {
    if (d.rank == 0 || d.rank > 4) return invalid("rank must be in [1,4]");
    const size_t es = dtype_size(d.dtype);
    size_t n = 1;
    for (uint32_t i = 0; i < d.rank; ++i) n *= d.dims[i];
    if (es == 0 || n == 0) return invalid("unsupported dtype or empty buffer");
    if (numel) *numel = n;
    if (bytes) *bytes = n * es;
    return ok();
}

Session::~Session() {
    // The session's own stream is synchronised. A stream the caller attached
    // (fer_set_session_stream) belongs to the caller, who may already have
    // destroyed it (the reference's destructor never touches the stream):
    // the device is synchronised instead.
    if (stream) {
        if (pool && stream == gpu_hot_get_stream(pool, 0)) cudaStreamSynchronize(stream);
        else cudaDeviceSynchronize();
    }
    if (comm) {
        comm_release(comm);
        comm = nullptr;
    }
    models.clear();   // their workspace returns to the pool before it goes away
    for (auto& kv : jobs) {
        Job& j = kv.second;
        if (j.ev) { cudaEventSynchronize(j.ev); cudaEventDestroy(j.ev); j.ev = nullptr; }
        for (const Temp& t : j.temps) free_bytes(t.ptr, t.regime, t.tier, t.bytes);
        j.temps.clear();
    }
    jobs.clear();
    for (cudaEvent_t e : spare_events) cudaEventDestroy(e);
    spare_events.clear();
    jit.reset();
    for (auto& kv : buffers) {
        Buffer& b = kv.second;
        if (!b.external) free_bytes(b.ptr, b.regime, b.tier, b.bytes);
        else if (b.deleter) b.deleter(b.ptr, b.deleter_ctx);
    }
    buffers.clear();
    if (dev_err) cudaFree(dev_err);
    if (pool) gpu_hot_shutdown(pool);
}

fer_status_t Session::resolve_regime(uint32_t requested, uint32_t* out) const {
    const uint32_t r = requested == FER_MEMORY_AUTO ? default_regime : requested;
    if (r <= FER_MEMORY_CUDA_MANAGED) { *out = r; return ok(); }
    if (custom.find(r) == custom.end()) return not_found("custom allocator regime not registered");
    *out = r;
    return ok();
}

fer_status_t Session::alloc_bytes(size_t bytes, uint32_t tier, uint32_t tag, uint32_t regime, void** out) {
    *out = nullptr;
    if (bytes == 0) return internal("builtin regime allocation failed");
    if (regime == FER_MEMORY_CUSTOM_POOL) {
        void* p = gpu_hot_alloc(pool, (bytes + 255) & ~static_cast<size_t>(255));
        if (!p) return internal("builtin regime allocation failed");
        *out = p;
        return ok();
    }
    if (regime == FER_MEMORY_CUDA_MALLOC || regime == FER_MEMORY_CUDA_MANAGED) {
        const uint64_t cap = tier == FER_ALLOC_TIER_IMMUTABLE ? cfg.immutable_bytes : cfg.mutable_bytes;
        if (cap > 0 && live_bytes[tier ? 1 : 0] + bytes > cap) return internal("builtin regime allocation failed");
        void* p = nullptr;
        const cudaError_t e = regime == FER_MEMORY_CUDA_MALLOC ? cudaMalloc(&p, bytes)
                                                                 : cudaMallocManaged(&p, bytes, cudaMemAttachGlobal);
        if (e != cudaSuccess) { cudaGetLastError(); return internal("builtin regime allocation failed"); }
        live_bytes[tier ? 1 : 0] += bytes;
        *out = p;
        return ok();
    }
    auto it = custom.find(regime);
    if (it == custom.end()) return not_found("custom allocator regime not registered");
    const CustomAlloc& c = it->second;
    void* p = c.alloc ? c.alloc(bytes, tier, tag, c.ctx) : c.hot_alloc(c.runtime, bytes);
    if (!p) return internal("custom allocator returned null");
    *out = p;
    return ok();
}

fer_status_t Session::free_bytes(void* ptr, uint32_t regime, uint32_t tier, size_t bytes) {
    if (!ptr) return ok();
    if (regime == FER_MEMORY_CUSTOM_POOL) { gpu_hot_free(pool, ptr); return ok(); }
    if (regime == FER_MEMORY_CUDA_MALLOC || regime == FER_MEMORY_CUDA_MANAGED) {
        cudaFree(ptr);
        size_t& lb = live_bytes[tier ? 1 : 0];
        lb = lb >= bytes ? lb - bytes : 0;
        return ok();
    }
    auto it = custom.find(regime);
    if (it == custom.end()) return not_found("custom allocator regime not registered");
    const CustomAlloc& c = it->second;
    if (c.free) c.free(ptr, c.ctx);
    else c.hot_free(c.runtime, ptr);
    return ok();
}

fer_status_t Session::alloc_temp(size_t bytes, uint32_t regime_req, Temp* out) {
    uint32_t regime = 0;
    fer_status_t st = resolve_regime(regime_req, &regime);
    if (st.code != FER_STATUS_OK) return st;
    void* p = nullptr;
    st = alloc_bytes(bytes, FER_ALLOC_TIER_MUTABLE, 0, regime, &p);
    if (st.code != FER_STATUS_OK) return st;
    *out = Temp{p, regime, FER_ALLOC_TIER_MUTABLE, bytes};
    return ok();
}

const Buffer* Session::find(uint64_t id) const {
    auto it = buffers.find(id);
    return it == buffers.end() ? nullptr : &it->second;
}

fer_status_t Session::add_buffer(const fer_buffer_desc_t& d, void* ptr, uint32_t regime, bool external,
                                 fer_external_buffer_deleter_fn del, void* del_ctx, uint64_t* out_id) {
    Buffer b;
    b.ptr = ptr;
    b.desc = d;
    check_desc(d, &b.numel, &b.bytes);
    b.regime = regime;
    b.tier = d.immutable ? FER_ALLOC_TIER_IMMUTABLE : FER_ALLOC_TIER_MUTABLE;
    b.external = external;
    b.deleter = del;
    b.deleter_ctx = del_ctx;
    const uint64_t id = next_buffer++;
    buffers.emplace(id, b);
    *out_id = id;
    return ok();
}

// A caller that never polls its jobs would otherwise cost one
// cudaEventCreate per submission: once 64 jobs are outstanding, the oldest
// (by then normally complete) is finalized and its event reused.
// Work on one stream completes in submission order, so once the event of a
// pending job is complete, every older pending job recorded on the same
// stream is complete too: one query retires up to kReclaimBatch jobs.
void Session::reclaim_oldest() {
    constexpr size_t kReclaimBatch = 32;
    while (!pending.empty()) {
        auto it = jobs.find(pending.front());
        if (it != jobs.end() && !it->second.finalized) break;
        pending.pop_front();
    }
    if (pending.empty()) return;
    size_t k = (pending.size() < kReclaimBatch ? pending.size() : kReclaimBatch) - 1;
    const Job* probe = nullptr;
    for (;; --k) {
        auto it = jobs.find(pending[k]);
        if (it != jobs.end() && !it->second.finalized) {
            probe = &it->second;
            break;
        }
        if (k == 0) return;
    }
    const cudaStream_t st = probe->stream;
    if (cudaEventQuery(probe->ev) != cudaSuccess) {
        // the oldest alone may still be done
        Job& j = jobs[pending.front()];
        if (cudaEventQuery(j.ev) == cudaSuccess) {
            finalize_done(j);
            pending.pop_front();
        }
        return;
    }
    for (size_t i = 0; i <= k && !pending.empty(); ++i) {
        auto it = jobs.find(pending.front());
        if (it != jobs.end() && !it->second.finalized) {
            if (it->second.stream != st) return;   // another stream: no ordering to rely on
            finalize_done(it->second);
        }
        pending.pop_front();
    }
}

void Session::finalize_done(Job& j) {
    for (const Temp& t : j.temps) free_bytes(t.ptr, t.regime, t.tier, t.bytes);
    j.temps.clear();
    spare_events.push_back(j.ev);
    j.ev = nullptr;
    j.finalized = true;
}

namespace {
constexpr uint64_t kJobsPerEvent = 16;   // submissions that share one completion event at most
}

fer_status_t Session::close_open() {
    if (!open_first) return ok();
    cudaEvent_t ev = nullptr;
    if (spare_events.empty() && pending.size() >= 64) reclaim_oldest();
    if (!spare_events.empty()) {
        ev = spare_events.back();
        spare_events.pop_back();
    } else if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
        return internal("cudaEventCreate failed");
    }
    if (cudaEventRecord(ev, open_stream) != cudaSuccess) {
        spare_events.push_back(ev);
        return internal("cudaEventRecord failed");
    }
    // the run is contiguous: every job since open_first was submitted on open_stream
    const uint64_t last = next_job - 1;
    Job& l = jobs[last];
    l.ev = ev;
    l.cover = last;
    pending.push_back(last);
    for (uint64_t id = open_first; id < last; ++id) {
        auto it = jobs.find(id);
        if (it != jobs.end()) it->second.cover = last;
    }
    open_first = 0;
    return ok();
}

fer_status_t Session::cover_of(uint64_t id, uint64_t* out) {
    auto it = jobs.find(id);
    if (it == jobs.end()) return not_found("job id not found");
    if (it->second.cover == 0) {
        const fer_status_t st = close_open();
        if (st.code != FER_STATUS_OK) return st;
    }
    *out = it->second.cover;
    return ok();
}

fer_status_t Session::make_job(std::vector<Temp> temps, uint64_t* out_job) {
    if (open_first && open_stream != stream) {
        const fer_status_t st = close_open();
        if (st.code != FER_STATUS_OK) {
            for (const Temp& t : temps) free_bytes(t.ptr, t.regime, t.tier, t.bytes);
            return st;
        }
    }
    if (temps.empty()) {
        const uint64_t id = next_job++;
        Job& j = jobs[id];
        j.stream = stream;
        if (!open_first) {
            open_first = id;
            open_stream = stream;
        }
        if (out_job) *out_job = id;
        // a failed record leaves the run open; a later query records it
        if (id - open_first + 1 >= kJobsPerEvent) close_open();
        return ok();
    }
    cudaEvent_t ev = nullptr;
    if (spare_events.empty() && pending.size() >= 64) reclaim_oldest();
    if (!spare_events.empty()) {
        ev = spare_events.back();
        spare_events.pop_back();
    } else if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
        for (const Temp& t : temps) free_bytes(t.ptr, t.regime, t.tier, t.bytes);
        return internal("cudaEventCreate failed");
    }
    if (cudaEventRecord(ev, stream) != cudaSuccess) {
        spare_events.push_back(ev);
        for (const Temp& t : temps) free_bytes(t.ptr, t.regime, t.tier, t.bytes);
        return internal("cudaEventRecord failed");
    }
    const uint64_t id = next_job++;
    Job& j = jobs[id];
    j.ev = ev;
    j.stream = stream;
    j.cover = id;
    j.temps = std::move(temps);
    pending.push_back(id);
    if (open_first) {
        // an open run on this stream completes before this event
        for (uint64_t k = open_first; k < id; ++k) {
            auto it = jobs.find(k);
            if (it != jobs.end()) it->second.cover = id;
        }
        open_first = 0;
    }
    if (out_job) *out_job = id;
    return ok();
}

unsigned Session::pdl_early(const uintptr_t* in_lo, const uintptr_t* in_hi, uint32_t n_in, uintptr_t out_lo,
                            uintptr_t out_hi) const {
    const PdlOp& p = last_pdl;
    if (!p.valid || p.stream != stream || p.mark != fer_pdl_launch_count()) return 0;
    auto overlaps = [](uintptr_t a0, uintptr_t a1, uintptr_t b0, uintptr_t b1) { return a0 < b1 && b0 < a1; };
    for (uint32_t i = 0; i < n_in; ++i)
        if (overlaps(in_lo[i], in_hi[i], p.out_lo, p.out_hi)) return 0;
    if (overlaps(out_lo, out_hi, p.out_lo, p.out_hi)) return 1;
    for (uint32_t i = 0; i < p.n_in; ++i)
        if (overlaps(out_lo, out_hi, p.in_lo[i], p.in_hi[i])) return 1;
    return 2;
}

void Session::pdl_record(const uintptr_t* in_lo, const uintptr_t* in_hi, uint32_t n_in, uintptr_t out_lo,
                         uintptr_t out_hi) {
    PdlOp& p = last_pdl;
    p.valid = true;
    p.stream = stream;
    p.mark = fer_pdl_launch_count();
    p.n_in = n_in > 4 ? 4 : n_in;
    for (uint32_t i = 0; i < p.n_in; ++i) {
        p.in_lo[i] = in_lo[i];
        p.in_hi[i] = in_hi[i];
    }
    p.out_lo = out_lo;
    p.out_hi = out_hi;
}

fer_status_t Session::finalize(uint64_t id, bool* done) {
    auto it = jobs.find(id);
    if (it == jobs.end()) return not_found("job id not found");
    Job& j = it->second;
    if (j.finalized) { *done = true; return ok(); }
    uint64_t c = 0;
    fer_status_t st = cover_of(id, &c);
    if (st.code != FER_STATUS_OK) return st;
    if (c != id) {
        bool cd = false;
        st = finalize(c, &cd);
        if (st.code != FER_STATUS_OK) return st;
        if (cd) j.finalized = true;
        *done = cd;
        return ok();
    }
    const cudaError_t q = cudaEventQuery(j.ev);
    if (q == cudaErrorNotReady) { *done = false; return ok(); }
    if (q != cudaSuccess) return internal("cudaEventQuery failed");
    finalize_done(j);
    *done = true;
    return ok();
}

}  // namespace fer::capi

using fer::capi::Buffer;
using fer::capi::Session;
using fer::capi::internal;
using fer::capi::invalid;
using fer::capi::not_found;
using fer::capi::ok;

#define FER_SESSION(s)                                         \
    if (!(s)) return invalid("session is null");               \
    Session& S = (s)->impl

extern "C" {

fer_status_t fer_session_create(int32_t device, const fer_pool_config_t* cfg, fer_session_t** out_session) {
    if (!out_session) return invalid("out_session is null");
    *out_session = nullptr;
    try {
        if (cudaSetDevice(device) != cudaSuccess) {
            cudaGetLastError();
            return internal("session creation failure");
        }
        auto* s = new fer_session();
        Session& S = s->impl;
        S.device = device;
        if (cfg) S.cfg = *cfg;
        S.default_regime = (S.cfg.memory_regime <= FER_MEMORY_CUDA_MANAGED) ? S.cfg.memory_regime
                                                                             : FER_MEMORY_CUSTOM_POOL;
        GPUHotConfig pc = gpu_hot_default_config();
        uint64_t pool_bytes = S.cfg.mutable_bytes + S.cfg.immutable_bytes;
        if (pool_bytes < (64ull << 20)) pool_bytes = 64ull << 20;
        pc.fixed_pool_size = pool_bytes;
        pc.min_pool_size = 0;
        pc.reserve_vram = S.cfg.cuda_reserve;
        pc.quiet_init = !S.cfg.verbose;
        S.pool = gpu_hot_init_with_config(device, "fercuda", &pc);
        if (!S.pool) { delete s; return internal("session creation failure"); }
        S.stream = gpu_hot_get_stream(S.pool, 0);
        if (cudaMalloc(reinterpret_cast<void**>(&S.dev_err), sizeof(uint32_t)) != cudaSuccess ||
            cudaMemset(S.dev_err, 0, sizeof(uint32_t)) != cudaSuccess) {
            delete s;
            return internal("session creation failure");
        }
        S.jit = std::make_unique<fer::capi::JitManager>(&S);
        *out_session = s;
        return ok();
    } catch (const std::bad_alloc&) {
        return internal("allocation failure");
    } catch (...) {
        return internal("session creation failure");
    }
}

fer_status_t fer_session_destroy(fer_session_t* session) {
    if (!session) return ok();
    try {
        delete session;
        return ok();
    } catch (...) {
        return internal("session destroy failure");
    }
}

fer_status_t fer_register_custom_allocator(fer_session_t* session, uint32_t regime_id,
                                           const fer_custom_allocator_t* allocator) {
    FER_SESSION(session);
    if (!allocator) return invalid("allocator is null");
    if (!allocator->alloc || !allocator->free) return invalid("allocator callbacks must be non-null");
    if (regime_id <= FER_MEMORY_CUDA_MANAGED || regime_id == FER_MEMORY_AUTO)
        return invalid("regime id is reserved for builtin/auto");
    fer::capi::CustomAlloc c;
    c.alloc = allocator->alloc;
    c.free = allocator->free;
    c.ctx = allocator->user_ctx;
    S.custom[regime_id] = c;
    return ok();
}

fer_status_t fer_register_gpu_hot_allocator(fer_session_t* session, uint32_t regime_id,
                                            const fer_gpu_hot_allocator_t* allocator) {
    FER_SESSION(session);
    if (!allocator) return invalid("allocator is null");
    if (!allocator->alloc || !allocator->free) return invalid("allocator callbacks must be non-null");
    if (regime_id <= FER_MEMORY_CUDA_MANAGED || regime_id == FER_MEMORY_AUTO)
        return invalid("regime id is reserved for builtin/auto");
    fer::capi::CustomAlloc c;
    c.hot_alloc = allocator->alloc;
    c.hot_free = allocator->free;
    c.runtime = allocator->runtime;
    S.custom[regime_id] = c;
    return ok();
}

fer_status_t fer_unregister_custom_allocator(fer_session_t* session, uint32_t regime_id) {
    FER_SESSION(session);
    if (regime_id <= FER_MEMORY_CUDA_MANAGED || regime_id == FER_MEMORY_AUTO)
        return invalid("cannot unregister builtin/auto regime");
    auto it = S.custom.find(regime_id);
    if (it == S.custom.end()) return not_found("custom allocator regime not registered");
    if (S.default_regime == regime_id) S.default_regime = FER_MEMORY_CUSTOM_POOL;
    S.custom.erase(it);
    return ok();
}

fer_status_t fer_set_default_memory_regime(fer_session_t* session, uint32_t regime_id) {
    FER_SESSION(session);
    uint32_t r = 0;
    fer_status_t st = S.resolve_regime(regime_id, &r);
    if (st.code != FER_STATUS_OK) return st;
    S.default_regime = r;
    return ok();
}

fer_status_t fer_get_default_memory_regime(fer_session_t* session, uint32_t* out_regime_id) {
    FER_SESSION(session);
    if (!out_regime_id) return invalid("out_regime_id is null");
    *out_regime_id = S.default_regime;
    return ok();
}

fer_status_t fer_list_registered_regimes(fer_session_t* session, uint32_t* out_regime_ids, size_t capacity,
                                         size_t* out_count) {
    FER_SESSION(session);
    if (!out_count) return invalid("out_count is null");
    std::vector<uint32_t> ids = {FER_MEMORY_CUSTOM_POOL, FER_MEMORY_CUDA_MALLOC, FER_MEMORY_CUDA_MANAGED};
    for (const auto& kv : S.custom) ids.push_back(kv.first);
    std::sort(ids.begin(), ids.end());
    *out_count = ids.size();
    if (out_regime_ids)
        for (size_t i = 0; i < ids.size() && i < capacity; ++i) out_regime_ids[i] = ids[i];
    return ok();
}

fer_status_t fer_alloc_buffer_in_regime(fer_session_t* session, const fer_buffer_desc_t* desc, uint32_t regime_id,
                                        uint64_t* out_buffer_id) {
    FER_SESSION(session);
    if (!desc) return invalid("desc is null");
    if (!out_buffer_id) return invalid("out_id is null");
    size_t numel = 0, bytes = 0;
    fer_status_t st = fer::capi::check_desc(*desc, &numel, &bytes);
    if (st.code != FER_STATUS_OK) return st;
    uint32_t regime = 0;
    st = S.resolve_regime(regime_id, &regime);
    if (st.code != FER_STATUS_OK) return st;
    void* p = nullptr;
    st = S.alloc_bytes(bytes, desc->immutable ? FER_ALLOC_TIER_IMMUTABLE : FER_ALLOC_TIER_MUTABLE, desc->tag,
                       regime, &p);
    if (st.code != FER_STATUS_OK) return st;
    return S.add_buffer(*desc, p, regime, false, nullptr, nullptr, out_buffer_id);
}

fer_status_t fer_alloc_buffer(fer_session_t* session, const fer_buffer_desc_t* desc, uint64_t* out_buffer_id) {
    return fer_alloc_buffer_in_regime(session, desc, FER_MEMORY_AUTO, out_buffer_id);
}

fer_status_t fer_import_external_buffer_with_deleter(fer_session_t* session, const fer_buffer_desc_t* desc,
                                                     void* device_ptr, uint32_t regime_id,
                                                     fer_external_buffer_deleter_fn deleter, void* deleter_user_ctx,
                                                     uint64_t* out_buffer_id) {
    FER_SESSION(session);
    if (!desc) return invalid("desc is null");
    if (!out_buffer_id) return invalid("out_id is null");
    if (!device_ptr) return invalid("device_ptr is null");
    fer_status_t st = fer::capi::check_desc(*desc, nullptr, nullptr);
    if (st.code != FER_STATUS_OK) return st;
    uint32_t regime = 0;
    st = S.resolve_regime(regime_id, &regime);
    if (st.code != FER_STATUS_OK) return st;
    return S.add_buffer(*desc, device_ptr, regime, true, deleter, deleter_user_ctx, out_buffer_id);
}

fer_status_t fer_import_external_buffer(fer_session_t* session, const fer_buffer_desc_t* desc, void* device_ptr,
                                        uint32_t regime_id, uint64_t* out_buffer_id) {
    return fer_import_external_buffer_with_deleter(session, desc, device_ptr, regime_id, nullptr, nullptr,
                                                   out_buffer_id);
}

fer_status_t fer_export_buffer_device_ptr(fer_session_t* session, uint64_t buffer_id, void** out_device_ptr) {
    FER_SESSION(session);
    if (!out_device_ptr) return invalid("out_ptr is null");
    const Buffer* b = S.find(buffer_id);
    if (!b) return not_found("buffer id not found");
    *out_device_ptr = b->ptr;
    return ok();
}

fer_status_t fer_free_buffer(fer_session_t* session, uint64_t buffer_id) {
    FER_SESSION(session);
    auto it = S.buffers.find(buffer_id);
    if (it == S.buffers.end()) return not_found("buffer id not found");
    Buffer& b = it->second;
    if (!b.external) {
        fer_status_t st = S.free_bytes(b.ptr, b.regime, b.tier, b.bytes);
        if (st.code != FER_STATUS_OK) return st;
    } else if (b.deleter) {
        b.deleter(b.ptr, b.deleter_ctx);
    }
    S.buffers.erase(it);
    return ok();
}

fer_status_t fer_upload_bytes(fer_session_t* session, uint64_t buffer_id, const void* host, size_t bytes) {
    FER_SESSION(session);
    if (!host) return invalid("host pointer is null");
    const Buffer* b = S.find(buffer_id);
    if (!b) return not_found("buffer id not found");
    if (bytes != b->bytes) return invalid("upload byte size mismatch");
    if (cudaMemcpyAsync(b->ptr, host, bytes, cudaMemcpyHostToDevice, S.stream) != cudaSuccess) {
        cudaGetLastError();
        return internal("cudaMemcpyAsync H2D failed");
    }
    return ok();
}

fer_status_t fer_upload_f32(fer_session_t* session, uint64_t buffer_id, const float* host, size_t count) {
    FER_SESSION(session);
    if (!host) return invalid("host pointer is null");
    const Buffer* b = S.find(buffer_id);
    if (!b) return not_found("buffer id not found");
    if (b->desc.dtype != FER_DTYPE_F32) return invalid("buffer is not f32");
    if (count != b->numel) return invalid("upload count mismatch");
    return fer_upload_bytes(session, buffer_id, host, count * sizeof(float));
}

fer_status_t fer_download_bytes(fer_session_t* session, uint64_t buffer_id, void* host, size_t bytes) {
    FER_SESSION(session);
    if (!host) return invalid("host pointer is null");
    const Buffer* b = S.find(buffer_id);
    if (!b) return not_found("buffer id not found");
    if (bytes != b->bytes) return invalid("download byte size mismatch");
    if (cudaMemcpyAsync(host, b->ptr, bytes, cudaMemcpyDeviceToHost, S.stream) != cudaSuccess ||
        cudaStreamSynchronize(S.stream) != cudaSuccess) {
        cudaGetLastError();
        return internal("cudaMemcpy D2H failed");
    }
    return ok();
}

fer_status_t fer_download_f32(fer_session_t* session, uint64_t buffer_id, float* host, size_t count) {
    FER_SESSION(session);
    if (!host) return invalid("host pointer is null");
    const Buffer* b = S.find(buffer_id);
    if (!b) return not_found("buffer id not found");
    if (b->desc.dtype != FER_DTYPE_F32) return invalid("buffer is not f32");
    if (count != b->numel) return invalid("download count mismatch");
    return fer_download_bytes(session, buffer_id, host, count * sizeof(float));
}

fer_status_t fer_set_session_stream(fer_session_t* session, uint64_t stream_handle) {
    FER_SESSION(session);
    const cudaStream_t next = reinterpret_cast<cudaStream_t>(static_cast<uintptr_t>(stream_handle));
    // jobs still waiting for a shared completion event get it on the stream
    // they ran on now, while that stream is certainly alive
    if (next != S.stream) S.close_open();
    S.stream = next;
    return ok();
}

fer_status_t fer_get_session_stream(fer_session_t* session, uint64_t* out_stream_handle) {
    FER_SESSION(session);
    if (!out_stream_handle) return invalid("out_stream_handle is null");
    *out_stream_handle = static_cast<uint64_t>(reinterpret_cast<uintptr_t>(S.stream));
    return ok();
}

fer_status_t fer_stream_attach(fer_session_t* session, uint64_t stream_handle) {
    return fer_set_session_stream(session, stream_handle);
}

fer_status_t fer_stream_current(fer_session_t* session, uint64_t* out_stream_handle) {
    return fer_get_session_stream(session, out_stream_handle);
}

fer_status_t fer_job_status(fer_session_t* session, uint64_t job_id, uint8_t* out_done) {
    FER_SESSION(session);
    if (!out_done) return invalid("out_done is null");
    bool done = false;
    fer_status_t st = S.finalize(job_id, &done);
    *out_done = done ? 1u : 0u;
    return st;
}

fer_status_t fer_job_wait(fer_session_t* session, uint64_t job_id) {
    FER_SESSION(session);
    auto it = S.jobs.find(job_id);
    if (it == S.jobs.end()) return not_found("job id not found");
    if (!it->second.finalized) {
        uint64_t c = 0;
        const fer_status_t st = S.cover_of(job_id, &c);
        if (st.code != FER_STATUS_OK) return st;
        const fer::capi::Job& cj = S.jobs[c];
        if (!cj.finalized && cudaEventSynchronize(cj.ev) != cudaSuccess) return internal("cudaEventSynchronize failed");
    }
    bool done = false;
    return S.finalize(job_id, &done);
}

fer_status_t fer_tensor_create(fer_session_t* session, const fer_tensor_spec_t* spec, fer_tensor_handle_t* out_tensor) {
    if (!out_tensor) return invalid("out_tensor is null");
    out_tensor->id = 0;
    if (!spec) return invalid("spec is null");
    fer_buffer_desc_t d{};
    d.dtype = spec->dtype;
    d.rank = spec->rank;
    for (int i = 0; i < 4; ++i) d.dims[i] = spec->dims[i];
    d.immutable = spec->immutable;
    d.tag = spec->tag;
    uint64_t id = 0;
    fer_status_t st = fer_alloc_buffer_in_regime(session, &d, spec->memory_regime, &id);
    if (st.code != FER_STATUS_OK) return st;
    out_tensor->id = id;
    return ok();
}

fer_status_t fer_tensor_attach_external(fer_session_t* session, const fer_tensor_spec_t* spec, void* device_ptr,
                                        fer_external_buffer_deleter_fn deleter, void* deleter_user_ctx,
                                        fer_tensor_handle_t* out_tensor) {
    if (!out_tensor) return invalid("out_tensor is null");
    out_tensor->id = 0;
    if (!spec) return invalid("spec is null");
    fer_buffer_desc_t d{};
    d.dtype = spec->dtype;
    d.rank = spec->rank;
    for (int i = 0; i < 4; ++i) d.dims[i] = spec->dims[i];
    d.immutable = spec->immutable;
    d.tag = spec->tag;
    uint64_t id = 0;
    fer_status_t st = fer_import_external_buffer_with_deleter(session, &d, device_ptr, spec->memory_regime, deleter,
                                                              deleter_user_ctx, &id);
    if (st.code != FER_STATUS_OK) return st;
    out_tensor->id = id;
    return ok();
}

fer_status_t fer_tensor_device_ptr(fer_session_t* session, fer_tensor_handle_t tensor, void** out_device_ptr) {
    return fer_export_buffer_device_ptr(session, tensor.id, out_device_ptr);
}

fer_status_t fer_tensor_release(fer_session_t* session, fer_tensor_handle_t tensor) {
    return fer_free_buffer(session, tensor.id);
}

fer_status_t fer_tensor_upload(fer_session_t* session, fer_tensor_handle_t tensor, const void* host, size_t bytes) {
    return fer_upload_bytes(session, tensor.id, host, bytes);
}

fer_status_t fer_tensor_download(fer_session_t* session, fer_tensor_handle_t tensor, void* host, size_t bytes) {
    return fer_download_bytes(session, tensor.id, host, bytes);
}

// ---- extensions -------------------------------------------------------------

fer_status_t fer_session_device_errors(fer_session_t* session, uint32_t* out_bits, uint8_t clear) {
    FER_SESSION(session);
    if (!out_bits) return invalid("out_bits is null");
    uint32_t v = 0;
    if (cudaMemcpyAsync(&v, S.dev_err, sizeof(v), cudaMemcpyDeviceToHost, S.stream) != cudaSuccess ||
        cudaStreamSynchronize(S.stream) != cudaSuccess)
        return internal("device error word read failed");
    if (clear && v && cudaMemsetAsync(S.dev_err, 0, sizeof(uint32_t), S.stream) != cudaSuccess)
        return internal("device error word clear failed");
    *out_bits = v;
    return ok();
}

fer_status_t fer_pool_get_stats(fer_session_t* session, fer_pool_stats_t* out) {
    FER_SESSION(session);
    if (!out) return invalid("out_stats is null");
    TLSFPoolStats s{};
    gpu_hot_get_tlsf_stats(S.pool, &s);
    out->pool_bytes = s.total_pool_size;
    out->allocated_bytes = s.allocated_bytes;
    out->peak_allocated_bytes = s.peak_allocated;
    out->largest_free_block = s.largest_free_block;
    out->total_allocations = s.total_allocations;
    out->total_frees = s.total_frees;
    out->allocated_blocks = s.allocated_blocks;
    out->free_blocks = s.free_blocks;
    return ok();
}

fer_status_t fer_pool_alloc_raw(fer_session_t* session, uint64_t bytes, void** out_ptr) {
    FER_SESSION(session);
    if (!out_ptr) return invalid("out_ptr is null");
    if (bytes == 0) return invalid("bytes must be > 0");
    *out_ptr = gpu_hot_alloc(S.pool, (bytes + 255) & ~static_cast<uint64_t>(255));
    return *out_ptr ? ok() : internal("pool exhausted");
}

fer_status_t fer_pool_free_raw(fer_session_t* session, void* ptr) {
    FER_SESSION(session);
    if (!ptr) return ok();
    if (!gpu_hot_owns_ptr(S.pool, ptr)) return not_found("pointer not owned by the session pool");
    gpu_hot_free(S.pool, ptr);
    return ok();
}

}  // extern "C"
