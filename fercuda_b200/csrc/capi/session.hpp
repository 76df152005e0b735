// Internal state behind fer_session_t.
//
// Mirrors the reference RuntimeSession (src/runtime/session.cu:62-416),
// RegimeManager (regime_manager.cu:15-123), ElasticPool (elastic_pool.cu:37-131)
// and JobManager (job_manager.cu:23-92) in one object:
//   - buffers: id -> record, ids from a counter starting at 1;
//   - regimes: builtin CUSTOM_POOL (this session's TLSF pool), CUDA_MALLOC,
//     CUDA_MANAGED, plus registered custom allocators;
//   - jobs: an event recorded on the session stream plus the temporaries to
//     release once the event is observed complete; events are pooled;
//   - one session stream (the pool runtime's stream 0, non-blocking).
// Like the reference, a session is used from one thread at a time.
#pragma once

#include "fercuda/api/c_api.h"
#include "fercuda/b200/ext.h"
#include "fercuda/jit/api.h"
#include "gpu/gpu_hot_runtime.h"

#include <cuda_runtime_api.h>

#include <cstdint>
#include <deque>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

// Process-wide count of launches of kernels that trigger their dependents
// (libptx_kernels.so, kernels/pdl.cu).
extern "C" uint64_t fer_pdl_launch_count();
extern "C" void fer_pdl_note_launch();

namespace fer::capi {

inline fer_status_t ok() { return fer_status_t{FER_STATUS_OK, "ok"}; }
inline fer_status_t invalid(const char* m) { return fer_status_t{FER_STATUS_INVALID_ARGUMENT, m}; }
inline fer_status_t not_found(const char* m) { return fer_status_t{FER_STATUS_NOT_FOUND, m}; }
inline fer_status_t internal(const char* m) { return fer_status_t{FER_STATUS_INTERNAL_ERROR, m}; }

size_t dtype_size(uint32_t dtype);

struct Buffer {
    void* ptr = nullptr;
    fer_buffer_desc_t desc{};
    size_t numel = 0;
    size_t bytes = 0;
    uint32_t regime = 0;
    uint32_t tier = 0;
    bool external = false;
    fer_external_buffer_deleter_fn deleter = nullptr;
    void* deleter_ctx = nullptr;
};

struct Temp {
    void* ptr;
    uint32_t regime;
    uint32_t tier;
    size_t bytes;
};

// A job without temporaries shares the completion event of a later job on
// the same stream (`cover`, recorded at most 16 submissions later, or when
// the job is queried, or when the stream changes); a job with temporaries,
// and each covering job, records its own event (cover == its own id).
struct Job {
    cudaEvent_t ev = nullptr;   // own event; null once finalized or when covered
    cudaStream_t stream = nullptr;   // where the job was submitted
    uint64_t cover = 0;         // job whose event covers this one; 0 while not yet recorded
    std::vector<Temp> temps;
    bool finalized = false;
};

struct CustomAlloc {
    fer_allocator_alloc_fn alloc = nullptr;
    fer_allocator_free_fn free = nullptr;
    void* ctx = nullptr;
    // gpu_hot-style registration
    fer_gpu_hot_alloc_fn hot_alloc = nullptr;
    fer_gpu_hot_free_fn hot_free = nullptr;
    void* runtime = nullptr;
};

class JitManager;
struct Transformer;
struct CommState;                 // NCCL communicator of a sharded session (comm.cpp)
void comm_release(CommState* c);  // finalizes (bounded) or aborts, then frees

struct Session {
    int device = 0;
    fer_pool_config_t cfg{};
    GPUHotRuntime* pool = nullptr;
    cudaStream_t stream = nullptr;
    uint32_t default_regime = FER_MEMORY_CUSTOM_POOL;
    std::unordered_map<uint32_t, CustomAlloc> custom;
    std::unordered_map<uint64_t, Buffer> buffers;
    uint64_t next_buffer = 1;
    std::unordered_map<uint64_t, Job> jobs;
    uint64_t next_job = 1;
    std::vector<cudaEvent_t> spare_events;
    std::deque<uint64_t> pending;    // jobs with an event, not yet finalized, oldest first
    uint64_t open_first = 0;         // first job of the run still waiting for an event (0: none)
    cudaStream_t open_stream = nullptr;
    // The last kernel with a known footprint (chain and fast row kernels)
    // this session launched: its stream, the bytes it read and wrote, and the
    // process-wide count of dependent-triggering launches right after it.
    struct PdlOp {
        bool valid = false;
        cudaStream_t stream = nullptr;
        uint64_t mark = 0;
        uint32_t n_in = 0;
        uintptr_t in_lo[4] = {0, 0, 0, 0}, in_hi[4] = {0, 0, 0, 0};
        uintptr_t out_lo = 0, out_hi = 0;
    } last_pdl;
    // How much of a kernel reading [in_lo[i], in_hi[i]) and writing
    // [out_lo, out_hi) may run before its programmatic launch wait, if it is
    // launched next on the session stream: 0 nothing, 1 its reads (the
    // kernel before writes none of the inputs), 2 everything (that kernel
    // also neither reads nor writes the output). Nonzero only when the
    // kernel before is last_pdl: no launch of another kernel that triggers
    // its dependents anywhere in the process since. A kernel that never
    // triggers its dependents cannot be overlapped by the next one, so it
    // needs no record.
    unsigned pdl_early(const uintptr_t* in_lo, const uintptr_t* in_hi, uint32_t n_in, uintptr_t out_lo,
                       uintptr_t out_hi) const;
    void pdl_record(const uintptr_t* in_lo, const uintptr_t* in_hi, uint32_t n_in, uintptr_t out_lo,
                    uintptr_t out_hi);
    size_t live_bytes[2] = {0, 0};   // CUDA_MALLOC / MANAGED budget per tier
    uint32_t* dev_err = nullptr;     // device error word (cudaMalloc'd)
    std::unique_ptr<JitManager> jit;
    std::unordered_map<uint64_t, std::shared_ptr<Transformer>> models;
    uint64_t next_model = 1;
    CommState* comm = nullptr;

    ~Session();

    // Regimes and memory.
    fer_status_t resolve_regime(uint32_t requested, uint32_t* out) const;
    fer_status_t alloc_bytes(size_t bytes, uint32_t tier, uint32_t tag, uint32_t regime, void** out);
    fer_status_t free_bytes(void* ptr, uint32_t regime, uint32_t tier, size_t bytes);
    fer_status_t alloc_temp(size_t bytes, uint32_t regime, Temp* out);

    // Buffers.
    const Buffer* find(uint64_t id) const;
    fer_status_t add_buffer(const fer_buffer_desc_t& d, void* ptr, uint32_t regime, bool external,
                            fer_external_buffer_deleter_fn del, void* del_ctx, uint64_t* out_id);

    // Jobs: records completion of everything queued so far on the stream.
    fer_status_t make_job(std::vector<Temp> temps, uint64_t* out_job);
    fer_status_t finalize(uint64_t id, bool* done);
    void finalize_done(Job& j);   // j's event has completed
    // Records one event for the open run of jobs without their own event.
    fer_status_t close_open();
    // Job id whose event covers `id` (recording it first if needed).
    fer_status_t cover_of(uint64_t id, uint64_t* out);
    // Finalizes completed outstanding jobs, oldest first (up to 32 per event
    // query, relying on in-order completion on one stream), returning their
    // events to spare_events.
    void reclaim_oldest();
};

// Validates a buffer descriptor (rank 1..4, known dtype, nonzero size).
fer_status_t check_desc(const fer_buffer_desc_t& d, size_t* numel, size_t* bytes);

}  // namespace fer::capi

struct fer_session {
    fer::capi::Session impl;
};

// Kernel launchers exported by libptx_kernels.so.
extern "C" {
cudaError_t fer_rows_f32(const float* x, float* y, const float* gamma, const float* beta, int rows, int cols,
                         float eps, uint32_t flags, uint32_t* err, cudaStream_t stream);
cudaError_t fer_rows_f32_pdl(const float* x, float* y, const float* gamma, const float* beta, int rows, int cols,
                             float eps, uint32_t flags, uint32_t early, uint32_t* err, cudaStream_t stream);
cudaError_t fer_layer_norm_typed(const void* x, void* y, int rows, int cols, float eps, uint32_t dtype,
                                 uint32_t* err, cudaStream_t stream);
cudaError_t fer_matmul_ref_order(const void* a, const void* b, void* c, int M, int K, int N, uint32_t dtype,
                                 cudaStream_t stream);
cudaError_t fer_cast_to_f32(const void* in, float* out, size_t n, uint32_t dtype, cudaStream_t stream);
cudaError_t fer_cast_from_f32(const float* in, void* out, size_t n, uint32_t dtype, cudaStream_t stream);
cudaError_t fer_matmul_bf16_f32_ref_order(const void* a, const void* b, float* c, int M, int K, int N,
                                          cudaStream_t stream);
cudaError_t fer_gemm_bf16_tc(const void* a, const void* b, void* c, int M, int N, int K, uint32_t out_dtype,
                             uint32_t* err, cudaStream_t stream);
cudaError_t fer_gemm_bf16_tc_ex(const void* a, const void* b, void* c, const float* resid, int M, int N, int K, int epi,
                                uint32_t* err, cudaStream_t stream);
cudaError_t fer_fill_normal_bf16(void* out, size_t n, uint64_t seed, float stddev, cudaStream_t s);
cudaError_t fer_fill_f32(float* out, size_t n, float v, cudaStream_t s);
cudaError_t fer_embed_f32(const int* tok, const void* emb, float* x, int T, int d, int vocab, uint32_t* err,
                          cudaStream_t s);
cudaError_t fer_embed_ln_bf16(const int* tok, const void* emb, float* x, const float* g, const float* b, void* out,
                              int T, int d, int vocab, float eps, uint32_t* err, cudaStream_t s);
cudaError_t fer_ln_bf16(const float* x, const float* g, const float* b, void* out, int T, int d, float eps,
                        cudaStream_t s);
cudaError_t fer_rows_fast_f32(const float* x, float* y, const float* gamma, const float* beta, int rows, int cols,
                              float eps, uint32_t flags, uint32_t* err, cudaStream_t stream);
cudaError_t fer_rows_fast_f32_pdl(const float* x, float* y, const float* gamma, const float* beta, int rows, int cols,
                                  float eps, uint32_t flags, uint32_t early, uint32_t* err, cudaStream_t stream);
cudaError_t fer_attn_causal(const void* qkv, void* out, int B, int S, int d, int heads, cudaStream_t s);
size_t fer_gemm_splitk_workspace_bytes(int M, int N, int K);
cudaError_t fer_gemm_bf16_tc_splitk(const void* a, const void* b, void* c, int M, int N, int K, int epi, int splits,
                                    float* ws, size_t ws_bytes, int flags, uint32_t* err, cudaStream_t stream);
cudaError_t fer_kv_store(const void* qkv, void* k_cache, void* v_cache, int B, int S, int d, int heads, int max_seq,
                         int pos0, cudaStream_t s);
size_t fer_attn_decode_scratch_floats(int B, int heads, int n_keys);
cudaError_t fer_decode_kv_attention(const void* qkv_dec, void* k_cache, void* v_cache, void* out, float* scratch,
                                    int* counters, int B, int d, int heads, int max_seq, int* d_len, uint32_t* err,
                                    cudaStream_t s);
cudaError_t fer_device_int_add(int* d_len, int v, cudaStream_t s);
cudaError_t fer_device_int_set(int* d_len, int v, cudaStream_t s);
cudaError_t fer_attn_decode(const void* qkv_dec, const void* k_cache, const void* v_cache, void* out, float* scratch,
                            int B, int d, int heads, int max_seq, int n_keys, uint32_t* err, cudaStream_t s);
cudaError_t fer_attn_causal_ex(const void* qkv, void* out, int B, int S, int d, int heads, int flags, uint32_t* err,
                               cudaStream_t s);
}
