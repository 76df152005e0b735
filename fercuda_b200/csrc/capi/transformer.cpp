// fer_transformer_*: the decoder-only transformer forward on this library's
// kernels (gemm_tc.cu, xfmr_kernels.cu), every buffer from the session pool.
//
// The reference has no transformer of its own: its demo
// (rust/deps/ferrite-torch/examples/transformer_demo.rs:18-70, 72-224) runs a
// pre-LN block through libtorch on TLSF memory. This driver computes the same
// block structure with token embedding, final LN and LM head added; per layer
//   a   = LN1(x)                      ln_bf16            f32 -> bf16
//   qkv = a @ Wqkv                    tcgen05 GEMM       bf16 out
//   o   = causal_attention(qkv)       attn_causal        bf16 out
//   x   = x + o @ Wo                  tcgen05 GEMM       f32 residual epilogue, in place
//   a   = LN2(x)
//   h   = gelu(a @ W1)                tcgen05 GEMM       exact-GELU bf16 epilogue
//   x   = x + h @ W2                  tcgen05 GEMM       f32 residual epilogue
// then logits = LN_f(x) @ Wlm in f32. Sequences of a batch never interact,
// so any split of the batch across GPUs gives the same logits bit for bit.
#include "session.hpp"

#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <unordered_map>
#include <vector>

namespace fer::capi {

// Keys and values of up to max_batch sequences x max_seq positions, per
// layer [max_batch][heads][max_seq][64] bf16 each (K block, then V block).
struct KvCache {
    uint32_t max_batch = 0, max_seq = 0;
    uint32_t batch = 0, len = 0;     // set by prefill, len advanced by decode
    uint16_t* kv = nullptr;          // layers x 2 x max_batch x heads x max_seq x 64
    float* scratch = nullptr;        // decode attention chunk partials
    int* attn_counters = nullptr;    // decode attention: chunks done per (sequence, head)
    float* gemm_ws = nullptr;        // split-K partials of the decode GEMMs
    size_t gemm_ws_bytes = 0;
    int* d_len = nullptr;            // device copy of len (position of the next token)
    int* tok_stage = nullptr;        // decode tokens [max_batch] and logits [max_batch, vocab]
    float* logit_stage = nullptr;    // at fixed addresses, so a captured step replays
    cudaGraphExec_t graph = nullptr; // the decode step, captured on the second call with a batch
    uint32_t graph_batch = 0;
    uint32_t eager_batch = 0;
    size_t layer_elems = 0;          // elements of one layer's K (or V) block
};

struct Transformer {
    fer_transformer_config_t cfg{};
    Session* S = nullptr;
    uint64_t weight_buf = 0;
    uint16_t* W = nullptr;      // bf16 blob
    size_t w_elems = 0;
    float* ln = nullptr;        // gamma / beta blob
    size_t ln_elems = 0;
    size_t off_emb = 0, off_lm = 0;
    std::vector<size_t> off_qkv, off_o, off_w1, off_w2;
    // workspace for max_tokens
    float* x = nullptr;
    uint16_t* a = nullptr;
    uint16_t* qkv = nullptr;
    uint16_t* att = nullptr;
    uint16_t* hid = nullptr;
    // profiling
    bool profiling = false;
    struct Mark { cudaEvent_t a, b; int cls; double flops; };
    std::vector<Mark> marks;
    std::vector<cudaEvent_t> spare;
    fer_transformer_profile_t prof{};
    // CUDA graphs of the forward, one per (tokens, logits, batch, seq): the
    // second forward with a signature is captured, later ones replay it.
    struct Graph {
        const void* tokens;
        void* logits;
        int B, Sq;
        cudaGraphExec_t exec;
    };
    std::vector<Graph> graphs;
    bool graphs_off = false;
    std::unordered_map<uint64_t, KvCache> caches;
    // fer_transformer_forward_host: two staging slots for chunk tokens and
    // logits, the stream their D2H copies run on, and per-slot events
    int* stage_tok[2] = {nullptr, nullptr};
    float* stage_logits[2] = {nullptr, nullptr};
    size_t stage_tokens = 0;
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t computed[2] = {nullptr, nullptr}, copied[2] = {nullptr, nullptr};

    void free_cache(KvCache& kc) {
        if (kc.graph) cudaGraphExecDestroy(kc.graph);
        for (void* p : {static_cast<void*>(kc.kv), static_cast<void*>(kc.scratch),
                        static_cast<void*>(kc.attn_counters), static_cast<void*>(kc.gemm_ws),
                        static_cast<void*>(kc.d_len), static_cast<void*>(kc.tok_stage),
                        static_cast<void*>(kc.logit_stage)})
            if (p) gpu_hot_free(S->pool, p);
        kc = KvCache{};
    }

    cudaEvent_t event() {
        cudaEvent_t e = nullptr;
        if (!spare.empty()) {
            e = spare.back();
            spare.pop_back();
        } else {
            cudaEventCreate(&e);
        }
        return e;
    }
    void release_marks() {
        for (auto& m : marks) {
            spare.push_back(m.a);
            spare.push_back(m.b);
        }
        marks.clear();
    }

    ~Transformer() {
        if (!S) return;
        for (auto& kv : caches) free_cache(kv.second);
        for (auto& g : graphs)
            if (g.exec) cudaGraphExecDestroy(g.exec);
        release_marks();
        for (cudaEvent_t e : spare) cudaEventDestroy(e);
        if (copy_stream) {
            cudaStreamSynchronize(copy_stream);
            cudaStreamDestroy(copy_stream);
        }
        for (int s = 0; s < 2; ++s) {
            for (cudaEvent_t e : {computed[s], copied[s]})
                if (e) cudaEventDestroy(e);
            for (void* p : {static_cast<void*>(stage_tok[s]), static_cast<void*>(stage_logits[s])})
                if (p) gpu_hot_free(S->pool, p);
        }
        for (void* p : {static_cast<void*>(x), static_cast<void*>(a), static_cast<void*>(qkv),
                        static_cast<void*>(att), static_cast<void*>(hid), static_cast<void*>(ln)})
            if (p) gpu_hot_free(S->pool, p);
        auto it = S->buffers.find(weight_buf);
        if (it != S->buffers.end()) {
            S->free_bytes(it->second.ptr, it->second.regime, it->second.tier, it->second.bytes);
            S->buffers.erase(it);
        }
    }
};

}  // namespace fer::capi

using fer::capi::Buffer;
using fer::capi::KvCache;
using fer::capi::Session;
using fer::capi::Transformer;
using fer::capi::internal;
using fer::capi::invalid;
using fer::capi::not_found;
using fer::capi::ok;

namespace {

enum : int { kEpiF32 = 0, kEpiBF16 = 1, kEpiGeluBF16 = 2, kEpiResidF32 = 3 };

size_t up128(size_t n) { return (n + 127) & ~static_cast<size_t>(127); }

Transformer* find_model(Session& S, uint64_t id) {
    auto it = S.models.find(id);
    return it == S.models.end() ? nullptr : it->second.get();
}

void* pool_alloc(Session& S, size_t bytes) { return gpu_hot_alloc(S.pool, (bytes + 255) & ~static_cast<size_t>(255)); }

}  // namespace

extern "C" {

fer_status_t fer_transformer_create(fer_session_t* session, const fer_transformer_config_t* cfg, uint64_t* out_model) {
    if (!session) return invalid("session is null");
    if (!cfg || !out_model) return invalid("config or out_model is null");
    Session& S = session->impl;
    const fer_transformer_config_t c = *cfg;
    if (c.layers == 0 || c.heads == 0 || c.d_model != c.heads * 64u) return invalid("transformer requires head_dim 64");
    if (c.d_model % 256 || c.d_model > 4096) return invalid("transformer d_model must be a multiple of 256, <= 4096");
    if (c.ffn == 0 || c.ffn % 8 || c.vocab == 0 || c.vocab % 8) return invalid("transformer ffn and vocab must be multiples of 8");
    if (c.max_tokens == 0) return invalid("transformer max_tokens must be > 0");
    auto m = std::shared_ptr<Transformer>(new Transformer());
    m->cfg = c;
    if (m->cfg.eps <= 0.0f) m->cfg.eps = 1e-5f;
    const size_t d = c.d_model, F = c.ffn, V = c.vocab;
    size_t off = 0;
    m->off_emb = off;
    off = up128(off + V * d);
    for (uint32_t l = 0; l < c.layers; ++l) {
        m->off_qkv.push_back(off);
        off = up128(off + d * 3 * d);
        m->off_o.push_back(off);
        off = up128(off + d * d);
        m->off_w1.push_back(off);
        off = up128(off + d * F);
        m->off_w2.push_back(off);
        off = up128(off + F * d);
    }
    m->off_lm = off;
    off = up128(off + d * V);
    m->w_elems = off;
    if (m->w_elems > 0xFFFFFFFFull) return invalid("transformer weights exceed a rank-1 buffer");
    fer_buffer_desc_t wd{};
    wd.dtype = FER_DTYPE_BF16;
    wd.rank = 1;
    wd.dims[0] = static_cast<uint32_t>(m->w_elems);
    wd.immutable = 0;
    void* wp = nullptr;
    fer_status_t st = S.alloc_bytes(m->w_elems * 2, FER_ALLOC_TIER_MUTABLE, 0, FER_MEMORY_CUSTOM_POOL, &wp);
    if (st.code != FER_STATUS_OK) return st;
    S.add_buffer(wd, wp, FER_MEMORY_CUSTOM_POOL, false, nullptr, nullptr, &m->weight_buf);
    m->W = static_cast<uint16_t*>(wp);
    m->S = &S;
    m->ln_elems = static_cast<size_t>(4 * c.layers + 2) * d;
    m->ln = static_cast<float*>(pool_alloc(S, m->ln_elems * 4));
    const size_t T = c.max_tokens;
    m->x = static_cast<float*>(pool_alloc(S, T * d * 4));
    m->a = static_cast<uint16_t*>(pool_alloc(S, T * d * 2));
    m->qkv = static_cast<uint16_t*>(pool_alloc(S, T * 3 * d * 2));
    m->att = static_cast<uint16_t*>(pool_alloc(S, T * d * 2));
    m->hid = static_cast<uint16_t*>(pool_alloc(S, T * F * 2));
    if (!m->ln || !m->x || !m->a || !m->qkv || !m->att || !m->hid) return internal("transformer workspace allocation failed");
    const uint64_t id = S.next_model++;
    S.models.emplace(id, m);
    *out_model = id;
    return fer_transformer_init_weights(session, id, 4, 0.02f);
}

fer_status_t fer_transformer_init_weights(fer_session_t* session, uint64_t model, uint64_t seed, float stddev) {
    if (!session) return invalid("session is null");
    Session& S = session->impl;
    Transformer* m = find_model(S, model);
    if (!m) return not_found("model id not found");
    cudaError_t e = fer_fill_normal_bf16(m->W, m->w_elems, seed, stddev, S.stream);
    const size_t d = m->cfg.d_model;
    for (uint32_t blk = 0; blk < 2 * m->cfg.layers + 1 && e == cudaSuccess; ++blk) {
        e = fer_fill_f32(m->ln + 2 * blk * d, d, 1.0f, S.stream);               // gamma
        if (e == cudaSuccess) e = fer_fill_f32(m->ln + (2 * blk + 1) * d, d, 0.0f, S.stream);   // beta
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return internal("kernel launch failed");
    }
    return ok();
}

fer_status_t fer_transformer_weight_buffer(fer_session_t* session, uint64_t model, uint64_t* out_buffer_id) {
    if (!session || !out_buffer_id) return invalid("session or out_buffer_id is null");
    Transformer* m = find_model(session->impl, model);
    if (!m) return not_found("model id not found");
    *out_buffer_id = m->weight_buf;
    return ok();
}

}  // extern "C"

namespace {

// Queues one forward of B sequences of Sq tokens (tok: device i32 [B*Sq];
// logits: device f32 [B*Sq, vocab]) on the session stream: eager on the
// first use of a (tok, logits, B, Sq) signature, captured into a CUDA graph
// on the second, replayed after that.
cudaError_t forward_ptrs(Session& S, Transformer* m, const int* tok, float* logits, int B, int Sq) {
    const size_t T = static_cast<size_t>(B) * Sq;
    const fer_transformer_config_t& c = m->cfg;
    const int d = static_cast<int>(c.d_model), F = static_cast<int>(c.ffn), V = static_cast<int>(c.vocab);
    const int Ti = static_cast<int>(T);
    cudaStream_t st = S.stream;
    uint32_t* err = S.dev_err;
    const uint16_t* W = m->W;
    // Each launch goes through `run`, which brackets it with an event pair
    // when profiling is on (class 0 gemm, 1 attention, 2 norm, 3 other).
    cudaError_t e = cudaSuccess;
    auto run = [&](int cls, double flops, auto&& launch) {
        if (e != cudaSuccess) return;
        if (!m->profiling) {
            e = launch();
            return;
        }
        Transformer::Mark mk{m->event(), m->event(), cls, flops};
        cudaEventRecord(mk.a, st);
        e = launch();
        cudaEventRecord(mk.b, st);
        m->marks.push_back(mk);
    };
    const double Td = static_cast<double>(T);
    const double gq = 2.0 * Td * 3 * d * d, go = 2.0 * Td * d * d, g1f = 2.0 * Td * d * F, glm = 2.0 * Td * d * V;
    // causal attention: S(S+1)/2 (query, key) pairs per sequence and head, 2*64 flops each for QK^T and for PV
    const double ga = 4.0 * 64.0 * (static_cast<double>(Sq) * (Sq + 1) / 2.0) * B * c.heads;
    auto issue = [&]() {
        for (uint32_t l = 0; l < c.layers && e == cudaSuccess; ++l) {
            const float* g1 = m->ln + (4 * l + 0) * static_cast<size_t>(d);
            const float* b1 = m->ln + (4 * l + 1) * static_cast<size_t>(d);
            const float* g2 = m->ln + (4 * l + 2) * static_cast<size_t>(d);
            const float* b2 = m->ln + (4 * l + 3) * static_cast<size_t>(d);
            if (l == 0)   // embedding and the first layer norm in one pass
                run(2, 0.0, [&] {
                    return fer_embed_ln_bf16(tok, W + m->off_emb, m->x, g1, b1, m->a, Ti,
                                             d, V, c.eps, err, st);
                });
            else
                run(2, 0.0, [&] { return fer_ln_bf16(m->x, g1, b1, m->a, Ti, d, c.eps, st); });
            run(0, gq, [&] { return fer_gemm_bf16_tc_ex(m->a, W + m->off_qkv[l], m->qkv, nullptr, Ti, 3 * d, d, kEpiBF16, err, st); });
            run(1, ga, [&] { return fer_attn_causal_ex(m->qkv, m->att, B, Sq, d, static_cast<int>(c.heads), 0, err, st); });
            run(0, go, [&] { return fer_gemm_bf16_tc_ex(m->att, W + m->off_o[l], m->x, m->x, Ti, d, d, kEpiResidF32, err, st); });
            run(2, 0.0, [&] { return fer_ln_bf16(m->x, g2, b2, m->a, Ti, d, c.eps, st); });
            run(0, g1f, [&] { return fer_gemm_bf16_tc_ex(m->a, W + m->off_w1[l], m->hid, nullptr, Ti, F, d, kEpiGeluBF16, err, st); });
            run(0, g1f, [&] { return fer_gemm_bf16_tc_ex(m->hid, W + m->off_w2[l], m->x, m->x, Ti, d, F, kEpiResidF32, err, st); });
        }
        const float* gf = m->ln + (4 * static_cast<size_t>(c.layers)) * d;
        const float* bf = gf + d;
        run(2, 0.0, [&] { return fer_ln_bf16(m->x, gf, bf, m->a, Ti, d, c.eps, st); });
        run(0, glm, [&] { return fer_gemm_bf16_tc_ex(m->a, W + m->off_lm, logits, nullptr, Ti, V, d, kEpiF32, err, st); });
    };
    static const int graphs_env = [] {
        const char* ev = std::getenv("FERCUDA_XFMR_GRAPH");
        return (ev && ev[0] == '0') ? 0 : 1;
    }();
    Transformer::Graph* g = nullptr;
    if (!m->profiling && graphs_env && !m->graphs_off) {
        for (auto& x : m->graphs)
            if (x.tokens == tok && x.logits == logits && x.B == B && x.Sq == Sq) g = &x;
        if (!g && m->graphs.size() < 8) {
            m->graphs.push_back(Transformer::Graph{tok, logits, B, Sq, nullptr});   // first use: eager
        } else if (g && !g->exec) {
            // second use: capture the 59 launches once
            cudaGraph_t graph = nullptr;
            if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
                issue();
                const cudaError_t ce = cudaStreamEndCapture(st, &graph);
                if (e == cudaSuccess && ce == cudaSuccess && graph &&
                    cudaGraphInstantiate(&g->exec, graph, 0) != cudaSuccess)
                    g->exec = nullptr;
                if (graph) cudaGraphDestroy(graph);
                if (e != cudaSuccess || ce != cudaSuccess || !g->exec) {
                    cudaGetLastError();
                    m->graphs_off = true;   // this driver / these kernels: stay eager
                    g->exec = nullptr;
                    e = cudaSuccess;
                }
            } else {
                cudaGetLastError();
                m->graphs_off = true;
            }
        }
    }
    if (g && g->exec) e = cudaGraphLaunch(g->exec, st);
    else issue();
    if (e == cudaSuccess && m->profiling) m->prof.forwards++;
    return e;
}

// Chunk size of fer_transformer_forward_host when the caller passes 0: at
// most about 4096 tokens (8 sequences of 512) and at least four chunks when
// the batch allows (only the first chunk's forward is not under a copy),
// within max_tokens.
uint32_t default_chunk(const fer_transformer_config_t& c, uint32_t batch, uint32_t seq) {
    uint32_t k = seq >= 4096 ? 1u : 4096u / seq;
    k = std::min<uint32_t>(k, (batch + 3) / 4);
    k = std::min<uint32_t>(k, std::max<uint32_t>(1u, c.max_tokens / seq));
    return std::max<uint32_t>(1u, std::min(k, batch));
}

}  // namespace

extern "C" {

fer_status_t fer_transformer_forward(fer_session_t* session, uint64_t model, uint64_t tokens, uint64_t logits,
                                     uint64_t* out_job_id) {
    if (!session) return invalid("session is null");
    Session& S = session->impl;
    Transformer* m = find_model(S, model);
    if (!m) return not_found("model id not found");
    const Buffer* tb = S.find(tokens);
    const Buffer* lb = S.find(logits);
    if (!tb || !lb) return not_found("buffer id not found");
    if (tb->desc.dtype != FER_DTYPE_I32 || (tb->desc.rank != 1 && tb->desc.rank != 2))
        return invalid("tokens must be i32 [batch, seq] or [seq]");
    const int B = tb->desc.rank == 2 ? static_cast<int>(tb->desc.dims[0]) : 1;
    const int Sq = tb->desc.rank == 2 ? static_cast<int>(tb->desc.dims[1]) : static_cast<int>(tb->desc.dims[0]);
    const size_t T = static_cast<size_t>(B) * Sq;
    const fer_transformer_config_t& c = m->cfg;
    if (T > c.max_tokens) return invalid("batch * seq exceeds the model's max_tokens");
    if (lb->desc.dtype != FER_DTYPE_F32 || lb->numel != T * c.vocab) return invalid("logits must be f32 [batch, seq, vocab]");
    if (forward_ptrs(S, m, static_cast<const int*>(tb->ptr), static_cast<float*>(lb->ptr), B, Sq) != cudaSuccess) {
        cudaGetLastError();
        return internal("kernel launch failed");
    }
    return S.make_job({}, out_job_id);
}

fer_status_t fer_transformer_forward_host(fer_session_t* session, uint64_t model, const int32_t* host_tokens,
                                          uint32_t batch, uint32_t seq, float* host_logits, uint32_t chunk_seqs) {
    if (!session) return invalid("session is null");
    if (!host_tokens || !host_logits) return invalid("host_tokens or host_logits is null");
    Session& S = session->impl;
    Transformer* m = find_model(S, model);
    if (!m) return not_found("model id not found");
    const fer_transformer_config_t& c = m->cfg;
    if (batch == 0 || seq == 0) return invalid("batch and seq must be > 0");
    if (seq > c.max_tokens) return invalid("seq exceeds the model's max_tokens");
    const uint32_t k = chunk_seqs ? chunk_seqs : default_chunk(c, batch, seq);
    if (static_cast<size_t>(k) * seq > c.max_tokens) return invalid("chunk_seqs * seq exceeds the model's max_tokens");
    const uint32_t kk = std::min(k, batch);
    const size_t chunk_T = static_cast<size_t>(kk) * seq;
    const size_t V = c.vocab;
    // two staging slots (tokens + logits); chunk i uses slot i % 2
    if (m->stage_tokens < chunk_T) {
        for (int s = 0; s < 2; ++s) {
            if (m->stage_tok[s]) gpu_hot_free(S.pool, m->stage_tok[s]);
            if (m->stage_logits[s]) gpu_hot_free(S.pool, m->stage_logits[s]);
            m->stage_tok[s] = static_cast<int*>(pool_alloc(S, chunk_T * 4));
            m->stage_logits[s] = static_cast<float*>(pool_alloc(S, chunk_T * V * 4));
        }
        m->stage_tokens = chunk_T;
        if (!m->stage_tok[0] || !m->stage_tok[1] || !m->stage_logits[0] || !m->stage_logits[1]) {
            for (int s = 0; s < 2; ++s) {
                if (m->stage_tok[s]) gpu_hot_free(S.pool, m->stage_tok[s]);
                if (m->stage_logits[s]) gpu_hot_free(S.pool, m->stage_logits[s]);
                m->stage_tok[s] = nullptr;
                m->stage_logits[s] = nullptr;
            }
            m->stage_tokens = 0;
            return internal("staging allocation failed (session pool too small)");
        }
    }
    if (!m->copy_stream && cudaStreamCreateWithFlags(&m->copy_stream, cudaStreamNonBlocking) != cudaSuccess) {
        m->copy_stream = nullptr;
        cudaGetLastError();
        return internal("cudaStreamCreate failed");
    }
    for (int s = 0; s < 2; ++s)
        for (cudaEvent_t* ev : {&m->computed[s], &m->copied[s]})
            if (!*ev && cudaEventCreateWithFlags(ev, cudaEventDisableTiming) != cudaSuccess) {
                *ev = nullptr;
                cudaGetLastError();
                return internal("cudaEventCreate failed");
            }
    const cudaStream_t cs = S.stream, ds = m->copy_stream;
    const uint32_t chunks = (batch + kk - 1) / kk;
    cudaError_t e = cudaSuccess;
    // D2H of chunk i, on the copy stream after its forward; the forward of
    // chunk i+1 is queued first, so it runs under this copy even when the
    // host buffer is pageable (a pageable copy returns only when done)
    auto drain = [&](uint32_t i) {
        const int s = static_cast<int>(i & 1);
        const size_t seqs = std::min<size_t>(kk, batch - static_cast<size_t>(i) * kk);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(ds, m->computed[s], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(host_logits + static_cast<size_t>(i) * chunk_T * V, m->stage_logits[s],
                                seqs * seq * V * 4, cudaMemcpyDeviceToHost, ds);
        if (e == cudaSuccess) e = cudaEventRecord(m->copied[s], ds);
    };
    for (uint32_t i = 0; i < chunks && e == cudaSuccess; ++i) {
        const int s = static_cast<int>(i & 1);
        const size_t seqs = std::min<size_t>(kk, batch - static_cast<size_t>(i) * kk);
        // slot s is free once chunk i-2's logits have left the device
        if (i >= 2) e = cudaStreamWaitEvent(cs, m->copied[s], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(m->stage_tok[s], host_tokens + static_cast<size_t>(i) * chunk_T, seqs * seq * 4,
                                cudaMemcpyHostToDevice, cs);
        if (e == cudaSuccess) e = forward_ptrs(S, m, m->stage_tok[s], m->stage_logits[s], static_cast<int>(seqs),
                                               static_cast<int>(seq));
        if (e == cudaSuccess) e = cudaEventRecord(m->computed[s], cs);
        if (i >= 1) drain(i - 1);
    }
    if (chunks) drain(chunks - 1);
    // the compute stream has nothing queued after the last forward's event,
    // which the last copy waited on: the copy stream finishing means all done
    const cudaError_t w = cudaStreamSynchronize(ds);
    if (e == cudaSuccess) e = w;
    if (e == cudaSuccess) e = cudaStreamSynchronize(cs);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return internal("pipelined forward failed");
    }
    return ok();
}

fer_status_t fer_transformer_profile(fer_session_t* session, uint64_t model, uint32_t enable) {
    if (!session) return invalid("session is null");
    Session& S = session->impl;
    Transformer* m = find_model(S, model);
    if (!m) return not_found("model id not found");
    cudaStreamSynchronize(S.stream);
    m->release_marks();
    m->prof = fer_transformer_profile_t{};
    m->profiling = enable != 0;
    return ok();
}

fer_status_t fer_transformer_profile_read(fer_session_t* session, uint64_t model, fer_transformer_profile_t* out) {
    if (!session || !out) return invalid("session or out is null");
    Session& S = session->impl;
    Transformer* m = find_model(S, model);
    if (!m) return not_found("model id not found");
    if (cudaStreamSynchronize(S.stream) != cudaSuccess) return internal("stream synchronize failed");
    for (const auto& mk : m->marks) {
        float ms = 0.0f;
        if (cudaEventElapsedTime(&ms, mk.a, mk.b) != cudaSuccess) return internal("event timing failed");
        double* slot = mk.cls == 0 ? &m->prof.gemm_ms : mk.cls == 1 ? &m->prof.attn_ms : mk.cls == 2 ? &m->prof.norm_ms
                                                                                         : &m->prof.other_ms;
        *slot += ms;
        if (mk.cls == 0) m->prof.gemm_flops += mk.flops;
        if (mk.cls == 1) m->prof.attn_flops += mk.flops;
        m->prof.launches++;
    }
    m->release_marks();
    *out = m->prof;
    return ok();
}

fer_status_t fer_transformer_kv_create(fer_session_t* session, uint64_t model, uint32_t max_batch, uint32_t max_seq,
                                       uint64_t* out_cache) {
    if (!session || !out_cache) return invalid("session or out_cache is null");
    Session& S = session->impl;
    Transformer* m = find_model(S, model);
    if (!m) return not_found("model id not found");
    if (max_batch == 0 || max_seq == 0) return invalid("kv cache needs max_batch > 0 and max_seq > 0");
    const fer_transformer_config_t& c = m->cfg;
    KvCache kc;
    kc.max_batch = max_batch;
    kc.max_seq = max_seq;
    kc.layer_elems = static_cast<size_t>(max_batch) * c.d_model * max_seq;   // heads * 64 == d_model
    kc.kv = static_cast<uint16_t*>(pool_alloc(S, kc.layer_elems * 2 * c.layers * sizeof(uint16_t)));
    const size_t sf = fer_attn_decode_scratch_floats(static_cast<int>(max_batch), static_cast<int>(c.heads),
                                                     static_cast<int>(max_seq));
    kc.scratch = sf ? static_cast<float*>(pool_alloc(S, sf * sizeof(float))) : nullptr;
    const size_t n_counters = static_cast<size_t>(max_batch) * c.heads;
    kc.attn_counters = static_cast<int*>(pool_alloc(S, n_counters * sizeof(int)));
    {
        const int Mb = static_cast<int>(max_batch), d = static_cast<int>(c.d_model), F = static_cast<int>(c.ffn);
        const int V = static_cast<int>(c.vocab);
        const int shapes[5][2] = {{3 * d, d}, {d, d}, {F, d}, {d, F}, {V, d}};
        for (const auto& nk : shapes) {
            const size_t b = fer_gemm_splitk_workspace_bytes(Mb, nk[0], nk[1]);
            if (b > kc.gemm_ws_bytes) kc.gemm_ws_bytes = b;
        }
        kc.gemm_ws = static_cast<float*>(pool_alloc(S, kc.gemm_ws_bytes));
    }
    kc.d_len = static_cast<int*>(pool_alloc(S, sizeof(int)));
    kc.tok_stage = static_cast<int*>(pool_alloc(S, static_cast<size_t>(max_batch) * sizeof(int)));
    kc.logit_stage = static_cast<float*>(pool_alloc(S, static_cast<size_t>(max_batch) * c.vocab * sizeof(float)));
    if (!kc.kv || (sf && !kc.scratch) || !kc.attn_counters || !kc.gemm_ws || !kc.d_len || !kc.tok_stage ||
        !kc.logit_stage) {
        m->free_cache(kc);
        return internal("kv cache allocation failed");
    }
    if (fer_device_int_set(kc.d_len, 0, S.stream) != cudaSuccess ||
        cudaMemsetAsync(kc.attn_counters, 0, n_counters * sizeof(int), S.stream) != cudaSuccess) {
        cudaGetLastError();
        m->free_cache(kc);
        return internal("kernel launch failed");
    }
    const uint64_t id = S.next_model++;
    m->caches.emplace(id, kc);
    *out_cache = id;
    return ok();
}

fer_status_t fer_transformer_kv_destroy(fer_session_t* session, uint64_t model, uint64_t cache) {
    if (!session) return invalid("session is null");
    Session& S = session->impl;
    Transformer* m = find_model(S, model);
    if (!m) return not_found("model id not found");
    auto it = m->caches.find(cache);
    if (it == m->caches.end()) return not_found("kv cache id not found");
    cudaStreamSynchronize(S.stream);
    m->free_cache(it->second);
    m->caches.erase(it);
    return ok();
}

fer_status_t fer_transformer_kv_length(fer_session_t* session, uint64_t model, uint64_t cache, uint32_t* out_batch,
                                       uint32_t* out_len) {
    if (!session) return invalid("session is null");
    Transformer* m = find_model(session->impl, model);
    if (!m) return not_found("model id not found");
    auto it = m->caches.find(cache);
    if (it == m->caches.end()) return not_found("kv cache id not found");
    if (out_batch) *out_batch = it->second.batch;
    if (out_len) *out_len = it->second.len;
    return ok();
}

// The forward over a prompt that also fills the cache (positions 0 .. S-1 of
// sequences 0 .. B-1). logits: f32 [B, S, vocab], or [B, vocab] for the last
// position of each sequence only.
fer_status_t fer_transformer_prefill(fer_session_t* session, uint64_t model, uint64_t cache, uint64_t tokens,
                                     uint64_t logits, uint64_t* out_job_id) {
    if (!session) return invalid("session is null");
    Session& S = session->impl;
    Transformer* m = find_model(S, model);
    if (!m) return not_found("model id not found");
    auto cit = m->caches.find(cache);
    if (cit == m->caches.end()) return not_found("kv cache id not found");
    KvCache& kc = cit->second;
    const Buffer* tb = S.find(tokens);
    const Buffer* lb = S.find(logits);
    if (!tb || !lb) return not_found("buffer id not found");
    if (tb->desc.dtype != FER_DTYPE_I32 || (tb->desc.rank != 1 && tb->desc.rank != 2))
        return invalid("tokens must be i32 [batch, seq] or [seq]");
    const int B = tb->desc.rank == 2 ? static_cast<int>(tb->desc.dims[0]) : 1;
    const int Sq = tb->desc.rank == 2 ? static_cast<int>(tb->desc.dims[1]) : static_cast<int>(tb->desc.dims[0]);
    const size_t T = static_cast<size_t>(B) * Sq;
    const fer_transformer_config_t& c = m->cfg;
    if (T > c.max_tokens) return invalid("batch * seq exceeds the model's max_tokens");
    if (static_cast<uint32_t>(B) > kc.max_batch || static_cast<uint32_t>(Sq) > kc.max_seq)
        return invalid("prompt exceeds the kv cache");
    const bool last_only = lb->numel == static_cast<size_t>(B) * c.vocab;
    if (lb->desc.dtype != FER_DTYPE_F32 || !(last_only || lb->numel == T * c.vocab))
        return invalid("logits must be f32 [batch, seq, vocab] or [batch, vocab]");
    const int d = static_cast<int>(c.d_model), F = static_cast<int>(c.ffn), V = static_cast<int>(c.vocab);
    const int H = static_cast<int>(c.heads), Ti = static_cast<int>(T);
    cudaStream_t st = S.stream;
    uint32_t* err = S.dev_err;
    const uint16_t* W = m->W;
    cudaError_t e = cudaSuccess;
    for (uint32_t l = 0; l < c.layers && e == cudaSuccess; ++l) {
        const float* g1 = m->ln + (4 * l + 0) * static_cast<size_t>(d);
        const float* b1 = m->ln + (4 * l + 1) * static_cast<size_t>(d);
        const float* g2 = m->ln + (4 * l + 2) * static_cast<size_t>(d);
        const float* b2 = m->ln + (4 * l + 3) * static_cast<size_t>(d);
        uint16_t* kcache = kc.kv + 2 * l * kc.layer_elems;
        uint16_t* vcache = kcache + kc.layer_elems;
        e = l == 0 ? fer_embed_ln_bf16(static_cast<const int*>(tb->ptr), W + m->off_emb, m->x, g1, b1, m->a, Ti, d, V,
                                       c.eps, err, st)
                   : fer_ln_bf16(m->x, g1, b1, m->a, Ti, d, c.eps, st);
        if (e == cudaSuccess)
            e = fer_gemm_bf16_tc_ex(m->a, W + m->off_qkv[l], m->qkv, nullptr, Ti, 3 * d, d, kEpiBF16, err, st);
        if (e == cudaSuccess)
            e = fer_kv_store(m->qkv, kcache, vcache, B, Sq, d, H, static_cast<int>(kc.max_seq), 0, st);
        if (e == cudaSuccess) e = fer_attn_causal_ex(m->qkv, m->att, B, Sq, d, H, 0, err, st);
        if (e == cudaSuccess)
            e = fer_gemm_bf16_tc_ex(m->att, W + m->off_o[l], m->x, m->x, Ti, d, d, kEpiResidF32, err, st);
        if (e == cudaSuccess) e = fer_ln_bf16(m->x, g2, b2, m->a, Ti, d, c.eps, st);
        if (e == cudaSuccess)
            e = fer_gemm_bf16_tc_ex(m->a, W + m->off_w1[l], m->hid, nullptr, Ti, F, d, kEpiGeluBF16, err, st);
        if (e == cudaSuccess)
            e = fer_gemm_bf16_tc_ex(m->hid, W + m->off_w2[l], m->x, m->x, Ti, d, F, kEpiResidF32, err, st);
    }
    const float* gf = m->ln + (4 * static_cast<size_t>(c.layers)) * d;
    if (e == cudaSuccess) e = fer_ln_bf16(m->x, gf, gf + d, m->a, Ti, d, c.eps, st);
    if (e == cudaSuccess) {
        if (last_only) {
            // rows b * S + S - 1 of the final-LN output, then the LM head on B rows
            e = cudaMemcpy2DAsync(m->att, static_cast<size_t>(d) * 2, m->a + static_cast<size_t>(Sq - 1) * d,
                                  static_cast<size_t>(Sq) * d * 2, static_cast<size_t>(d) * 2, B,
                                  cudaMemcpyDeviceToDevice, st);
            if (e == cudaSuccess)
                e = fer_gemm_bf16_tc_ex(m->att, W + m->off_lm, lb->ptr, nullptr, B, V, d, kEpiF32, err, st);
        } else {
            e = fer_gemm_bf16_tc_ex(m->a, W + m->off_lm, lb->ptr, nullptr, Ti, V, d, kEpiF32, err, st);
        }
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return internal("kernel launch failed");
    }
    if (fer_device_int_set(kc.d_len, Sq, st) != cudaSuccess) {
        cudaGetLastError();
        return internal("kernel launch failed");
    }
    kc.batch = static_cast<uint32_t>(B);
    kc.len = static_cast<uint32_t>(Sq);
    return S.make_job({}, out_job_id);
}

// One step of incremental decoding: token b (i32 [B]) appended to sequence
// b of the cache at position len, attending to positions 0 .. len; logits
// f32 [B, vocab]. The cache's len advances by one.
fer_status_t fer_transformer_decode(fer_session_t* session, uint64_t model, uint64_t cache, uint64_t tokens,
                                    uint64_t logits, uint64_t* out_job_id) {
    if (!session) return invalid("session is null");
    Session& S = session->impl;
    Transformer* m = find_model(S, model);
    if (!m) return not_found("model id not found");
    auto cit = m->caches.find(cache);
    if (cit == m->caches.end()) return not_found("kv cache id not found");
    KvCache& kc = cit->second;
    const Buffer* tb = S.find(tokens);
    const Buffer* lb = S.find(logits);
    if (!tb || !lb) return not_found("buffer id not found");
    const fer_transformer_config_t& c = m->cfg;
    if (tb->desc.dtype != FER_DTYPE_I32 || tb->numel != kc.batch || kc.batch == 0)
        return invalid("decode takes one i32 token per sequence of the prefilled cache");
    if (lb->desc.dtype != FER_DTYPE_F32 || lb->numel != static_cast<size_t>(kc.batch) * c.vocab)
        return invalid("logits must be f32 [batch, vocab]");
    if (kc.len >= kc.max_seq) return invalid("kv cache is full");
    const int B = static_cast<int>(kc.batch);
    const int d = static_cast<int>(c.d_model), F = static_cast<int>(c.ffn), V = static_cast<int>(c.vocab);
    const int H = static_cast<int>(c.heads), max_seq = static_cast<int>(kc.max_seq);
    cudaStream_t st = S.stream;
    uint32_t* err = S.dev_err;
    const uint16_t* W = m->W;
    // M = B rows: split-K GEMMs, so that a short batch still spreads each
    // weight matrix over the whole GPU. The position lives in kc.d_len on
    // the device and every buffer address is fixed, so the whole step is
    // captured once per batch size and replayed (first call eager).
    auto gemm = [&](const void* a, const void* b, void* cc, int N, int K, int epi) {
        return fer_gemm_bf16_tc_splitk(a, b, cc, B, N, K, epi, 0, kc.gemm_ws, kc.gemm_ws_bytes, 1, err, st);
    };
    cudaError_t e = cudaSuccess;
    auto issue = [&]() {
        for (uint32_t l = 0; l < c.layers && e == cudaSuccess; ++l) {
            const float* g1 = m->ln + (4 * l + 0) * static_cast<size_t>(d);
            const float* b1 = m->ln + (4 * l + 1) * static_cast<size_t>(d);
            const float* g2 = m->ln + (4 * l + 2) * static_cast<size_t>(d);
            const float* b2 = m->ln + (4 * l + 3) * static_cast<size_t>(d);
            uint16_t* kcache = kc.kv + 2 * l * kc.layer_elems;
            uint16_t* vcache = kcache + kc.layer_elems;
            e = l == 0 ? fer_embed_ln_bf16(kc.tok_stage, W + m->off_emb, m->x, g1, b1, m->a, B, d, V, c.eps, err, st)
                       : fer_ln_bf16(m->x, g1, b1, m->a, B, d, c.eps, st);
            if (e == cudaSuccess) e = gemm(m->a, W + m->off_qkv[l], m->qkv, 3 * d, d, kEpiBF16);
            if (e == cudaSuccess)
                e = fer_decode_kv_attention(m->qkv, kcache, vcache, m->att, kc.scratch, kc.attn_counters, B, d, H,
                                            max_seq, kc.d_len, err, st);
            if (e == cudaSuccess) e = gemm(m->att, W + m->off_o[l], m->x, d, d, kEpiResidF32);
            if (e == cudaSuccess) e = fer_ln_bf16(m->x, g2, b2, m->a, B, d, c.eps, st);
            if (e == cudaSuccess) e = gemm(m->a, W + m->off_w1[l], m->hid, F, d, kEpiGeluBF16);
            if (e == cudaSuccess) e = gemm(m->hid, W + m->off_w2[l], m->x, d, F, kEpiResidF32);
        }
        const float* gf = m->ln + (4 * static_cast<size_t>(c.layers)) * d;
        if (e == cudaSuccess) e = fer_ln_bf16(m->x, gf, gf + d, m->a, B, d, c.eps, st);
        if (e == cudaSuccess) e = gemm(m->a, W + m->off_lm, kc.logit_stage, V, d, kEpiF32);
        if (e == cudaSuccess) e = fer_device_int_add(kc.d_len, 1, st);
    };
    e = cudaMemcpyAsync(kc.tok_stage, tb->ptr, static_cast<size_t>(B) * sizeof(int), cudaMemcpyDeviceToDevice, st);
    static const int graphs_env = [] {
        const char* ev = std::getenv("FERCUDA_XFMR_GRAPH");
        return (ev && ev[0] == '0') ? 0 : 1;
    }();
    const bool use_graph = graphs_env && !m->profiling && !m->graphs_off;
    if (e == cudaSuccess) {
        if (use_graph && kc.graph && kc.graph_batch == kc.batch) {
            e = cudaGraphLaunch(kc.graph, st);
        } else if (use_graph && kc.eager_batch == kc.batch) {
            if (kc.graph) {
                cudaGraphExecDestroy(kc.graph);
                kc.graph = nullptr;
            }
            cudaGraph_t graph = nullptr;
            if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
                issue();
                const cudaError_t ce = cudaStreamEndCapture(st, &graph);
                if (e == cudaSuccess && ce == cudaSuccess && graph &&
                    cudaGraphInstantiate(&kc.graph, graph, 0) != cudaSuccess)
                    kc.graph = nullptr;
                if (graph) cudaGraphDestroy(graph);
                if (e != cudaSuccess || ce != cudaSuccess || !kc.graph) {
                    cudaGetLastError();
                    m->graphs_off = true;   // stay eager from now on
                    kc.graph = nullptr;
                    issue();
                } else {
                    kc.graph_batch = kc.batch;
                    e = cudaGraphLaunch(kc.graph, st);
                }
            } else {
                cudaGetLastError();
                m->graphs_off = true;
                issue();
            }
        } else {
            issue();
            kc.eager_batch = kc.batch;
        }
    }
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(lb->ptr, kc.logit_stage, static_cast<size_t>(B) * V * sizeof(float),
                            cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return internal("kernel launch failed");
    }
    kc.len += 1;
    return S.make_job({}, out_job_id);
}

fer_status_t fer_transformer_destroy(fer_session_t* session, uint64_t model) {
    if (!session) return invalid("session is null");
    Session& S = session->impl;
    auto it = S.models.find(model);
    if (it == S.models.end()) return not_found("model id not found");
    cudaStreamSynchronize(S.stream);
    S.models.erase(it);
    return ok();
}

}  // extern "C"
