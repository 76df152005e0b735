/*
 * fercuda B200 extensions to the C ABI. Everything here is additive: new
 * entry points and structs that the reference does not have, in
 * libfercuda_capi.so next to the reference-compatible ones.
 */
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "fercuda/api/c_api.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- row kernels ----------------------------------------------------------
 * Row softmax, row layer norm, or softmax followed by layer norm over a
 * rank-2 f32 buffer [rows, cols] (rank 1 = one row), in one fused pass.
 * By default numerics match the reference's ptx_tensor_softmax_f32 and
 * fer_submit_layer_norm applied row by row, bit for bit.
 * FER_ROWS_FAST selects a one-pass path with 128-bit accesses and an SFU
 * exponential: bit-identical run to run, within 1e-5 (of the largest output)
 * of the reference order; shapes it does not take (cols % 4 != 0,
 * cols > 8192, in place, unaligned) run the reference-order path.
 * gamma / beta: optional rank-1 f32 [cols] buffers (0 = none). */
#define FER_ROWS_SOFTMAX 1u
#define FER_ROWS_LAYER_NORM 2u
#define FER_ROWS_FAST 4u

typedef struct fer_rows_request {
    uint64_t x;
    uint64_t out;
    uint64_t gamma;
    uint64_t beta;
    float eps;
    uint32_t ops;            /* FER_ROWS_* bits */
    uint32_t memory_regime;
} fer_rows_request_t;

fer_status_t fer_submit_rows(fer_session_t* session, const fer_rows_request_t* req, uint64_t* out_job_id);

/* ---- fused elementwise chains ---------------------------------------------
 * A chain is a short stack program over f32 streams of equal length. Each op
 * follows the reference kernel of the same name, rounding step for rounding
 * step (no FMA contraction). The JIT emits one vectorised kernel per distinct
 * opcode sequence, compiles it once with NVRTC for the device, caches it in
 * memory (and on disk when FERCUDA_JIT_CACHE_DIR is set) and launches it;
 * scalar operands are kernel arguments, so new scalars need no recompile. */
typedef enum fer_chain_opcode {
    FER_CHAIN_LOAD = 0,        /* push input[arg] */
    FER_CHAIN_AFFINE = 1,      /* v = v * p0 + p1   (k_affine_f32) */
    FER_CHAIN_ADD_SCALAR = 2,  /* v = v + p0 */
    FER_CHAIN_MUL_SCALAR = 3,  /* v = v * p0 */
    FER_CHAIN_RELU = 4,        /* v = fmaxf(0, v)   (k_relu_f32) */
    FER_CHAIN_SIGMOID = 5,     /* v = 1 / (1 + expf(-v)) */
    FER_CHAIN_EXP = 6,         /* v = expf(v) */
    FER_CHAIN_TANH = 7,        /* v = tanhf(v) */
    FER_CHAIN_GELU_TANH = 8,   /* k_gelu_f32 tanh form */
    FER_CHAIN_SILU = 9,        /* v = v / (1 + expf(-v)) */
    FER_CHAIN_NEG = 10,
    FER_CHAIN_ABS = 11,
    FER_CHAIN_CLAMP = 12,      /* v = fminf(p1, fmaxf(p0, v)) */
    FER_CHAIN_ADD = 13,        /* pop b, pop a, push a + b */
    FER_CHAIN_SUB = 14,        /* a - b */
    FER_CHAIN_MUL = 15,        /* a * b */
    FER_CHAIN_DIV = 16,        /* a / b */
    FER_CHAIN_MAX = 17,        /* fmaxf(a, b) */
    FER_CHAIN_MIN = 18,        /* fminf(a, b) */
    FER_CHAIN_RELU_LT = 19,    /* v = v < 0 ? 0 : v   (JIT affine intent relu) */
    FER_CHAIN_FMA = 20,        /* v = fmaf(v, p0, p1), one rounding (JIT affine intent) */
    FER_CHAIN_OPCODE_COUNT = 21
} fer_chain_opcode_t;

typedef struct fer_chain_op {
    uint32_t opcode;
    uint32_t arg;      /* FER_CHAIN_LOAD: input index */
    float p0;
    float p1;
} fer_chain_op_t;

#define FER_CHAIN_MAX_OPS 32
#define FER_CHAIN_MAX_INPUTS 4

/* Runs out[i] = chain(inputs[0][i], ...) for i < numel(out). All buffers f32
 * with the same element count. Leaves exactly one value on the stack. */
fer_status_t fer_jit_run_chain_f32(fer_session_t* session, const fer_chain_op_t* ops, uint32_t n_ops,
                                   const uint64_t* inputs, uint32_t n_inputs, uint64_t output,
                                   uint64_t* out_job_id);

/* ---- deterministic tensor-core GEMM ---------------------------------------
 * out[M,N] = a[M,K] . b[K,N], bf16 operands, f32 accumulation in tensor
 * memory (tcgen05), fixed K order, no split-K: bit-identical run to run.
 * out dtype f32 or bf16 (round to nearest even). Row-major buffers; K and N
 * multiples of 8. Other shapes take the CUDA-core kernel with the reference's
 * sequential accumulation order (also deterministic). */
typedef struct fer_gemm_request {
    uint64_t a;
    uint64_t b;
    uint64_t out;
    uint32_t flags;          /* reserved, 0 */
    uint32_t memory_regime;
} fer_gemm_request_t;

fer_status_t fer_submit_gemm(fer_session_t* session, const fer_gemm_request_t* req, uint64_t* out_job_id);

/* ---- decoder-only transformer forward --------------------------------------
 * Pre-LN blocks (LN -> QKV -> causal multi-head attention -> out-proj +
 * residual -> LN -> W1 -> exact GELU -> W2 + residual), final LN, LM head;
 * token embedding, no biases, no positional embedding. Weights bf16, f32
 * residual stream and accumulation, logits f32. head_dim must be 64,
 * d_model a multiple of 256, ffn and vocab multiples of 8.
 * All weights live in one session buffer (bf16, rank 1) so a caller can
 * download it or broadcast it to other GPUs; layout, in elements, each
 * tensor starting at a multiple of 128: embedding [vocab, d], then per layer
 * Wqkv [d, 3d], Wo [d, d], W1 [d, ffn], W2 [ffn, d], then LM head [d, vocab]
 * (x @ W convention, row-major). Layer-norm gamma / beta are f32, 1 and 0. */
typedef struct fer_transformer_config {
    uint32_t layers;
    uint32_t d_model;
    uint32_t heads;
    uint32_t ffn;
    uint32_t vocab;
    uint32_t max_tokens;     /* largest batch*seq a forward may take (workspace size) */
    float eps;
    uint32_t reserved;
} fer_transformer_config_t;

fer_status_t fer_transformer_create(fer_session_t* session, const fer_transformer_config_t* cfg, uint64_t* out_model);
/* Fills every weight with N(0, stddev) bf16 from `seed` (device-side
 * splitmix64 + Box-Muller; element i of the weight buffer uses draws 2i+1 and
 * 2i+2 of the seed's stream) and resets gamma to 1, beta to 0. */
fer_status_t fer_transformer_init_weights(fer_session_t* session, uint64_t model, uint64_t seed, float stddev);
/* Buffer id of the model's weight buffer (bf16, rank 1). */
fer_status_t fer_transformer_weight_buffer(fer_session_t* session, uint64_t model, uint64_t* out_buffer_id);
/* tokens: i32 [batch, seq] (or [seq]); logits: f32 [batch, seq, vocab] (or
 * [batch*seq, vocab]). Sequences are independent (causal within each). */
fer_status_t fer_transformer_forward(fer_session_t* session, uint64_t model, uint64_t tokens, uint64_t logits,
                                     uint64_t* out_job_id);
/* The forward from host memory to host memory, pipelined: host_tokens i32
 * [batch, seq] in, host_logits f32 [batch, seq, vocab] out. The batch runs in
 * chunks of chunk_seqs sequences (0: at most about 4096 tokens and at least
 * four chunks where the batch allows; chunk_seqs x seq <= max_tokens); the logits of chunk i are copied to the host on a
 * second stream while chunk i+1 computes, through two staging slots the model
 * keeps (2 x chunk tokens x vocab x 4 bytes of the session pool). Returns
 * when every logit is in host_logits; bit-identical to fer_transformer_forward
 * of the whole batch followed by a download. Pinned host memory gives the
 * full PCIe rate; pageable memory works too. */
fer_status_t fer_transformer_forward_host(fer_session_t* session, uint64_t model, const int32_t* host_tokens,
                                          uint32_t batch, uint32_t seq, float* host_logits, uint32_t chunk_seqs);
fer_status_t fer_transformer_destroy(fer_session_t* session, uint64_t model);

/* ---- batch-sharded forward over the GPUs of one node ------------------------
 * One process (or host thread) per GPU, each with its own session. The root
 * rank makes the weights (fer_transformer_init_weights); one NCCL broadcast
 * over NVLink / NVSwitch copies them into every rank's weight buffer in
 * place; then each rank runs fer_transformer_forward on its contiguous shard
 * of the global batch, with no collective inside a forward (sequences never
 * interact, so the logits are bit-identical to a one-GPU forward of the
 * whole batch). Replaces the reference's gpu_broadcast_tensor
 * (native/core/runtime/modules/hot_multi_gpu_policy_main.inl:221-249), a
 * serial cudaMemcpyPeer from the source GPU to each other GPU of one process.
 *
 * fer_comm_unique_id: on one rank; the caller hands the 128 bytes to every
 * rank (any host channel). fer_comm_init: every rank, with the same id, its
 * rank and the world size; binds an NCCL communicator to the session's
 * device (released by fer_comm_destroy or fer_session_destroy). Waits are
 * bounded by timeout_ms (0: 120 s): a rank that never joins, or a broadcast
 * that does not finish, returns FER_STATUS_INTERNAL_ERROR (the communicator
 * is aborted) instead of hanging. NCCL is opened at the first call
 * (FERCUDA_NCCL_LIBRARY, else libnccl.so.2: the copy already loaded, if the
 * process has one). A process that also loads another NCCL-linked library
 * (PyTorch) should load that one first, so that one copy serves both. */
#define FER_COMM_UNIQUE_ID_BYTES 128
fer_status_t fer_comm_unique_id(uint8_t* out_id);
fer_status_t fer_comm_init(fer_session_t* session, const uint8_t* id, int32_t rank, int32_t world,
                           uint32_t timeout_ms);
fer_status_t fer_comm_destroy(fer_session_t* session);
/* Broadcasts the model's weight buffer from `root` into every rank's, in
 * place, ordered after the work queued on the session stream; returns when
 * it has completed. Every rank calls it with the same root. */
fer_status_t fer_transformer_broadcast_weights(fer_session_t* session, uint64_t model, int32_t root,
                                               uint64_t* out_bytes);
/* Rank's shard of a global batch: sequences [*out_first, *out_first +
 * *out_count); the batch must split evenly. */
fer_status_t fer_transformer_shard(uint32_t global_batch, int32_t world, int32_t rank, uint32_t* out_first,
                                   uint32_t* out_count);
/* 64-bit digest of each of `rows` consecutive rows of row_bytes bytes (a
 * multiple of 16) of a buffer: the sum mod 2^64 of a mixing hash of every
 * 16-byte chunk and its position within the row, so it depends only on the
 * row's bytes (not on the row's index or the order of summation). Used to
 * compare logits across ranks and GPU counts bit for bit. Synchronous;
 * rows <= 65535 per call. */
fer_status_t fer_buffer_row_digests(fer_session_t* session, uint64_t buffer, uint64_t row_bytes, uint32_t rows,
                                    uint64_t* out_digests);

/* ---- KV cache and incremental decoding --------------------------------------
 * A KV cache of a model holds, per layer, the keys and values of up to
 * max_batch sequences x max_seq positions (bf16, [max_batch][heads][max_seq][64]
 * for K and for V), from the session pool. prefill runs the forward over a
 * prompt (tokens i32 [batch, seq]) and stores its keys and values at
 * positions 0 .. seq-1; logits f32 [batch, seq, vocab], or [batch, vocab] for
 * each sequence's last position. decode appends one token per sequence
 * (tokens i32 [batch], batch as prefilled) at position len, attends to
 * positions 0 .. len and writes logits f32 [batch, vocab]; len advances by
 * one. Decode attention is split over 256-position chunks and combined in
 * chunk order: bit-identical run to run. The cache ids share the model id
 * space; destroying the model frees its caches. */
fer_status_t fer_transformer_kv_create(fer_session_t* session, uint64_t model, uint32_t max_batch, uint32_t max_seq,
                                       uint64_t* out_cache);
fer_status_t fer_transformer_kv_destroy(fer_session_t* session, uint64_t model, uint64_t cache);
/* Sequences and positions currently held (both 0 before the first prefill). */
fer_status_t fer_transformer_kv_length(fer_session_t* session, uint64_t model, uint64_t cache, uint32_t* out_batch,
                                       uint32_t* out_len);
fer_status_t fer_transformer_prefill(fer_session_t* session, uint64_t model, uint64_t cache, uint64_t tokens,
                                     uint64_t logits, uint64_t* out_job_id);
fer_status_t fer_transformer_decode(fer_session_t* session, uint64_t model, uint64_t cache, uint64_t tokens,
                                    uint64_t logits, uint64_t* out_job_id);

/* Per-kernel-class timing of forwards: while enabled, every forward records a
 * CUDA event pair around each of its launches on the session stream; reading
 * synchronises the stream and sums the elapsed times. Enabling resets. */
typedef struct fer_transformer_profile {
    double gemm_ms;          /* tensor-core GEMMs (QKV, out-proj, W1, W2, LM head) */
    double attn_ms;          /* causal attention */
    double norm_ms;          /* layer norms */
    double other_ms;         /* embedding */
    double gemm_flops;       /* 2*M*N*K summed over the GEMM launches timed */
    double attn_flops;       /* causal attention flops (QK^T and PV over unmasked pairs) */
    uint64_t forwards;
    uint64_t launches;
} fer_transformer_profile_t;

fer_status_t fer_transformer_profile(fer_session_t* session, uint64_t model, uint32_t enable);
fer_status_t fer_transformer_profile_read(fer_session_t* session, uint64_t model, fer_transformer_profile_t* out);

/* ---- diagnostics ------------------------------------------------------------ */

/* Error bits that kernels of this session reported (bounded waits that ran
 * out, shapes a kernel refused). Reads them after synchronising the session
 * stream; clears them when `clear` is nonzero. */
fer_status_t fer_session_device_errors(fer_session_t* session, uint32_t* out_bits, uint8_t clear);

typedef struct fer_pool_stats {
    uint64_t pool_bytes;
    uint64_t allocated_bytes;
    uint64_t peak_allocated_bytes;
    uint64_t largest_free_block;
    uint64_t total_allocations;
    uint64_t total_frees;
    uint32_t allocated_blocks;
    uint32_t free_blocks;
} fer_pool_stats_t;

/* Statistics of the session's TLSF pool (FER_MEMORY_CUSTOM_POOL). */
fer_status_t fer_pool_get_stats(fer_session_t* session, fer_pool_stats_t* out_stats);

/* Raw pool access for host-side stress work: one TLSF alloc / free without a
 * buffer record. The block comes from the session pool (256-byte aligned). */
fer_status_t fer_pool_alloc_raw(fer_session_t* session, uint64_t bytes, void** out_ptr);
fer_status_t fer_pool_free_raw(fer_session_t* session, void* ptr);

#ifdef __cplusplus
}
#endif
