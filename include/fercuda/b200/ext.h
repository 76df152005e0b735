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
 * Numerics match the reference's ptx_tensor_softmax_f32 and
 * fer_submit_layer_norm applied row by row, bit for bit.
 * gamma / beta: optional rank-1 f32 [cols] buffers (0 = none). */
#define FER_ROWS_SOFTMAX 1u
#define FER_ROWS_LAYER_NORM 2u

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
