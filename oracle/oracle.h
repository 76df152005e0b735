/*
 * ORACLE — test infrastructure only. A CPU restatement of the reference
 * (DaronPopov/feRcuda) algorithms on the hot path, used by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline / --impl reference
 * legs as the checker and CPU baseline. Nothing in the product links it.
 *
 * Every function names the reference file:line it restates. Floating-point
 * functions keep the reference's operation order and rounding steps (no FMA
 * contraction: built with -ffp-contract=off), so results are bit-identical to
 * the reference kernels except where the reference calls a CUDA transcendental
 * (expf, rsqrtf): glibc's expf / 1/sqrtf differ from CUDA's by a few ULP.
 * Pinning: tests/test_oracle.py checks these functions against the golden
 * vectors of the reference's own tests and, where the reference compiles
 * here, against oracle/_ref built from the reference sources.
 */
#ifndef FERCUDA_ORACLE_H
#define FERCUDA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* y = relu(x*a + b) * sigmoid(x), the reference's 4-kernel composition. */
void orc_chain_f32(const float* x, float* y, size_t n, float a, float b, int threads);
/* JIT affine intent: v = fmaf(alpha, in, beta); if (relu && v < 0) v = 0. */
void orc_affine_intent_f32(const float* x, float* y, size_t n, float alpha, float beta, int relu);
/* Row softmax in the reference kernel's 256-thread reduction order. */
void orc_softmax_rows_f32(const float* x, float* y, size_t rows, size_t cols, int threads);
/* Rank-1 layer norm in the reference kernel's reduction order. */
void orc_layer_norm_f32(const float* x, float* y, size_t n, float eps);
/* softmax then layer norm per row (gamma = 1, beta = 0). */
void orc_softmax_layernorm_rows_f32(const float* x, float* y, size_t rows, size_t cols, float eps, int threads);
/* C = A.B with one sequential fmaf chain per output, f32. Rows [r0, r1). */
void orc_matmul_f32(const float* A, const float* B, float* C, int M, int K, int N, int r0, int r1, int threads);
/* Same chain on bf16 operands upcast to f32; computes only the output tile
 * rows [r0,r1) x cols [c0,c1), written densely into C (ld = c1-c0). */
void orc_matmul_bf16_tile(const uint16_t* A, const uint16_t* B, float* C, int M, int K, int N,
                          int r0, int r1, int c0, int c1);

/* TLSF restatement (reference tlsf_allocator_internals.inl + api.inl):
 * offsets into a pool of pool_size bytes; alloc returns UINT64_MAX on failure. */
typedef struct orc_tlsf orc_tlsf;
orc_tlsf* orc_tlsf_create(uint64_t pool_size);
void orc_tlsf_destroy(orc_tlsf* t);
uint64_t orc_tlsf_alloc(orc_tlsf* t, uint64_t size);
int orc_tlsf_free(orc_tlsf* t, uint64_t off);
uint64_t orc_tlsf_allocated_bytes(const orc_tlsf* t);
uint32_t orc_tlsf_block_count(const orc_tlsf* t);

#ifdef __cplusplus
}
#endif

#endif
