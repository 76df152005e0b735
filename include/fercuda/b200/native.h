/*
 * Native launchers of libptx_kernels.so beyond the reference's tensor-op ABI.
 * No reference counterpart: these are the kernels the session layer
 * (libfercuda_capi.so) and the transformer driver call, exported so C/C++
 * callers that manage their own device memory can use them directly.
 *
 * Every launcher queues work on `stream` and returns without synchronising;
 * a non-cudaSuccess return means nothing was launched (argument errors are
 * cudaErrorInvalidValue, shapes a kernel does not take cudaErrorNotSupported).
 * `err` (may be null) is a device word the kernels OR error bits into:
 * 1 a bulk copy did not land within about one second, 2 a tensor-core commit
 * did not arrive in time, 4 a shape the kernel cannot take, 8 a producer /
 * consumer hand-off timed out.
 */
#ifndef FERCUDA_B200_NATIVE_H
#define FERCUDA_B200_NATIVE_H

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- GEMM on the tensor cores (tcgen05) ------------------------------------
 * C[M,N] = A[M,K] . B[K,N], A and B row-major bf16, f32 accumulation, fixed K
 * order, no split-K: bit-identical run to run. K % 8 == 0, N % 8 == 0, all
 * pointers 16-byte aligned.
 * epi: 0 C f32; 1 C bf16; 2 C bf16 = GELU(acc) (erf form); 3 C f32 =
 * resid + acc (resid == c adds in place; another resid is copied into c first
 * and must not partly overlap it). */
cudaError_t fer_gemm_bf16_tc_ex(const void* a, const void* b, void* c, const float* resid, int M, int N, int K,
                                int epi, uint32_t* err, cudaStream_t stream);
/* out_dtype: 0 f32, 2 bf16 (fer_buffer_dtype_t codes). */
cudaError_t fer_gemm_bf16_tc(const void* a, const void* b, void* c, int M, int N, int K, uint32_t out_dtype,
                             uint32_t* err, cudaStream_t stream);
/* Split-K form for short M (decode steps): K split into ranges of 64-deep
 * blocks computed by separate CTAs, partials added in range order before
 * `epi` (for epi 3 the residual is c). Deterministic; the additions are
 * grouped differently from fer_gemm_bf16_tc_ex.
 * splits <= 0: cluster form, one cluster of fer_gemm_splitk_cluster_splits()
 * CTAs per output tile adding the partials through distributed shared memory
 * in one kernel (ws unused), or the single-pass kernel when that is 1.
 * splits > 0 (or FERCUDA_SPLITK_CLUSTER=0): partials in the f32 workspace
 * `ws`, added by a second kernel; the count is reduced to fit ws_bytes.
 * Both forms give the same bits for the same split count.
 * flags bit 0: b is not written by the kernel just before this call on the
 * stream (weights); its first tiles are then fetched before the programmatic
 * launch wait, overlapping that kernel.
 * fer_gemm_splitk_workspace_bytes: ws for the workspace form's automatic count. */
size_t fer_gemm_splitk_workspace_bytes(int M, int N, int K);
int fer_gemm_splitk_cluster_splits(int M, int N, int K);
cudaError_t fer_gemm_bf16_tc_splitk(const void* a, const void* b, void* c, int M, int N, int K, int epi, int splits,
                                    float* ws, size_t ws_bytes, int flags, uint32_t* err, cudaStream_t stream);
/* 0 (default): 2-CTA cluster kernel for M > 128; 1: single-CTA kernel. Both
 * give the same bits. Process-wide. */
void fer_gemm_tc_set_mode(int mode);
/* 2-CTA clusters the GEMM launches at most (-1 before its first 2-CTA call). */
int fer_gemm_tc_clusters(void);

/* ---- reference-order matmul (CUDA cores) ----------------------------------
 * One sequential fmaf chain over K per output, the reference k_matmul_f32
 * order (src/runtime/ops_bridge.cu:13-31). dtype: fer_buffer_dtype_t of all
 * three matrices (f32, f16, bf16, i8, u8; computed in f32). */
cudaError_t fer_matmul_ref_order(const void* a, const void* b, void* c, int M, int K, int N, uint32_t dtype,
                                 cudaStream_t stream);
cudaError_t fer_matmul_bf16_f32_ref_order(const void* a, const void* b, float* c, int M, int K, int N,
                                          cudaStream_t stream);
/* Element casts used by the session layer's staging (dtype as above). */
cudaError_t fer_cast_to_f32(const void* in, float* out, size_t n, uint32_t dtype, cudaStream_t s);
cudaError_t fer_cast_from_f32(const float* in, void* out, size_t n, uint32_t dtype, cudaStream_t s);

/* ---- row kernels -------------------------------------------------------------
 * flags: 1 softmax, 2 layer norm, 3 softmax then layer norm; gamma / beta
 * optional [cols] f32. fer_rows_f32: bit-identical to the reference kernels.
 * fer_rows_fast_f32: deterministic, within 1e-5 of the largest output of the
 * reference order; cudaErrorNotSupported for cols % 4 != 0, cols > 8192,
 * in-place or unaligned buffers. fer_rows_f32_pdl / fer_rows_fast_f32_pdl:
 * the same launched
 * with programmatic dependent launch; early 1 lets the first loads,
 * early 2 the whole kernel run before it waits for the kernel just before it
 * on the stream (the caller promises that kernel writes none of x / gamma /
 * beta, and for 2 that it neither reads nor writes y). */
cudaError_t fer_rows_f32(const float* x, float* y, const float* gamma, const float* beta, int rows, int cols,
                         float eps, uint32_t flags, uint32_t* err, cudaStream_t stream);
cudaError_t fer_rows_f32_pdl(const float* x, float* y, const float* gamma, const float* beta, int rows, int cols,
                             float eps, uint32_t flags, uint32_t early, uint32_t* err, cudaStream_t stream);
cudaError_t fer_rows_fast_f32(const float* x, float* y, const float* gamma, const float* beta, int rows, int cols,
                              float eps, uint32_t flags, uint32_t* err, cudaStream_t stream);
cudaError_t fer_rows_fast_f32_pdl(const float* x, float* y, const float* gamma, const float* beta, int rows, int cols,
                                  float eps, uint32_t flags, uint32_t early, uint32_t* err, cudaStream_t stream);
/* Layer norm of every row of x [rows, cols] (no affine) for any buffer dtype
 * (fer_buffer_dtype_t): computed in f32 in the reference order, each value
 * widened on load and rounded back on store as the reference's cast staging
 * does (src/runtime/exec_planner.cu:304-387), so the bits equal cast ->
 * fer_rows_f32 -> cast; one launch, no temporaries; x == y allowed. f32 runs
 * fer_rows_f32. */
cudaError_t fer_layer_norm_typed(const void* x, void* y, int rows, int cols, float eps, uint32_t dtype,
                                 uint32_t* err, cudaStream_t stream);

/* ---- intents -------------------------------------------------------------------
 * Deterministic sum / max of n floats into out[0] (sum adds to out[0], as the
 * reference's atomics do); scratch holds fer_reduce_scratch_floats(n) floats. */
size_t fer_reduce_scratch_floats(unsigned int n);
cudaError_t fer_reduce_f32(const float* in, float* out, float* scratch, unsigned int n, int is_max, cudaStream_t s);
/* Direct 2-D convolution: input [H, W, C], weights [F, C, KH, KW], output
 * [out_h, out_w, F]; optional bias [F] and relu. */
cudaError_t fer_conv2d_f32(const float* input, const float* weights, const float* bias, float* output,
                           unsigned int H, unsigned int W, unsigned int C, unsigned int KH, unsigned int KW,
                           unsigned int F, unsigned int pad_h, unsigned int pad_w, unsigned int sh, unsigned int sw,
                           int relu, cudaStream_t s);

/* ---- transformer building blocks ------------------------------------------------
 * Causal attention, head_dim 64, from the fused activation qkv [B*S, 3d]
 * (q | k | v, head h at columns 64h of each third) into out [B*S, d], bf16.
 * flags bit 0 forces the mma.sync kernel; otherwise S % 128 == 0 takes the
 * tcgen05 kernel. fer_attn_causal == fer_attn_causal_ex(..., 0, NULL, s). */
cudaError_t fer_attn_causal_ex(const void* qkv, void* out, int B, int S, int d, int heads, int flags, uint32_t* err,
                               cudaStream_t s);
cudaError_t fer_attn_causal(const void* qkv, void* out, int B, int S, int d, int heads, cudaStream_t s);
/* The tcgen05 kernel alone: cudaErrorNotSupported where it does not apply. */
cudaError_t fer_attn_causal_tc(const void* qkv, void* out, int B, int S, int d, int heads, uint32_t* err,
                               cudaStream_t stream);
/* KV cache (per layer [max_batch][heads][max_seq][64] bf16, K and V blocks):
 * fer_kv_store copies the K and V parts of qkv [B*S, 3d] (rows b*S + s) to
 * positions pos0 + s of sequences b. fer_attn_decode: one query per sequence
 * (the Q part of row b of qkv_dec [B, 3d]) against positions 0 .. n_keys-1,
 * out [B, d] bf16; split into 256-position chunks combined in chunk order,
 * scratch of fer_attn_decode_scratch_floats(B, heads, n_keys) floats (0: none
 * needed). head_dim 64. err: optional device error word (bulk-copy wait
 * timeouts). */
cudaError_t fer_kv_store(const void* qkv, void* k_cache, void* v_cache, int B, int S, int d, int heads, int max_seq,
                         int pos0, cudaStream_t s);
size_t fer_attn_decode_scratch_floats(int B, int heads, int n_keys);
cudaError_t fer_attn_decode(const void* qkv_dec, const void* k_cache, const void* v_cache, void* out, float* scratch,
                            int B, int d, int heads, int max_seq, int n_keys, uint32_t* err, cudaStream_t s);
/* The decode step's cache store + attention in one kernel, with the position
 * in device memory (*d_len = position of the new token, advanced by the
 * caller with fer_device_int_add): launch arguments never change between
 * steps, so the step can be captured in a CUDA graph and replayed. scratch
 * as fer_attn_decode_scratch_floats(B, heads, max_seq); counters: B * heads
 * ints, zero before the first call and left zero by every call. */
cudaError_t fer_decode_kv_attention(const void* qkv_dec, void* k_cache, void* v_cache, void* out, float* scratch,
                                    int* counters, int B, int d, int heads, int max_seq, int* d_len, uint32_t* err,
                                    cudaStream_t s);
cudaError_t fer_device_int_add(int* d_len, int v, cudaStream_t s);
cudaError_t fer_device_int_set(int* d_len, int v, cudaStream_t s);
/* Per-token layer norm, x f32 [T, d] -> out bf16, d one of 128, 256, ..., 4096. */
cudaError_t fer_ln_bf16(const float* x, const float* g, const float* b, void* out, int T, int d, float eps,
                        cudaStream_t s);
/* x[t] = emb[tok[t]] as f32, emb bf16 [vocab, d], d % 256 == 0; an id outside
 * the vocabulary gives a zero row and error bit 4. */
cudaError_t fer_embed_f32(const int* tok, const void* emb, float* x, int T, int d, int vocab, uint32_t* err,
                          cudaStream_t s);
/* out[i] = bf16(stddev * N(0,1)), element i from draws 2i+1 and 2i+2 of the
 * splitmix64 stream of `seed` (Box-Muller). */
cudaError_t fer_fill_normal_bf16(void* out, size_t n, uint64_t seed, float stddev, cudaStream_t s);
cudaError_t fer_fill_f32(float* out, size_t n, float v, cudaStream_t s);
/* Fills `bytes` at dst (16-byte aligned) with the 32-bit pattern `value`
 * (trailing bytes short of a 16-byte word take its low byte). */
cudaError_t fer_fill_u32(void* dst, size_t bytes, uint32_t value, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FERCUDA_B200_NATIVE_H */
