/*
 * Native tensor-op ABI (libptx_kernels.so), the hot-path subset of the
 * reference native/core/include/gpu/tensor_ops.h:181-333. Same names,
 * argument order and meaning; every launcher queues work on `stream` and
 * returns without synchronising. Results are bit-identical to the reference
 * launchers of the same name.
 */
#ifndef FERCUDA_PTX_TENSOR_OPS_H
#define FERCUDA_PTX_TENSOR_OPS_H

#include <stddef.h>

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* out[i] = a[i] + b[i]        (reference tensor_kernels_ops_core.inl:5-11, launcher :1287) */
void ptx_tensor_add_f32(float* a, float* b, float* out, size_t n, cudaStream_t stream);
/* out[i] = a[i] * b[i]        (ops_core.inl:21-27, launcher :1295) */
void ptx_tensor_mul_f32(float* a, float* b, float* out, size_t n, cudaStream_t stream);
/* out[i] = fmaxf(0, in[i])    (ops_core.inl:257-262, launcher :1418) */
void ptx_tensor_relu_f32(float* in, float* out, size_t n, cudaStream_t stream);
/* out[i] = 1/(1+expf(-in[i])) (ops_core.inl:308-313, launcher :1442) */
void ptx_tensor_sigmoid_f32(float* in, float* out, size_t n, cudaStream_t stream);
/* out[i] = in[i]*mul + add    (ops_core.inl:375-381, launcher :1471) */
void ptx_tensor_affine_f32(float* in, float* out, size_t n, float mul, float add, cudaStream_t stream);
/* row softmax over [batch, dim] (ops_core.inl:733-808, launcher indexing_scan.inl:391-394) */
void ptx_tensor_softmax_f32(float* in, float* out, size_t batch, size_t dim, cudaStream_t stream);

/* Additive (no reference counterpart): fused row softmax -> layer norm, and
 * row-batched layer norm; gamma / beta optional (NULL). */
void ptx_tensor_softmax_layer_norm_f32(float* in, float* out, const float* gamma, const float* beta,
                                       size_t rows, size_t cols, float eps, cudaStream_t stream);
void ptx_tensor_layer_norm_rows_f32(float* in, float* out, const float* gamma, const float* beta,
                                    size_t rows, size_t cols, float eps, cudaStream_t stream);

/* No counterpart in the reference. Sum (is_max = 0: out[0] += sum(in)) or
 * maximum (is_max != 0: out[0] = max(out[0], max(in))) of n f32 values, the
 * same deterministic two-stage reduction as the REDUCE_SUM / REDUCE_MAX JIT
 * intents, for callers that cannot allocate device memory at that moment
 * (allocator callbacks, processes whose cudaMalloc is routed into the pool
 * being managed, processes that reserved all device memory up front). The
 * scratch is a fixed device array inside this library (held by every GPU
 * that loads it until exit); the call allocates nothing.
 *   - n <= PTX_REDUCE_NOALLOC_MAX_ELEMENTS, else cudaErrorInvalidValue and no
 *     launch;
 *   - calls share the scratch: calls that overlap on the GPU race, so
 *     serialise them;
 *   - the first call on a device resolves the scratch address; make it
 *     before any stream capture begins. */
#define PTX_REDUCE_NOALLOC_MAX_ELEMENTS 33554432u
cudaError_t ptx_tensor_reduce_f32_noalloc(const float* in, float* out, size_t n, int is_max, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif
