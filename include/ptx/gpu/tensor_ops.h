/*
 * Native tensor-op ABI (libptx_kernels.so): the reference's
 * native/core/include/gpu/tensor_ops.h. Same names, argument order and
 * meaning, same opcode / dtype values and struct layouts (:17-165); every
 * launcher queues work on `stream` and returns without synchronising.
 * Floating-point results are bit-identical to the reference launchers of the
 * same name (same operations in the same order, built without FMA
 * contraction); index results (argsort, topk, argmax, gather, ...) are
 * identical, ties included. scatter_add with at least 1024 output columns is
 * deterministic (sources added in index order); the reference always uses
 * atomics, so with repeated indices its low-order bits vary run to run.
 */
#ifndef FERCUDA_PTX_TENSOR_OPS_H
#define FERCUDA_PTX_TENSOR_OPS_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include <cuda_fp16.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- opcodes, dtypes, descriptors (tensor_ops.h:17-165, values fixed) ---- */
typedef enum PTXTensorOpcode {
    PTX_OP_ADD = 0x10, PTX_OP_SUB = 0x11, PTX_OP_MUL = 0x12, PTX_OP_DIV = 0x13,
    PTX_OP_MAX = 0x14, PTX_OP_MIN = 0x15, PTX_OP_POW = 0x16, PTX_OP_MOD = 0x17,
    PTX_OP_NEG = 0x20, PTX_OP_ABS = 0x21, PTX_OP_EXP = 0x22, PTX_OP_LOG = 0x23,
    PTX_OP_LOG2 = 0x24, PTX_OP_LOG10 = 0x25, PTX_OP_SQRT = 0x26, PTX_OP_RSQRT = 0x27,
    PTX_OP_SIN = 0x28, PTX_OP_COS = 0x29, PTX_OP_TAN = 0x2A, PTX_OP_TANH = 0x2B,
    PTX_OP_SINH = 0x2C, PTX_OP_COSH = 0x2D, PTX_OP_CEIL = 0x2E, PTX_OP_FLOOR = 0x2F,
    PTX_OP_ROUND = 0x30, PTX_OP_SIGN = 0x31, PTX_OP_RECIP = 0x32, PTX_OP_SQR = 0x33,
    PTX_OP_ERF = 0x34,
    PTX_OP_RELU = 0x40, PTX_OP_RELU6 = 0x41, PTX_OP_LEAKY_RELU = 0x42, PTX_OP_ELU = 0x43,
    PTX_OP_SELU = 0x44, PTX_OP_GELU = 0x45, PTX_OP_GELU_TANH = 0x46, PTX_OP_SIGMOID = 0x47,
    PTX_OP_SILU = 0x48, PTX_OP_SOFTPLUS = 0x49, PTX_OP_MISH = 0x4A, PTX_OP_HARDSWISH = 0x4B,
    PTX_OP_HARDSIGMOID = 0x4C,
    PTX_OP_REDUCE_SUM = 0x50, PTX_OP_REDUCE_MEAN = 0x51, PTX_OP_REDUCE_MAX = 0x52,
    PTX_OP_REDUCE_MIN = 0x53, PTX_OP_REDUCE_PROD = 0x54, PTX_OP_REDUCE_ARGMAX = 0x55,
    PTX_OP_REDUCE_ARGMIN = 0x56,
    PTX_OP_SOFTMAX = 0x60, PTX_OP_LOG_SOFTMAX = 0x61,
    PTX_OP_CMP_EQ = 0x70, PTX_OP_CMP_NE = 0x71, PTX_OP_CMP_LT = 0x72, PTX_OP_CMP_LE = 0x73,
    PTX_OP_CMP_GT = 0x74, PTX_OP_CMP_GE = 0x75,
    PTX_OP_AFFINE = 0x80, PTX_OP_CLAMP = 0x81, PTX_OP_WHERE = 0x82,
    PTX_OP_COPY = 0x90, PTX_OP_CAST = 0x91, PTX_OP_FILL = 0x92,
    PTX_OP_GATHER = 0xB0, PTX_OP_SCATTER_ADD = 0xB1, PTX_OP_INDEX_SELECT = 0xB2, PTX_OP_INDEX_ADD = 0xB3,
    PTX_OP_CUMSUM = 0xC0,
    PTX_OP_ARGSORT = 0xE1, PTX_OP_TOPK = 0xE2
} PTXTensorOpcode;

typedef enum PTXDType {
    PTX_DTYPE_F32 = 0, PTX_DTYPE_F64 = 1, PTX_DTYPE_F16 = 2, PTX_DTYPE_BF16 = 3, PTX_DTYPE_I8 = 4,
    PTX_DTYPE_I16 = 5, PTX_DTYPE_I32 = 6, PTX_DTYPE_I64 = 7, PTX_DTYPE_U8 = 8, PTX_DTYPE_U32 = 9
} PTXDType;

typedef struct PTXTensorDesc {
    void* data;
    size_t elem_count;
    PTXDType dtype;
    uint32_t ndim;
    uint32_t shape[8];
    uint32_t strides[8];
    bool is_contiguous;
} PTXTensorDesc;

/* One operation for ptx_tensor_dispatch. Elementwise: elem_count elements of
 * input_a (and input_b) into output. Reductions, softmax, cumsum: outer_size
 * x reduce_size x inner_size view. Scalars: affine mul/add, clamp lo/hi,
 * leaky/elu alpha and pow exponent in scalar_a (/ scalar_b). Packed forms,
 * as in the reference: GATHER / INDEX_SELECT / SCATTER_ADD take the index
 * array in input_b and (outer_size, reduce_size, inner_size, elem_count) as
 * their four sizes; TOPK takes k in elem_count, largest = scalar_a > 0.5 and
 * the index output in input_b; ARGSORT takes rows, cols in outer_size,
 * reduce_size and ascending = scalar_a > 0.5; WHERE computes
 * output = input_a ? input_b : output. */
typedef struct PTXTensorOp {
    PTXTensorOpcode opcode;
    PTXDType dtype;
    void* input_a;
    void* input_b;
    void* output;
    size_t elem_count;
    float scalar_a;
    float scalar_b;
    uint32_t reduce_dim;
    uint32_t reduce_size;
    uint32_t outer_size;
    uint32_t inner_size;
    cudaStream_t stream;
} PTXTensorOp;

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

/* ---- f32 binary (ops_core.inl:1-60) ---- */
void ptx_tensor_sub_f32(float* a, float* b, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_div_f32(float* a, float* b, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_max_f32(float* a, float* b, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_min_f32(float* a, float* b, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_mod_f32(float* a, float* b, float* out, size_t n, cudaStream_t stream);
/* scalar on the right (ops_core.inl:60-95) */
void ptx_tensor_add_scalar_f32(float* a, float scalar, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_sub_scalar_f32(float* a, float scalar, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_mul_scalar_f32(float* a, float scalar, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_div_scalar_f32(float* a, float scalar, float* out, size_t n, cudaStream_t stream);

/* ---- f32 unary (ops_core.inl:95-250) ---- */
void ptx_tensor_neg_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_abs_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_exp_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_log_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_sqrt_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_rsqrt_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_sin_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_cos_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_tanh_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_ceil_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_floor_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_round_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_sqr_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_recip_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_log2_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_log10_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_tan_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_sinh_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_cosh_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_sign_f32(float* in, float* out, size_t n, cudaStream_t stream);
/* Abramowitz & Stegun 7.1.26 approximation, as the reference (max error ~1.5e-7) */
void ptx_tensor_erf_f32(float* in, float* out, size_t n, cudaStream_t stream);

/* ---- f32 activations (ops_core.inl:250-345) ---- */
void ptx_tensor_relu6_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_leaky_relu_f32(float* in, float* out, size_t n, float alpha, cudaStream_t stream);
void ptx_tensor_elu_f32(float* in, float* out, size_t n, float alpha, cudaStream_t stream);
void ptx_tensor_selu_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_gelu_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_gelu_tanh_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_silu_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_softplus_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_mish_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_hardswish_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_hardsigmoid_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_clamp_f32(float* in, float* out, size_t n, float min_val, float max_val, cudaStream_t stream);
void ptx_tensor_powf_f32(float* in, float* out, size_t n, float exp, cudaStream_t stream);

/* ---- reductions over an [outer, reduce, inner] view into [outer, inner]
 * (ops_core.inl:480-730; launchers :1519-1565) ---- */
void ptx_tensor_reduce_sum_f32(float* in, float* out, size_t outer, size_t reduce, size_t inner, cudaStream_t stream);
void ptx_tensor_reduce_mean_f32(float* in, float* out, size_t outer, size_t reduce, size_t inner, cudaStream_t stream);
void ptx_tensor_reduce_max_f32(float* in, float* out, size_t outer, size_t reduce, size_t inner, cudaStream_t stream);
void ptx_tensor_reduce_min_f32(float* in, float* out, size_t outer, size_t reduce, size_t inner, cudaStream_t stream);
void ptx_tensor_reduce_prod_f32(float* in, float* out, size_t outer, size_t reduce, size_t inner, cudaStream_t stream);
/* index of the first maximum / minimum along the reduced axis (0 if none) */
void ptx_tensor_reduce_argmax_f32(float* in, int32_t* out, size_t outer, size_t reduce, size_t inner,
                                  cudaStream_t stream);
void ptx_tensor_reduce_argmin_f32(float* in, int32_t* out, size_t outer, size_t reduce, size_t inner,
                                  cudaStream_t stream);

/* ---- gather / scatter (indexing_scan.inl); negative indices count from the
 * end; gather / index_select clamp out-of-range indices, scatter_add skips
 * them ---- */
void ptx_tensor_gather_f32(float* in, int32_t* indices, float* out, size_t outer, size_t input_dim_size,
                           size_t idx_dim_size, size_t inner, cudaStream_t stream);
void ptx_tensor_index_select_f32(float* in, int32_t* ids, float* out, size_t left_size, size_t src_dim_size,
                                 size_t ids_dim_size, size_t right_size, cudaStream_t stream);
void ptx_tensor_scatter_add_f32(int32_t* ids, float* src, float* out, size_t left_size, size_t src_dim_size,
                                size_t dst_dim_size, size_t right_size, cudaStream_t stream);

/* ---- scan, sort, select (indexing_scan.inl) ---- */
void ptx_tensor_cumsum_f32(float* in, float* out, size_t outer, size_t dim_size, size_t inner, cudaStream_t stream);
/* per row of [nrows, ncols]; ncols up to 16384 (the reference: 8192) */
void ptx_tensor_argsort_f32(float* in, uint32_t* out, size_t nrows, size_t ncols, int ascending,
                            cudaStream_t stream);
/* k best along dim_size (ties: lower index first); values [outer, k, inner],
 * indices likewise (may be NULL) */
void ptx_tensor_topk_f32(float* in, float* values_out, int32_t* indices_out, size_t outer, size_t dim_size,
                         size_t inner, size_t k, int largest, cudaStream_t stream);

/* ---- softmax variants (ops_core.inl:809-860, 1050-1110, 1180-1230) ---- */
void ptx_tensor_log_softmax_f32(float* in, float* out, size_t batch, size_t dim, cudaStream_t stream);
void ptx_tensor_softmax_f64(double* in, double* out, size_t batch, size_t dim, cudaStream_t stream);
void ptx_tensor_softmax_f16(__half* in, __half* out, size_t batch, size_t dim, cudaStream_t stream);

/* ---- comparisons (1 / 0 bytes), select, copy, fill, casts ---- */
void ptx_tensor_cmp_eq_f32(float* a, float* b, uint8_t* out, size_t n, cudaStream_t stream);
void ptx_tensor_cmp_ne_f32(float* a, float* b, uint8_t* out, size_t n, cudaStream_t stream);
void ptx_tensor_cmp_lt_f32(float* a, float* b, uint8_t* out, size_t n, cudaStream_t stream);
void ptx_tensor_cmp_le_f32(float* a, float* b, uint8_t* out, size_t n, cudaStream_t stream);
void ptx_tensor_cmp_gt_f32(float* a, float* b, uint8_t* out, size_t n, cudaStream_t stream);
void ptx_tensor_cmp_ge_f32(float* a, float* b, uint8_t* out, size_t n, cudaStream_t stream);
void ptx_tensor_where_f32(uint8_t* cond, float* t, float* f, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_copy_f32(float* in, float* out, size_t n, cudaStream_t stream);
void ptx_tensor_fill_f32(float* out, size_t n, float value, cudaStream_t stream);
void ptx_tensor_cast_f32_to_f16(float* in, __half* out, size_t n, cudaStream_t stream);
void ptx_tensor_cast_f16_to_f32(__half* in, float* out, size_t n, cudaStream_t stream);

/* ---- f64 (ops_core.inl:860-1110) ---- */
void ptx_tensor_add_f64(double* a, double* b, double* out, size_t n, cudaStream_t stream);
void ptx_tensor_sub_f64(double* a, double* b, double* out, size_t n, cudaStream_t stream);
void ptx_tensor_mul_f64(double* a, double* b, double* out, size_t n, cudaStream_t stream);
void ptx_tensor_div_f64(double* a, double* b, double* out, size_t n, cudaStream_t stream);
void ptx_tensor_neg_f64(double* in, double* out, size_t n, cudaStream_t stream);
void ptx_tensor_exp_f64(double* in, double* out, size_t n, cudaStream_t stream);
void ptx_tensor_log_f64(double* in, double* out, size_t n, cudaStream_t stream);
void ptx_tensor_sqrt_f64(double* in, double* out, size_t n, cudaStream_t stream);
void ptx_tensor_tanh_f64(double* in, double* out, size_t n, cudaStream_t stream);
void ptx_tensor_relu_f64(double* in, double* out, size_t n, cudaStream_t stream);
void ptx_tensor_gelu_f64(double* in, double* out, size_t n, cudaStream_t stream);
void ptx_tensor_sigmoid_f64(double* in, double* out, size_t n, cudaStream_t stream);
void ptx_tensor_reduce_sum_f64(double* in, double* out, size_t outer, size_t reduce, size_t inner,
                               cudaStream_t stream);
void ptx_tensor_reduce_max_f64(double* in, double* out, size_t outer, size_t reduce, size_t inner,
                               cudaStream_t stream);
/* the reference's k_reduce_min_f64 combines inside each warp with fmax; this
 * returns the same value it does */
void ptx_tensor_reduce_min_f64(double* in, double* out, size_t outer, size_t reduce, size_t inner,
                               cudaStream_t stream);
void ptx_tensor_affine_f64(double* in, double* out, size_t n, double mul, double add, cudaStream_t stream);

/* ---- f16 (ops_core.inl:1140-1230) ---- */
void ptx_tensor_add_f16(__half* a, __half* b, __half* out, size_t n, cudaStream_t stream);
void ptx_tensor_sub_f16(__half* a, __half* b, __half* out, size_t n, cudaStream_t stream);
void ptx_tensor_mul_f16(__half* a, __half* b, __half* out, size_t n, cudaStream_t stream);
void ptx_tensor_div_f16(__half* a, __half* b, __half* out, size_t n, cudaStream_t stream);
void ptx_tensor_relu_f16(__half* in, __half* out, size_t n, cudaStream_t stream);
void ptx_tensor_gelu_f16(__half* in, __half* out, size_t n, cudaStream_t stream);
void ptx_tensor_sigmoid_f16(__half* in, __half* out, size_t n, cudaStream_t stream);

/* ---- dispatch by opcode and dtype (util_dispatch.inl:200-606): an
 * unsupported dtype queues nothing and returns the last launch status; an
 * unknown opcode returns cudaErrorInvalidValue. _sync waits for op->stream
 * (the device when it is NULL). ---- */
cudaError_t ptx_tensor_dispatch(const PTXTensorOp* op);
cudaError_t ptx_tensor_dispatch_sync(const PTXTensorOp* op);

/* ---- CUDA graph capture of a sequence of launches (util_dispatch.inl:608-622) ---- */
cudaError_t ptx_tensor_graph_begin_capture(cudaStream_t stream);
cudaError_t ptx_tensor_graph_end_capture(cudaStream_t stream, cudaGraph_t* graph_out);
cudaError_t ptx_tensor_graph_instantiate(cudaGraph_t graph, cudaGraphExec_t* exec_out);
cudaError_t ptx_tensor_graph_launch(cudaGraphExec_t exec, cudaStream_t stream);

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
 * scratch is a fixed 256 KiB device array inside this library; the call
 * allocates nothing.
 *   - n <= PTX_REDUCE_NOALLOC_MAX_ELEMENTS, else cudaErrorInvalidValue and no
 *     launch;
 *   - calls share the scratch: calls that overlap on the GPU race, so
 *     serialise them;
 *   - the first call in a device's context loads the array and the kernels
 *     (device memory, taken then and held until the context is destroyed)
 *     and resolves the scratch address: make that first call (a warm-up call
 *     will do) before reserving the rest of the device's memory, and before
 *     any stream capture begins. After cudaDeviceReset the next call repeats
 *     that set-up. */
#define PTX_REDUCE_NOALLOC_MAX_ELEMENTS 33554432u
cudaError_t ptx_tensor_reduce_f32_noalloc(const float* in, float* out, size_t n, int is_max, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif
