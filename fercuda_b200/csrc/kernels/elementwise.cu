// Native elementwise launchers (ptx_tensor_* subset on the hot path).
//
// Per-element arithmetic is the reference's (built -fmad=false there and here),
// so each launcher is bit-identical to its reference counterpart:
//   ptx_tensor_add_f32      tensor_kernels_ops_core.inl:5-11     a + b
//   ptx_tensor_mul_f32      tensor_kernels_ops_core.inl:21-27    a * b
//   ptx_tensor_relu_f32     tensor_kernels_ops_core.inl:257-262  fmaxf(0, x)
//   ptx_tensor_sigmoid_f32  tensor_kernels_ops_core.inl:308-313  1 / (1 + expf(-x))
//   ptx_tensor_affine_f32   tensor_kernels_ops_core.inl:375-381  x * mul + add
// The data path differs: 128-bit loads and stores, four vectors in flight per
// thread, and a grid of at most 8 CTAs per SM that strides over the array
// (the reference uses one scalar element per thread, ceil(n/256) CTAs).
// Misaligned pointers take a scalar grid-stride loop.
#include <cuda_runtime.h>

#include <cstdint>

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

struct OpAdd { __device__ float operator()(float a, float b) const { return a + b; } };
struct OpMul { __device__ float operator()(float a, float b) const { return a * b; } };
struct OpRelu { __device__ float operator()(float x) const { return fmaxf(0.0f, x); } };
struct OpSigmoid { __device__ float operator()(float x) const { return 1.0f / (1.0f + expf(-x)); } };
struct OpAffine {
    float mul, add;
    __device__ float operator()(float x) const { return x * mul + add; }
};

template <typename Op>
__global__ void __launch_bounds__(kThreads) unary_v4(const float4* __restrict__ in, float4* __restrict__ out,
                                                     size_t n4, Op op) {
    const size_t stride = static_cast<size_t>(gridDim.x) * kThreads;
    size_t i = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x;
    for (; i + (kUnroll - 1) * stride < n4; i += kUnroll * stride) {
        float4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) v[u] = __ldcs(in + i + u * stride);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            float4 r;
            r.x = op(v[u].x); r.y = op(v[u].y); r.z = op(v[u].z); r.w = op(v[u].w);
            __stcs(out + i + u * stride, r);
        }
    }
    for (; i < n4; i += stride) {
        const float4 v = __ldcs(in + i);
        float4 r;
        r.x = op(v.x); r.y = op(v.y); r.z = op(v.z); r.w = op(v.w);
        __stcs(out + i, r);
    }
}

template <typename Op>
__global__ void __launch_bounds__(kThreads) binary_v4(const float4* __restrict__ a, const float4* __restrict__ b,
                                                      float4* __restrict__ out, size_t n4, Op op) {
    const size_t stride = static_cast<size_t>(gridDim.x) * kThreads;
    for (size_t i = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; i < n4; i += stride) {
        const float4 x = __ldcs(a + i), y = __ldcs(b + i);
        float4 r;
        r.x = op(x.x, y.x); r.y = op(x.y, y.y); r.z = op(x.z, y.z); r.w = op(x.w, y.w);
        __stcs(out + i, r);
    }
}

template <typename Op>
__global__ void unary_s1(const float* in, float* out, size_t lo, size_t n, Op op) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = lo + static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = op(in[i]);
}

template <typename Op>
__global__ void binary_s1(const float* a, const float* b, float* out, size_t lo, size_t n, Op op) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = lo + static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = op(a[i], b[i]);
}

int sm_count() {
    static const int n = [] {
        int dev = 0, v = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v > 0 ? v : 148;
    }();
    return n;
}

unsigned grid_for(size_t work_items) {
    const size_t cap = static_cast<size_t>(sm_count()) * 8;
    size_t g = (work_items + kThreads - 1) / kThreads;
    if (g > cap) g = cap;
    return static_cast<unsigned>(g ? g : 1);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename Op>
void run_unary(const float* in, float* out, size_t n, Op op, cudaStream_t s) {
    if (n == 0) return;
    size_t done = 0;
    if (aligned16(in) && aligned16(out)) {
        const size_t n4 = n / 4;
        if (n4) unary_v4<<<grid_for(n4), kThreads, 0, s>>>(reinterpret_cast<const float4*>(in),
                                                            reinterpret_cast<float4*>(out), n4, op);
        done = n4 * 4;
    }
    if (done < n) unary_s1<<<grid_for(n - done), kThreads, 0, s>>>(in, out, done, n, op);
}

template <typename Op>
void run_binary(const float* a, const float* b, float* out, size_t n, Op op, cudaStream_t s) {
    if (n == 0) return;
    size_t done = 0;
    if (aligned16(a) && aligned16(b) && aligned16(out)) {
        const size_t n4 = n / 4;
        if (n4)
            binary_v4<<<grid_for(n4), kThreads, 0, s>>>(reinterpret_cast<const float4*>(a),
                                                         reinterpret_cast<const float4*>(b),
                                                         reinterpret_cast<float4*>(out), n4, op);
        done = n4 * 4;
    }
    if (done < n) binary_s1<<<grid_for(n - done), kThreads, 0, s>>>(a, b, out, done, n, op);
}

}  // namespace

extern "C" {

void ptx_tensor_add_f32(float* a, float* b, float* out, size_t n, cudaStream_t stream) {
    run_binary(a, b, out, n, OpAdd{}, stream);
}

void ptx_tensor_mul_f32(float* a, float* b, float* out, size_t n, cudaStream_t stream) {
    run_binary(a, b, out, n, OpMul{}, stream);
}

void ptx_tensor_relu_f32(float* in, float* out, size_t n, cudaStream_t stream) {
    run_unary(in, out, n, OpRelu{}, stream);
}

void ptx_tensor_sigmoid_f32(float* in, float* out, size_t n, cudaStream_t stream) {
    run_unary(in, out, n, OpSigmoid{}, stream);
}

void ptx_tensor_affine_f32(float* in, float* out, size_t n, float mul, float add, cudaStream_t stream) {
    run_unary(in, out, n, OpAffine{mul, add}, stream);
}

}  // extern "C"

namespace {

__global__ void fill_u32_kernel(uint4* __restrict__ dst, size_t n16, uint32_t v) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const uint4 w = make_uint4(v, v, v, v);
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16; i += stride) dst[i] = w;
}

__global__ void fill_u8_tail(uint8_t* dst, size_t n, uint8_t v) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = v;
}

}  // namespace

// Fills `bytes` bytes at dst (16-byte aligned) with the 32-bit pattern
// `value` (the trailing bytes that do not fill a 16-byte word take its low byte).
extern "C" cudaError_t fer_fill_u32(void* dst, size_t bytes, uint32_t value, cudaStream_t stream) {
    if (bytes == 0) return cudaSuccess;
    if (reinterpret_cast<uintptr_t>(dst) & 15u) return cudaErrorInvalidValue;
    const size_t n16 = bytes / 16;
    if (n16) fill_u32_kernel<<<grid_for(n16), kThreads, 0, stream>>>(static_cast<uint4*>(dst), n16, value);
    const size_t tail = bytes - n16 * 16;
    if (tail) fill_u8_tail<<<1, 16, 0, stream>>>(static_cast<uint8_t*>(dst) + n16 * 16, tail, static_cast<uint8_t>(value));
    return cudaGetLastError();
}
