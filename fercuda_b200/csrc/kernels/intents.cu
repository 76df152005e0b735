// Kernels behind the non-elementwise JIT intents (reduce_sum, reduce_max,
// conv2d). The intent ABI (include/fercuda/jit/intent/intent.h) is the
// reference's; the kernels are deterministic rewrites of the reference's
// NVRTC sources (native/core/jit/intent/intent_runtime.cpp:120-221):
//   reduce_sum  reference: per-CTA tree, then atomicAdd of each CTA's partial
//               into out[0] (order varies run to run). Here: the same per-CTA
//               tree into a partials array, then one CTA sums the partials in a
//               fixed order and adds the total to out[0]. Bit-identical run to run.
//   reduce_max  per-CTA tree as the reference, then a fixed-order max over the
//               partials; out[0] = total if total > out[0] (the reference's CAS loop).
//   conv2d      one output per thread, accumulation order c, kh, kw with one
//               fused multiply-add per tap (what the reference's NVRTC build,
//               which contracts `acc += iv * wv`, computes).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

namespace {

constexpr int kBlock = 256;

template <bool kMax>
__global__ void __launch_bounds__(kBlock) reduce_stage1(const float* __restrict__ in, float* __restrict__ part,
                                                        unsigned int n) {
    __shared__ float sdata[kBlock];
    const unsigned int tid = threadIdx.x;
    const unsigned int i = blockIdx.x * (kBlock * 2u) + tid;
    float v;
    if (kMax) {
        v = -1e30f;
        if (i < n) v = in[i];
        if (i + kBlock < n) v = fmaxf(v, in[i + kBlock]);
    } else {
        v = 0.0f;
        if (i < n) v = in[i];
        if (i + kBlock < n) v += in[i + kBlock];
    }
    sdata[tid] = v;
    __syncthreads();
    for (unsigned int s = kBlock / 2; s > 0; s >>= 1) {
        if (tid < s) sdata[tid] = kMax ? fmaxf(sdata[tid], sdata[tid + s]) : sdata[tid] + sdata[tid + s];
        __syncthreads();
    }
    if (tid == 0) part[blockIdx.x] = sdata[0];
}

template <bool kMax>
__global__ void __launch_bounds__(1024) reduce_stage2(const float* __restrict__ part, unsigned int nparts,
                                                      float* __restrict__ out) {
    __shared__ float sdata[1024];
    const unsigned int tid = threadIdx.x;
    float v = kMax ? -1e30f : 0.0f;
    for (unsigned int j = tid; j < nparts; j += 1024) v = kMax ? fmaxf(v, part[j]) : v + part[j];
    sdata[tid] = v;
    __syncthreads();
    for (unsigned int s = 512; s > 0; s >>= 1) {
        if (tid < s) sdata[tid] = kMax ? fmaxf(sdata[tid], sdata[tid + s]) : sdata[tid] + sdata[tid + s];
        __syncthreads();
    }
    if (tid == 0) {
        if (kMax) {
            if (sdata[0] > out[0]) out[0] = sdata[0];
        } else {
            out[0] = out[0] + sdata[0];
        }
    }
}

__global__ void conv2d_direct(const float* __restrict__ input, const float* __restrict__ weights,
                              const float* __restrict__ bias, float* __restrict__ output, unsigned int H,
                              unsigned int W, unsigned int C, unsigned int KH, unsigned int KW, unsigned int F,
                              unsigned int pad_h, unsigned int pad_w, unsigned int sh, unsigned int sw, int relu) {
    const unsigned int out_h = (H + 2 * pad_h - KH) / sh + 1;
    const unsigned int out_w = (W + 2 * pad_w - KW) / sw + 1;
    const unsigned int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= out_h * out_w * F) return;
    const unsigned int f = idx % F;
    const unsigned int pw = (idx / F) % out_w;
    const unsigned int ph = (idx / F) / out_w;
    float acc = bias ? bias[f] : 0.0f;
    for (unsigned int c = 0; c < C; ++c)
        for (unsigned int kh = 0; kh < KH; ++kh)
            for (unsigned int kw = 0; kw < KW; ++kw) {
                const int ih = static_cast<int>(ph * sh + kh) - static_cast<int>(pad_h);
                const int iw = static_cast<int>(pw * sw + kw) - static_cast<int>(pad_w);
                if (ih >= 0 && ih < static_cast<int>(H) && iw >= 0 && iw < static_cast<int>(W)) {
                    const float iv = input[(static_cast<unsigned int>(ih) * W + static_cast<unsigned int>(iw)) * C + c];
                    const float wv = weights[((f * C + c) * KH + kh) * KW + kw];
                    acc = __fmaf_rn(iv, wv, acc);
                }
            }
    if (relu && acc < 0.0f) acc = 0.0f;
    output[(ph * out_w + pw) * F + f] = acc;
}

}  // namespace

// Partials scratch: ceil(n / 512) floats.
extern "C" size_t fer_reduce_scratch_floats(unsigned int n) { return (n + 2u * kBlock - 1u) / (2u * kBlock); }

extern "C" cudaError_t fer_reduce_f32(const float* in, float* out, float* scratch, unsigned int n, int is_max,
                                      cudaStream_t s) {
    if (n == 0) return cudaErrorInvalidValue;
    const unsigned int grid = (n + 2u * kBlock - 1u) / (2u * kBlock);
    if (is_max) {
        reduce_stage1<true><<<grid, kBlock, 0, s>>>(in, scratch, n);
        reduce_stage2<true><<<1, 1024, 0, s>>>(scratch, grid, out);
    } else {
        reduce_stage1<false><<<grid, kBlock, 0, s>>>(in, scratch, n);
        reduce_stage2<false><<<1, 1024, 0, s>>>(scratch, grid, out);
    }
    return cudaGetLastError();
}

extern "C" cudaError_t fer_conv2d_f32(const float* input, const float* weights, const float* bias, float* output,
                                      unsigned int H, unsigned int W, unsigned int C, unsigned int KH, unsigned int KW,
                                      unsigned int F, unsigned int pad_h, unsigned int pad_w, unsigned int sh,
                                      unsigned int sw, int relu, cudaStream_t s) {
    const unsigned int out_h = (H + 2 * pad_h - KH) / sh + 1;
    const unsigned int out_w = (W + 2 * pad_w - KW) / sw + 1;
    const unsigned int total = out_h * out_w * F;
    conv2d_direct<<<(total + 255) / 256, 256, 0, s>>>(input, weights, bias, output, H, W, C, KH, KW, F, pad_h, pad_w,
                                                      sh, sw, relu);
    return cudaGetLastError();
}

// ---- reduction into caller-provided memory only ------------------------------
// Some callers cannot allocate device memory at the moment they need a
// reduction:
//   - a custom allocator callback registered with fer_register_custom_allocator
//     (or any code inside an allocator) would re-enter the allocator it is
//     part of;
//   - a process whose cudaMalloc is interposed and routed into the pool being
//     managed cannot allocate from inside that pool's own bookkeeping;
//   - a process that has reserved nearly all device memory for its pools at
//     start-up may have nothing left for cudaMalloc to return.
// ptx_tensor_reduce_f32_noalloc serves them: the per-CTA partials live in the
// fixed device array below instead of allocated scratch, so the call itself
// allocates nothing.
//   - At most kNoAllocMaxPartials partials, i.e. n <= 33,554,432 elements;
//     larger n is rejected with cudaErrorInvalidValue before any launch.
//   - All calls share the array. Each call overwrites every partial it reads
//     before reading it, so nothing needs clearing between calls; calls that
//     overlap on the GPU (different streams, or several host threads) race
//     on the array and must be serialised by the caller.
//   - Set-up, once per device and context: the first call with a device's
//     context current loads this file's module (the 256 KiB array and the two
//     reduction kernels, which lazy module loading would otherwise load on
//     first launch) and looks the array's device address up with
//     cudaGetSymbolAddress. Loading the module takes device memory, so that
//     first call (a warm-up call will do) belongs before the caller reserves
//     its memory, and before any stream capture. From then on the device
//     holds the array until its context is destroyed.
//   - The address is remembered per device together with the context's
//     unique id (cuCtxGetId). After cudaDeviceReset, or any other teardown
//     and re-creation of the context, the id differs and the next call
//     repeats the set-up; that call again loads the module.
constexpr unsigned kNoAllocMaxPartials = 65536;   // 256 KiB of f32 partials
static __device__ __align__(256) float g_noalloc_partials[kNoAllocMaxPartials];

namespace {

using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

struct NoAllocSlot {
    unsigned long long ctx_id = 0;   // 0: not set up (context ids start at 1)
    float* addr = nullptr;
};

std::mutex g_noalloc_mu;
NoAllocSlot g_noalloc_slot[64];
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;

// Unique id of the context current on this thread (making the device's
// primary context current first if none is). Caller holds g_noalloc_mu.
cudaError_t current_context_id(int dev, unsigned long long* id) {
    if (!g_ctx_get_current || !g_ctx_get_id) {
        void* f0 = nullptr;
        void* f1 = nullptr;
        cudaDriverEntryPointQueryResult q0, q1;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f0, 12000, cudaEnableDefault, &q0);
        if (e == cudaSuccess) e = cudaGetDriverEntryPointByVersion("cuCtxGetId", &f1, 12000, cudaEnableDefault, &q1);
        if (e != cudaSuccess) return e;
        if (q0 != cudaDriverEntryPointSuccess || q1 != cudaDriverEntryPointSuccess || !f0 || !f1)
            return cudaErrorNotSupported;
        g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f0);
        g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f1);
    }
    CUcontext ctx = nullptr;
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) return cudaErrorUnknown;
    if (!ctx) {
        const cudaError_t e = cudaSetDevice(dev);   // initialises and binds the primary context
        if (e != cudaSuccess) return e;
        if (g_ctx_get_current(&ctx) != CUDA_SUCCESS || !ctx) return cudaErrorDeviceUninitialized;
    }
    return g_ctx_get_id(ctx, id) == CUDA_SUCCESS ? cudaSuccess : cudaErrorUnknown;
}

// Device address of g_noalloc_partials in the current context. In host code
// the symbol itself is only a host-side stand-in, so kernels get this address.
cudaError_t noalloc_partials(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    unsigned long long id = 0;
    e = current_context_id(dev, &id);
    if (e != cudaSuccess) return e;
    NoAllocSlot& slot = g_noalloc_slot[dev];
    if (slot.ctx_id != id || !slot.addr) {
        cudaFuncAttributes fa;
        e = cudaFuncGetAttributes(&fa, reduce_stage1<false>);
        if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, reduce_stage2<false>);
        if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, reduce_stage1<true>);
        if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, reduce_stage2<true>);
        void* p = nullptr;
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&p, g_noalloc_partials);
        if (e != cudaSuccess) return e;
        slot.addr = static_cast<float*>(p);
        slot.ctx_id = id;
    }
    *out = slot.addr;
    return cudaSuccess;
}

}  // namespace

extern "C" cudaError_t ptx_tensor_reduce_f32_noalloc(const float* in, float* out, size_t n, int is_max,
                                                     cudaStream_t stream) {
    if (!in || !out || n == 0) return cudaErrorInvalidValue;
    if (n > static_cast<size_t>(kNoAllocMaxPartials) * 2u * kBlock) return cudaErrorInvalidValue;
    float* partials = nullptr;
    const cudaError_t e = noalloc_partials(&partials);
    if (e != cudaSuccess) return e;
    return fer_reduce_f32(in, out, partials, static_cast<unsigned int>(n), is_max, stream);
}
