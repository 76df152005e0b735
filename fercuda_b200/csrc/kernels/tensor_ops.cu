// Native tensor-op ABI, elementwise part: the f32 / f64 / f16 unary, binary,
// scalar, activation, comparison, select, fill and cast launchers of the
// reference's native/core/include/gpu/tensor_ops.h:181-333, the elementwise
// launchers its dispatch reaches beyond that range (mod, log2, log10, tan,
// sinh, cosh, sign, erf, gelu_tanh, hardswish, hardsigmoid, cmp_ne), the
// opcode dispatch and the graph-capture helpers.
//
// Each per-element function is the reference's expression, operation for
// operation (native/core/kernels/modules/tensor_kernels_ops_core.inl:1-470,
// 860-960, 1140-1180; constants tensor_kernels_common.inl:11-15), compiled
// like the reference with -fmad=false, so results are bit-identical. The data
// path is B200-first instead of one scalar element per thread over
// ceil(n/256) CTAs: 16-byte packs of the widest operand type (4 f32, 2 f64,
// 8 f16 per pack), four packs in flight per thread, at most 8 CTAs of 256
// threads per SM striding over the array; unaligned pointers and the tail
// past the last whole pack take a scalar grid-stride loop with the same
// function. In place (out == an input) is allowed, as in the reference.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "ptx/gpu/tensor_ops.h"

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

constexpr float kSqrt2OverPi = 0.7978845608028654f;
constexpr float kGeluCoef = 0.044715f;
constexpr float kSeluAlpha = 1.6732632423543772f;
constexpr float kSeluLambda = 1.0507009873554805f;

template <typename T, int E>
struct alignas(sizeof(T) * E) Pack {
    T v[E];
};

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

bool aligned(const void* p, size_t bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

// ---------------------------------------------------------------- engine
// out[i] = f(a[i]) / f(a[i], b[i]) / f(c[i], a[i], b[i]) over whole packs.
template <int E, typename O, typename A, typename F>
__global__ void __launch_bounds__(kThreads) map1_packs(const A* __restrict__ a, O* __restrict__ out, size_t packs,
                                                       F f) {
    using PA = Pack<A, E>;
    using PO = Pack<O, E>;
    const PA* pa = reinterpret_cast<const PA*>(a);
    PO* po = reinterpret_cast<PO*>(out);
    const size_t stride = static_cast<size_t>(gridDim.x) * kThreads;
    size_t i = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x;
    for (; i + (kUnroll - 1) * stride < packs; i += kUnroll * stride) {
        PA x[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) x[u] = pa[i + u * stride];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            PO r;
#pragma unroll
            for (int e = 0; e < E; ++e) r.v[e] = f(x[u].v[e]);
            po[i + u * stride] = r;
        }
    }
    for (; i < packs; i += stride) {
        const PA x = pa[i];
        PO r;
#pragma unroll
        for (int e = 0; e < E; ++e) r.v[e] = f(x.v[e]);
        po[i] = r;
    }
}

template <int E, typename O, typename A, typename B, typename F>
__global__ void __launch_bounds__(kThreads) map2_packs(const A* __restrict__ a, const B* __restrict__ b,
                                                       O* __restrict__ out, size_t packs, F f) {
    using PA = Pack<A, E>;
    using PB = Pack<B, E>;
    using PO = Pack<O, E>;
    const PA* pa = reinterpret_cast<const PA*>(a);
    const PB* pb = reinterpret_cast<const PB*>(b);
    PO* po = reinterpret_cast<PO*>(out);
    const size_t stride = static_cast<size_t>(gridDim.x) * kThreads;
    size_t i = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x;
    for (; i + (kUnroll - 1) * stride < packs; i += kUnroll * stride) {
        PA x[kUnroll];
        PB y[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            x[u] = pa[i + u * stride];
            y[u] = pb[i + u * stride];
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            PO r;
#pragma unroll
            for (int e = 0; e < E; ++e) r.v[e] = f(x[u].v[e], y[u].v[e]);
            po[i + u * stride] = r;
        }
    }
    for (; i < packs; i += stride) {
        const PA x = pa[i];
        const PB y = pb[i];
        PO r;
#pragma unroll
        for (int e = 0; e < E; ++e) r.v[e] = f(x.v[e], y.v[e]);
        po[i] = r;
    }
}

template <int E, typename O, typename C, typename A, typename F>
__global__ void __launch_bounds__(kThreads) map3_packs(const C* __restrict__ c, const A* __restrict__ a,
                                                       const A* __restrict__ b, O* __restrict__ out, size_t packs,
                                                       F f) {
    using PC = Pack<C, E>;
    using PA = Pack<A, E>;
    using PO = Pack<O, E>;
    const size_t stride = static_cast<size_t>(gridDim.x) * kThreads;
    for (size_t i = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; i < packs; i += stride) {
        const PC z = reinterpret_cast<const PC*>(c)[i];
        const PA x = reinterpret_cast<const PA*>(a)[i];
        const PA y = reinterpret_cast<const PA*>(b)[i];
        PO r;
#pragma unroll
        for (int e = 0; e < E; ++e) r.v[e] = f(z.v[e], x.v[e], y.v[e]);
        reinterpret_cast<PO*>(out)[i] = r;
    }
}

template <typename O, typename A, typename F>
__global__ void map1_scalar(const A* a, O* out, size_t lo, size_t n, F f) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = lo + static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = f(a[i]);
}

template <typename O, typename A, typename B, typename F>
__global__ void map2_scalar(const A* a, const B* b, O* out, size_t lo, size_t n, F f) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = lo + static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = f(a[i], b[i]);
}

template <typename O, typename C, typename A, typename F>
__global__ void map3_scalar(const C* c, const A* a, const A* b, O* out, size_t lo, size_t n, F f) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = lo + static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = f(c[i], a[i], b[i]);
}

// Elements per pack: 16 bytes of the widest operand.
template <typename... T>
constexpr int pack_elems() {
    size_t w = 1;
    ((w = sizeof(T) > w ? sizeof(T) : w), ...);
    return static_cast<int>(16 / w);
}

template <typename O, typename A, typename F>
void run1(const A* a, O* out, size_t n, F f, cudaStream_t s) {
    if (n == 0) return;
    constexpr int E = pack_elems<O, A>();
    size_t done = 0;
    if (aligned(a, sizeof(A) * E) && aligned(out, sizeof(O) * E)) {
        const size_t packs = n / E;
        if (packs) map1_packs<E><<<grid_for(packs), kThreads, 0, s>>>(a, out, packs, f);
        done = packs * E;
    }
    if (done < n) map1_scalar<<<grid_for(n - done), kThreads, 0, s>>>(a, out, done, n, f);
}

template <typename O, typename A, typename B, typename F>
void run2(const A* a, const B* b, O* out, size_t n, F f, cudaStream_t s) {
    if (n == 0) return;
    constexpr int E = pack_elems<O, A, B>();
    size_t done = 0;
    if (aligned(a, sizeof(A) * E) && aligned(b, sizeof(B) * E) && aligned(out, sizeof(O) * E)) {
        const size_t packs = n / E;
        if (packs) map2_packs<E><<<grid_for(packs), kThreads, 0, s>>>(a, b, out, packs, f);
        done = packs * E;
    }
    if (done < n) map2_scalar<<<grid_for(n - done), kThreads, 0, s>>>(a, b, out, done, n, f);
}

template <typename O, typename C, typename A, typename F>
void run3(const C* c, const A* a, const A* b, O* out, size_t n, F f, cudaStream_t s) {
    if (n == 0) return;
    constexpr int E = pack_elems<O, C, A>();
    size_t done = 0;
    if (aligned(c, sizeof(C) * E) && aligned(a, sizeof(A) * E) && aligned(b, sizeof(A) * E) &&
        aligned(out, sizeof(O) * E)) {
        const size_t packs = n / E;
        if (packs) map3_packs<E><<<grid_for(packs), kThreads, 0, s>>>(c, a, b, out, packs, f);
        done = packs * E;
    }
    if (done < n) map3_scalar<<<grid_for(n - done), kThreads, 0, s>>>(c, a, b, out, done, n, f);
}

// Generator kernel for fill (no input).
template <typename T>
__global__ void __launch_bounds__(kThreads) fill_kernel(T* __restrict__ out, size_t n, T v) {
    const size_t stride = static_cast<size_t>(gridDim.x) * kThreads;
    for (size_t i = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride) out[i] = v;
}

// ---------------------------------------------------------------- f32 functions
#define FN1(NAME, EXPR) \
    struct NAME {       \
        __device__ float operator()(float x) const { return EXPR; } \
    };
#define FN2(NAME, EXPR) \
    struct NAME {       \
        __device__ float operator()(float a, float b) const { return EXPR; } \
    };

FN2(FSub, a - b)
FN2(FDiv, a / b)
FN2(FMax, fmaxf(a, b))
FN2(FMin, fminf(a, b))
FN2(FMod, fmodf(a, b))
FN1(FNeg, -x)
FN1(FAbs, fabsf(x))
FN1(FExp, expf(x))
FN1(FLog, logf(x))
FN1(FSqrt, sqrtf(x))
FN1(FRsqrt, rsqrtf(x))
FN1(FSin, sinf(x))
FN1(FCos, cosf(x))
FN1(FTanh, tanhf(x))
FN1(FCeil, ceilf(x))
FN1(FFloor, floorf(x))
FN1(FRound, roundf(x))
FN1(FSqr, x * x)
FN1(FRecip, 1.0f / x)
FN1(FLog2, log2f(x))
FN1(FLog10, log10f(x))
FN1(FTan, tanf(x))
FN1(FSinh, sinhf(x))
FN1(FCosh, coshf(x))
FN1(FSign, (x > 0.0f) ? 1.0f : ((x < 0.0f) ? -1.0f : 0.0f))
FN1(FRelu6, fminf(6.0f, fmaxf(0.0f, x)))
FN1(FSelu, kSeluLambda * (x > 0.0f ? x : kSeluAlpha * (expf(x) - 1.0f)))
FN1(FSilu, x / (1.0f + expf(-x)))
FN1(FHardswish, x * fminf(fmaxf(x + 3.0f, 0.0f), 6.0f) / 6.0f)
FN1(FHardsigmoid, fminf(fmaxf(x / 6.0f + 0.5f, 0.0f), 1.0f))

// Abramowitz & Stegun 7.1.26 rational approximation of erf, as the
// reference's k_erf_f32 evaluates it.
struct FErf {
    __device__ float operator()(float x) const {
        const float sign = (x >= 0.0f) ? 1.0f : -1.0f;
        const float a = fabsf(x);
        const float t = 1.0f / (1.0f + 0.3275911f * a);
        const float p = ((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t +
                        0.254829592f;
        const float y = 1.0f - p * t * expf(-a * a);
        return sign * y;
    }
};
// tanh form; x^3 first (k_gelu_f32) ...
struct FGelu {
    __device__ float operator()(float x) const {
        const float x3 = x * x * x;
        const float inner = kSqrt2OverPi * (x + kGeluCoef * x3);
        return 0.5f * x * (1.0f + tanhf(inner));
    }
};
// ... or coefficient times x, x, x left to right (k_gelu_tanh_f32).
struct FGeluTanh {
    __device__ float operator()(float x) const {
        const float inner = kSqrt2OverPi * (x + kGeluCoef * x * x * x);
        return 0.5f * x * (1.0f + tanhf(inner));
    }
};
struct FSoftplus {
    __device__ float operator()(float x) const {
        if (x > 20.0f) return x;
        if (x < -20.0f) return expf(x);
        return log1pf(expf(x));
    }
};
struct FMish {
    __device__ float operator()(float x) const {
        const float sp = (x > 20.0f) ? x : log1pf(expf(x));
        return x * tanhf(sp);
    }
};
struct FLeaky {
    float alpha;
    __device__ float operator()(float x) const { return x > 0.0f ? x : alpha * x; }
};
struct FElu {
    float alpha;
    __device__ float operator()(float x) const { return x > 0.0f ? x : alpha * (expf(x) - 1.0f); }
};
struct FClamp {
    float lo, hi;
    __device__ float operator()(float x) const { return fminf(hi, fmaxf(lo, x)); }
};
struct FPow {
    float e;
    __device__ float operator()(float x) const { return powf(x, e); }
};
struct FAddS {
    float s;
    __device__ float operator()(float x) const { return x + s; }
};
struct FSubS {
    float s;
    __device__ float operator()(float x) const { return x - s; }
};
struct FMulS {
    float s;
    __device__ float operator()(float x) const { return x * s; }
};
struct FDivS {
    float s;
    __device__ float operator()(float x) const { return x / s; }
};

#define CMP(NAME, OP)                                                                              \
    struct NAME {                                                                                  \
        __device__ uint8_t operator()(float a, float b) const { return (a OP b) ? 1 : 0; }       \
    };
CMP(CEq, ==)
CMP(CNe, !=)
CMP(CLt, <)
CMP(CLe, <=)
CMP(CGt, >)
CMP(CGe, >=)

struct FWhere {
    __device__ float operator()(uint8_t c, float t, float f) const { return c ? t : f; }
};
struct ToHalf {
    __device__ __half operator()(float x) const { return __float2half(x); }
};
struct FromHalf {
    __device__ float operator()(__half x) const { return __half2float(x); }
};

// ---------------------------------------------------------------- f64 functions
#define DFN1(NAME, EXPR) \
    struct NAME {        \
        __device__ double operator()(double x) const { return EXPR; } \
    };
#define DFN2(NAME, EXPR) \
    struct NAME {        \
        __device__ double operator()(double a, double b) const { return EXPR; } \
    };
DFN2(DAdd, a + b)
DFN2(DSub, a - b)
DFN2(DMul, a * b)
DFN2(DDiv, a / b)
DFN1(DNeg, -x)
DFN1(DExp, exp(x))
DFN1(DLog, log(x))
DFN1(DSqrt, sqrt(x))
DFN1(DTanh, tanh(x))
DFN1(DRelu, fmax(0.0, x))
DFN1(DSigmoid, 1.0 / (1.0 + exp(-x)))
struct DGelu {
    __device__ double operator()(double x) const {
        const double x3 = x * x * x;
        const double inner = 0.7978845608028654 * (x + 0.044715 * x3);
        return 0.5 * x * (1.0 + tanh(inner));
    }
};
struct DAffine {
    double mul, add;
    __device__ double operator()(double x) const { return x * mul + add; }
};

// ---------------------------------------------------------------- f16 functions
struct HAdd {
    __device__ __half operator()(__half a, __half b) const { return __hadd(a, b); }
};
struct HSub {
    __device__ __half operator()(__half a, __half b) const { return __hsub(a, b); }
};
struct HMul {
    __device__ __half operator()(__half a, __half b) const { return __hmul(a, b); }
};
struct HDiv {
    __device__ __half operator()(__half a, __half b) const { return __hdiv(a, b); }
};
struct HRelu {
    __device__ __half operator()(__half x) const {
        const __half zero = __float2half(0.0f);
        return __hgt(x, zero) ? x : zero;
    }
};
struct HGelu {
    __device__ __half operator()(__half h) const { return __float2half(FGelu{}(__half2float(h))); }
};
struct HSigmoid {
    __device__ __half operator()(__half h) const {
        const float x = __half2float(h);
        return __float2half(1.0f / (1.0f + expf(-x)));
    }
};

}  // namespace

extern "C" {

// ---- f32 binary, scalar, unary, activations (ops_core.inl:1-470) -----------------
void ptx_tensor_sub_f32(float* a, float* b, float* out, size_t n, cudaStream_t s) { run2(a, b, out, n, FSub{}, s); }
void ptx_tensor_div_f32(float* a, float* b, float* out, size_t n, cudaStream_t s) { run2(a, b, out, n, FDiv{}, s); }
void ptx_tensor_max_f32(float* a, float* b, float* out, size_t n, cudaStream_t s) { run2(a, b, out, n, FMax{}, s); }
void ptx_tensor_min_f32(float* a, float* b, float* out, size_t n, cudaStream_t s) { run2(a, b, out, n, FMin{}, s); }
void ptx_tensor_mod_f32(float* a, float* b, float* out, size_t n, cudaStream_t s) { run2(a, b, out, n, FMod{}, s); }

void ptx_tensor_add_scalar_f32(float* a, float v, float* out, size_t n, cudaStream_t s) { run1(a, out, n, FAddS{v}, s); }
void ptx_tensor_sub_scalar_f32(float* a, float v, float* out, size_t n, cudaStream_t s) { run1(a, out, n, FSubS{v}, s); }
void ptx_tensor_mul_scalar_f32(float* a, float v, float* out, size_t n, cudaStream_t s) { run1(a, out, n, FMulS{v}, s); }
void ptx_tensor_div_scalar_f32(float* a, float v, float* out, size_t n, cudaStream_t s) { run1(a, out, n, FDivS{v}, s); }

#define UNARY_F32(NAME, F) \
    void NAME(float* in, float* out, size_t n, cudaStream_t s) { run1(in, out, n, F{}, s); }
UNARY_F32(ptx_tensor_neg_f32, FNeg)
UNARY_F32(ptx_tensor_abs_f32, FAbs)
UNARY_F32(ptx_tensor_exp_f32, FExp)
UNARY_F32(ptx_tensor_log_f32, FLog)
UNARY_F32(ptx_tensor_sqrt_f32, FSqrt)
UNARY_F32(ptx_tensor_rsqrt_f32, FRsqrt)
UNARY_F32(ptx_tensor_sin_f32, FSin)
UNARY_F32(ptx_tensor_cos_f32, FCos)
UNARY_F32(ptx_tensor_tanh_f32, FTanh)
UNARY_F32(ptx_tensor_ceil_f32, FCeil)
UNARY_F32(ptx_tensor_floor_f32, FFloor)
UNARY_F32(ptx_tensor_round_f32, FRound)
UNARY_F32(ptx_tensor_sqr_f32, FSqr)
UNARY_F32(ptx_tensor_recip_f32, FRecip)
UNARY_F32(ptx_tensor_log2_f32, FLog2)
UNARY_F32(ptx_tensor_log10_f32, FLog10)
UNARY_F32(ptx_tensor_tan_f32, FTan)
UNARY_F32(ptx_tensor_sinh_f32, FSinh)
UNARY_F32(ptx_tensor_cosh_f32, FCosh)
UNARY_F32(ptx_tensor_sign_f32, FSign)
UNARY_F32(ptx_tensor_erf_f32, FErf)
UNARY_F32(ptx_tensor_relu6_f32, FRelu6)
UNARY_F32(ptx_tensor_selu_f32, FSelu)
UNARY_F32(ptx_tensor_gelu_f32, FGelu)
UNARY_F32(ptx_tensor_gelu_tanh_f32, FGeluTanh)
UNARY_F32(ptx_tensor_silu_f32, FSilu)
UNARY_F32(ptx_tensor_softplus_f32, FSoftplus)
UNARY_F32(ptx_tensor_mish_f32, FMish)
UNARY_F32(ptx_tensor_hardswish_f32, FHardswish)
UNARY_F32(ptx_tensor_hardsigmoid_f32, FHardsigmoid)

void ptx_tensor_leaky_relu_f32(float* in, float* out, size_t n, float alpha, cudaStream_t s) {
    run1(in, out, n, FLeaky{alpha}, s);
}
void ptx_tensor_elu_f32(float* in, float* out, size_t n, float alpha, cudaStream_t s) {
    run1(in, out, n, FElu{alpha}, s);
}
void ptx_tensor_clamp_f32(float* in, float* out, size_t n, float min_val, float max_val, cudaStream_t s) {
    run1(in, out, n, FClamp{min_val, max_val}, s);
}
void ptx_tensor_powf_f32(float* in, float* out, size_t n, float e, cudaStream_t s) { run1(in, out, n, FPow{e}, s); }

// ---- comparisons, select, copy, fill, casts (ops_core.inl:400-470, 1170-1180) ----------
#define CMP_F32(NAME, F) \
    void NAME(float* a, float* b, uint8_t* out, size_t n, cudaStream_t s) { run2(a, b, out, n, F{}, s); }
CMP_F32(ptx_tensor_cmp_eq_f32, CEq)
CMP_F32(ptx_tensor_cmp_ne_f32, CNe)
CMP_F32(ptx_tensor_cmp_lt_f32, CLt)
CMP_F32(ptx_tensor_cmp_le_f32, CLe)
CMP_F32(ptx_tensor_cmp_gt_f32, CGt)
CMP_F32(ptx_tensor_cmp_ge_f32, CGe)

void ptx_tensor_where_f32(uint8_t* cond, float* t, float* f, float* out, size_t n, cudaStream_t s) {
    run3(cond, t, f, out, n, FWhere{}, s);
}
void ptx_tensor_copy_f32(float* in, float* out, size_t n, cudaStream_t s) {
    if (n && in != out) cudaMemcpyAsync(out, in, n * sizeof(float), cudaMemcpyDeviceToDevice, s);
}
void ptx_tensor_fill_f32(float* out, size_t n, float value, cudaStream_t s) {
    if (n) fill_kernel<<<grid_for(n), kThreads, 0, s>>>(out, n, value);
}
void ptx_tensor_cast_f32_to_f16(float* in, __half* out, size_t n, cudaStream_t s) { run1(in, out, n, ToHalf{}, s); }
void ptx_tensor_cast_f16_to_f32(__half* in, float* out, size_t n, cudaStream_t s) { run1(in, out, n, FromHalf{}, s); }

// ---- f64 (ops_core.inl:860-960) -------------------------------------------------------
#define BIN_F64(NAME, F) \
    void NAME(double* a, double* b, double* out, size_t n, cudaStream_t s) { run2(a, b, out, n, F{}, s); }
#define UN_F64(NAME, F) \
    void NAME(double* in, double* out, size_t n, cudaStream_t s) { run1(in, out, n, F{}, s); }
BIN_F64(ptx_tensor_add_f64, DAdd)
BIN_F64(ptx_tensor_sub_f64, DSub)
BIN_F64(ptx_tensor_mul_f64, DMul)
BIN_F64(ptx_tensor_div_f64, DDiv)
UN_F64(ptx_tensor_neg_f64, DNeg)
UN_F64(ptx_tensor_exp_f64, DExp)
UN_F64(ptx_tensor_log_f64, DLog)
UN_F64(ptx_tensor_sqrt_f64, DSqrt)
UN_F64(ptx_tensor_tanh_f64, DTanh)
UN_F64(ptx_tensor_relu_f64, DRelu)
UN_F64(ptx_tensor_gelu_f64, DGelu)
UN_F64(ptx_tensor_sigmoid_f64, DSigmoid)
void ptx_tensor_affine_f64(double* in, double* out, size_t n, double mul, double add, cudaStream_t s) {
    run1(in, out, n, DAffine{mul, add}, s);
}

// ---- f16 (ops_core.inl:1140-1180) -----------------------------------------------------
#define BIN_F16(NAME, F) \
    void NAME(__half* a, __half* b, __half* out, size_t n, cudaStream_t s) { run2(a, b, out, n, F{}, s); }
#define UN_F16(NAME, F) \
    void NAME(__half* in, __half* out, size_t n, cudaStream_t s) { run1(in, out, n, F{}, s); }
BIN_F16(ptx_tensor_add_f16, HAdd)
BIN_F16(ptx_tensor_sub_f16, HSub)
BIN_F16(ptx_tensor_mul_f16, HMul)
BIN_F16(ptx_tensor_div_f16, HDiv)
UN_F16(ptx_tensor_relu_f16, HRelu)
UN_F16(ptx_tensor_gelu_f16, HGelu)
UN_F16(ptx_tensor_sigmoid_f16, HSigmoid)

// ---- graph capture (util_dispatch.inl:608-622) -----------------------------------------
cudaError_t ptx_tensor_graph_begin_capture(cudaStream_t stream) {
    return cudaStreamBeginCapture(stream, cudaStreamCaptureModeGlobal);
}
cudaError_t ptx_tensor_graph_end_capture(cudaStream_t stream, cudaGraph_t* graph_out) {
    return cudaStreamEndCapture(stream, graph_out);
}
cudaError_t ptx_tensor_graph_instantiate(cudaGraph_t graph, cudaGraphExec_t* exec_out) {
    return cudaGraphInstantiate(exec_out, graph, 0);
}
cudaError_t ptx_tensor_graph_launch(cudaGraphExec_t exec, cudaStream_t stream) { return cudaGraphLaunch(exec, stream); }

}  // extern "C"
