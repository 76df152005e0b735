// Element access by buffer dtype (fer_buffer_dtype_t codes of the C ABI),
// through f32: the conversions of the reference's cast kernels
// (src/runtime/exec_planner.cu:36-102, k_cast_to_f32 / k_cast_from_f32):
// exact widening on load; on store f16 / bf16 round to nearest even, i8 / u8
// clamp to their range and round to nearest even.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstddef>
#include <cstdint>

namespace fer::dev {

// Buffer dtype codes of the C ABI (fer_buffer_dtype_t).
enum : uint32_t { kF32 = 0, kF16 = 1, kBF16 = 2, kI8 = 3, kU8 = 4 };

template <uint32_t DT> struct Elem;
template <> struct Elem<kF32> {
    using T = float;
    __device__ static float load(const T* p, size_t i) { return p[i]; }
    __device__ static void store(T* p, size_t i, float v) { p[i] = v; }
};
template <> struct Elem<kF16> {
    using T = __half;
    __device__ static float load(const T* p, size_t i) { return __half2float(p[i]); }
    __device__ static void store(T* p, size_t i, float v) { p[i] = __float2half_rn(v); }
};
template <> struct Elem<kBF16> {
    using T = __nv_bfloat16;
    __device__ static float load(const T* p, size_t i) { return __bfloat162float(p[i]); }
    __device__ static void store(T* p, size_t i, float v) { p[i] = __float2bfloat16(v); }
};
template <> struct Elem<kI8> {
    using T = int8_t;
    __device__ static float load(const T* p, size_t i) { return static_cast<float>(p[i]); }
    __device__ static void store(T* p, size_t i, float v) {
        if (v > 127.0f) v = 127.0f;
        if (v < -128.0f) v = -128.0f;
        p[i] = static_cast<int8_t>(nearbyintf(v));
    }
};
template <> struct Elem<kU8> {
    using T = uint8_t;
    __device__ static float load(const T* p, size_t i) { return static_cast<float>(p[i]); }
    __device__ static void store(T* p, size_t i, float v) {
        if (v > 255.0f) v = 255.0f;
        if (v < 0.0f) v = 0.0f;
        p[i] = static_cast<uint8_t>(nearbyintf(v));
    }
};

}  // namespace fer::dev
