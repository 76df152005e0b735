// GEMM in the reference's accumulation order, and dtype casts.
//
// fer_submit_matmul in the reference (src/runtime/exec_planner.cu:189-302)
// casts non-f32 operands to f32 temporaries (k_cast_to_f32, :36-63), runs
// k_matmul_f32 (src/runtime/ops_bridge.cu:13-31) - one __fmaf_rn chain per
// output over k = 0 .. ceil(K/16)*16 - 1 with zero padding - and casts the
// result back (k_cast_from_f32, :65-102). This kernel computes the same chain
// per output, so results are bit-identical, but:
//   - it converts operands while staging tiles and converts the output in the
//     epilogue (no temporaries, no extra passes);
//   - each thread keeps an 8x8 block of accumulators in registers over a
//     128x128 output tile (the reference: one output per thread, 16x16 tiles).
// The K order per output is untouched: it is the chain that fixes the bits.
#include "elem.cuh"

#include <cuda_runtime.h>

#include <cstdint>

namespace {

using namespace fer::dev;

constexpr int BM = 128, BN = 128, BK = 16, TM = 8, TN = 8;
constexpr int kThreads = (BM / TM) * (BN / TN);  // 256

template <uint32_t DT, uint32_t DT_OUT = DT>
__global__ void __launch_bounds__(kThreads) matmul_ref_order(const typename Elem<DT>::T* __restrict__ A,
                                                             const typename Elem<DT>::T* __restrict__ B,
                                                             typename Elem<DT_OUT>::T* __restrict__ C, int M, int K,
                                                             int N) {
    __shared__ float As[2][BK][BM];
    __shared__ float Bs[2][BK][BN];
    const int tid = threadIdx.x;
    const int tx = tid % (BN / TN), ty = tid / (BN / TN);
    const int row0 = blockIdx.y * BM, col0 = blockIdx.x * BN;
    // k runs to the reference's padded bound; k >= K reads zeros.
    const int kpad = (K + 15) / 16 * 16;
    const int ntiles = kpad / BK;

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

    // Staging: each thread loads 8 A values and 8 B values per K tile.
    auto stage = [&](int buf, int kt) {
        const int k0 = kt * BK;
#pragma unroll
        for (int u = 0; u < (BM * BK) / kThreads; ++u) {
            const int e = tid + u * kThreads;     // 0 .. 2047
            const int m = e / BK, k = e % BK;     // consecutive threads walk k
            const int gr = row0 + m, gk = k0 + k;
            As[buf][k][m] = (gr < M && gk < K) ? Elem<DT>::load(A, static_cast<size_t>(gr) * K + gk) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < (BN * BK) / kThreads; ++u) {
            const int e = tid + u * kThreads;
            const int k = e / BN, n = e % BN;     // consecutive threads walk n
            const int gk = k0 + k, gc = col0 + n;
            Bs[buf][k][n] = (gk < K && gc < N) ? Elem<DT>::load(B, static_cast<size_t>(gk) * N + gc) : 0.0f;
        }
    };

    stage(0, 0);
    __syncthreads();
    for (int kt = 0; kt < ntiles; ++kt) {
        const int cur = kt & 1;
        if (kt + 1 < ntiles) stage(cur ^ 1, kt + 1);
#pragma unroll
        for (int k = 0; k < BK; ++k) {
            float a[TM], b[TN];
#pragma unroll
            for (int i = 0; i < TM; ++i) a[i] = As[cur][k][ty + i * (BM / TM)];
#pragma unroll
            for (int j = 0; j < TN; ++j) b[j] = Bs[cur][k][tx + j * (BN / TN)];
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int r = row0 + ty + i * (BM / TM);
        if (r >= M) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const int c = col0 + tx + j * (BN / TN);
            if (c < N) Elem<DT_OUT>::store(C, static_cast<size_t>(r) * N + c, acc[i][j]);
        }
    }
}

template <uint32_t DT>
cudaError_t launch_mm(const void* a, const void* b, void* c, int M, int K, int N, cudaStream_t s) {
    using T = typename Elem<DT>::T;
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    matmul_ref_order<DT><<<grid, kThreads, 0, s>>>(static_cast<const T*>(a), static_cast<const T*>(b),
                                                     static_cast<T*>(c), M, K, N);
    return cudaGetLastError();
}

template <uint32_t DT>
__global__ void cast_to_f32(const typename Elem<DT>::T* in, float* out, size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = Elem<DT>::load(in, i);
}

template <uint32_t DT>
__global__ void cast_from_f32(const float* in, typename Elem<DT>::T* out, size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        Elem<DT>::store(out, i, in[i]);
}

unsigned cast_grid(size_t n) {
    size_t g = (n + 255) / 256;
    if (g > 148 * 16) g = 148 * 16;
    return static_cast<unsigned>(g ? g : 1);
}

}  // namespace

extern "C" cudaError_t fer_matmul_ref_order(const void* a, const void* b, void* c, int M, int K, int N,
                                            uint32_t dtype, cudaStream_t stream) {
    if (M <= 0 || N <= 0 || K < 0) return cudaErrorInvalidValue;
    switch (dtype) {
        case kF32: return launch_mm<kF32>(a, b, c, M, K, N, stream);
        case kF16: return launch_mm<kF16>(a, b, c, M, K, N, stream);
        case kBF16: return launch_mm<kBF16>(a, b, c, M, K, N, stream);
        case kI8: return launch_mm<kI8>(a, b, c, M, K, N, stream);
        case kU8: return launch_mm<kU8>(a, b, c, M, K, N, stream);
        default: return cudaErrorInvalidValue;
    }
}

// bf16 operands, f32 output, same per-output chain (used by fer_submit_gemm
// for shapes the tensor-core kernel does not take).
extern "C" cudaError_t fer_matmul_bf16_f32_ref_order(const void* a, const void* b, float* c, int M, int K, int N,
                                                     cudaStream_t stream) {
    if (M <= 0 || N <= 0 || K < 0) return cudaErrorInvalidValue;
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    matmul_ref_order<kBF16, kF32><<<grid, kThreads, 0, stream>>>(static_cast<const __nv_bfloat16*>(a),
                                                                  static_cast<const __nv_bfloat16*>(b), c, M, K, N);
    return cudaGetLastError();
}

extern "C" cudaError_t fer_cast_to_f32(const void* in, float* out, size_t n, uint32_t dtype, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    switch (dtype) {
        case kF32: return cudaMemcpyAsync(out, in, n * 4, cudaMemcpyDeviceToDevice, s);
        case kF16: cast_to_f32<kF16><<<cast_grid(n), 256, 0, s>>>(static_cast<const __half*>(in), out, n); break;
        case kBF16: cast_to_f32<kBF16><<<cast_grid(n), 256, 0, s>>>(static_cast<const __nv_bfloat16*>(in), out, n); break;
        case kI8: cast_to_f32<kI8><<<cast_grid(n), 256, 0, s>>>(static_cast<const int8_t*>(in), out, n); break;
        case kU8: cast_to_f32<kU8><<<cast_grid(n), 256, 0, s>>>(static_cast<const uint8_t*>(in), out, n); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

extern "C" cudaError_t fer_cast_from_f32(const float* in, void* out, size_t n, uint32_t dtype, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    switch (dtype) {
        case kF32: return cudaMemcpyAsync(out, in, n * 4, cudaMemcpyDeviceToDevice, s);
        case kF16: cast_from_f32<kF16><<<cast_grid(n), 256, 0, s>>>(in, static_cast<__half*>(out), n); break;
        case kBF16: cast_from_f32<kBF16><<<cast_grid(n), 256, 0, s>>>(in, static_cast<__nv_bfloat16*>(out), n); break;
        case kI8: cast_from_f32<kI8><<<cast_grid(n), 256, 0, s>>>(in, static_cast<int8_t*>(out), n); break;
        case kU8: cast_from_f32<kU8><<<cast_grid(n), 256, 0, s>>>(in, static_cast<uint8_t*>(out), n); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}
