// Per-row 64-bit digests of device bytes, for comparing outputs (transformer
// logits) across ranks, GPU counts and runs bit for bit without moving them
// to the host. Row r's digest is the sum mod 2^64 of h(chunk, j) over its
// 16-byte chunks j, h a splitmix64-style mix of both 8-byte halves and j.
// Integer addition commutes exactly, so the result depends only on the row's
// bytes, whatever the grid, and the atomics add nothing nondeterministic.
#include <cuda_runtime.h>

#include <cstdint>

namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// grid (x: chunk blocks, y: rows); 256 threads, 4 chunks per thread in flight
__global__ void row_digest_kernel(const uint4* __restrict__ data, uint64_t chunks_per_row, uint64_t* out) {
    const uint64_t row = blockIdx.y;
    const uint4* src = data + row * chunks_per_row;
    uint64_t acc = 0;
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t j = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < chunks_per_row; j += stride) {
        const uint4 v = __ldg(src + j);
        const uint64_t lo = (static_cast<uint64_t>(v.y) << 32) | v.x, hi = (static_cast<uint64_t>(v.w) << 32) | v.z;
        acc += mix64(lo ^ mix64(hi + 0x9E3779B97F4A7C15ull * (j + 1)));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    __shared__ uint64_t warp_sum[8];
    if ((threadIdx.x & 31) == 0) warp_sum[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint64_t s = 0;
        for (int w = 0; w < 8; ++w) s += warp_sum[w];
        atomicAdd(reinterpret_cast<unsigned long long*>(out + row), static_cast<unsigned long long>(s));
    }
}

}  // namespace

extern "C" cudaError_t fer_row_digests(const void* data, uint64_t row_bytes, uint32_t rows, uint64_t* out,
                                       cudaStream_t s) {
    if (!data || !out || rows == 0 || row_bytes == 0 || row_bytes % 16 || rows > 65535u) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(out, 0, static_cast<size_t>(rows) * 8, s);
    if (e != cudaSuccess) return e;
    const uint64_t chunks = row_bytes / 16;
    uint64_t bx = (chunks + 1023) / 1024;              // about 4 chunks per thread
    const uint64_t cap = (148ull * 16 + rows - 1) / rows;   // ~16 CTAs per SM over all rows
    if (bx > cap) bx = cap;
    if (bx < 1) bx = 1;
    row_digest_kernel<<<dim3(static_cast<unsigned>(bx), rows), 256, 0, s>>>(static_cast<const uint4*>(data), chunks,
                                                                            out);
    return cudaGetLastError();
}
