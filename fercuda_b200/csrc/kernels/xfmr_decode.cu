// Incremental decoding kernels of the transformer driver: the KV cache store
// and single-query attention over the cache (flash-decoding).
//
// KV cache layout, per layer: K and V each [max_batch][heads][max_seq][64]
// bf16, so the history of one (sequence, head) is one contiguous run of
// 128-byte rows: a warp reading 32 consecutive positions reads 4 KB of
// contiguous memory.
//
// Decode attention for one new query per sequence: positions [0, len] of
// each (sequence, head) are split into chunks of kChunk; one CTA per
// (sequence, head, chunk) computes the chunk's scores q.k / 8, their maximum
// m, p = exp(s - m), l = sum p and o = sum p v in f32, in a fixed order; a
// second kernel combines the chunks in chunk order (max, rescale, sum) and
// writes o / l as bf16. With one chunk the first kernel writes the result.
// Every reduction order depends only on len, so results are bit-identical
// run to run.
#include "sm100_util.cuh"

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace {

using bf16 = __nv_bfloat16;
constexpr int HD = 64;
constexpr int kChunk = 256;      // positions per CTA
constexpr int kThreads = 128;

// K and V of rows t = b * S + s (s < S) of qkv [B*S, 3d] into the caches at
// position pos0 + s. One thread per 16-byte piece.
__global__ void kv_store(const bf16* __restrict__ qkv, bf16* __restrict__ kc, bf16* __restrict__ vc, int B, int S,
                         int d, int heads, int max_seq, int pos0) {
    const int per_row = 2 * d / 8;   // 16-byte pieces of K and V in one row
    const size_t total = static_cast<size_t>(B) * S * per_row;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const size_t t = i / per_row;
        const int j = static_cast<int>(i % per_row);
        const int kv = j / (d / 8), w = j % (d / 8);
        const int h = w / 8, part = w % 8;
        const int b = static_cast<int>(t / S), s = static_cast<int>(t % S);
        const uint4 val = *reinterpret_cast<const uint4*>(qkv + t * 3 * d + d + kv * d + h * HD + part * 8);
        bf16* dst = (kv ? vc : kc) + ((static_cast<size_t>(b) * heads + h) * max_seq + pos0 + s) * HD + part * 8;
        *reinterpret_cast<uint4*>(dst) = val;
    }
}

// One row per sequence (S = 1) at the position held in device memory, so a
// captured decode step replays unchanged as the position advances.
__global__ void kv_store_at(const bf16* __restrict__ qkv, bf16* __restrict__ kc, bf16* __restrict__ vc, int B, int d,
                            int heads, int max_seq, const int* __restrict__ d_pos) {
    const int pos = *d_pos;
    const int per_row = 2 * d / 8;
    const int total = B * per_row;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int b = i / per_row, j = i % per_row;
        const int kv = j / (d / 8), w = j % (d / 8);
        const int h = w / 8, part = w % 8;
        if (pos < 0 || pos >= max_seq) return;
        const uint4 val = *reinterpret_cast<const uint4*>(qkv + static_cast<size_t>(b) * 3 * d + d + kv * d + h * HD +
                                                          part * 8);
        bf16* dst = (kv ? vc : kc) + ((static_cast<size_t>(b) * heads + h) * max_seq + pos) * HD + part * 8;
        *reinterpret_cast<uint4*>(dst) = val;
    }
}

__global__ void add_to_int(int* p, int v) { *p += v; }
__global__ void set_int(int* p, int v) { *p = v; }

__device__ __forceinline__ float block_max(float v, float* sh) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    const float r = fmaxf(fmaxf(sh[0], sh[1]), fmaxf(sh[2], sh[3]));
    __syncthreads();
    return r;
}

__device__ __forceinline__ float block_sum(float v, float* sh) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    const float r = (sh[0] + sh[1]) + (sh[2] + sh[3]);
    __syncthreads();
    return r;
}

// grid (B * heads, chunks). q: row b of qkv_dec [B, 3d]. part: per (b, h,
// chunk) the chunk's m, l and o[64] (66 floats), unused when chunks == 1.
__global__ void __launch_bounds__(kThreads) decode_attn_chunk(const bf16* __restrict__ qkv_dec,
                                                              const bf16* __restrict__ kc,
                                                              const bf16* __restrict__ vc, bf16* __restrict__ out,
                                                              float* __restrict__ part, int d, int heads,
                                                              int max_seq, int n_keys_arg,
                                                              const int* __restrict__ d_len) {
    // d_len given: keys 0 .. *d_len (the new token included), and the grid
    // is sized for the cache's largest chunk count
    const int n_keys = d_len ? *d_len + 1 : n_keys_arg;
    const int chunks = (n_keys + kChunk - 1) / kChunk;
    if (static_cast<int>(blockIdx.y) >= chunks || n_keys > max_seq) return;
    __shared__ float q[HD];
    __shared__ float p[kChunk];
    __shared__ float red[4];
    __shared__ float ogrp[16][HD];
    const int bh = blockIdx.x, b = bh / heads, h = bh % heads;
    const int chunk = blockIdx.y;
    const int k0 = chunk * kChunk;
    const int nk = n_keys - k0 < kChunk ? n_keys - k0 : kChunk;
    const int t = threadIdx.x;
    if (t < HD) q[t] = __bfloat162float(qkv_dec[static_cast<size_t>(b) * 3 * d + h * HD + t]) * 0.125f;
    __syncthreads();
    const bf16* kb = kc + (static_cast<size_t>(bh) * max_seq + k0) * HD;
    const bf16* vb = vc + (static_cast<size_t>(bh) * max_seq + k0) * HD;
    // scores: thread t takes keys t, t + 128
    float smax = -INFINITY;
    for (int j = t; j < nk; j += kThreads) {
        const uint4* row = reinterpret_cast<const uint4*>(kb + static_cast<size_t>(j) * HD);
        float s = 0.0f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint4 u = row[c];
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]));
                s = fmaf(q[c * 8 + 2 * e], f.x, s);
                s = fmaf(q[c * 8 + 2 * e + 1], f.y, s);
            }
        }
        p[j] = s;
        smax = fmaxf(smax, s);
    }
    const float m = block_max(smax, red);
    float lsum = 0.0f;
    for (int j = t; j < nk; j += kThreads) {
        const float e = __expf(p[j] - m);
        p[j] = e;
        lsum += e;
    }
    const float l = block_sum(lsum, red);   // also orders the p[] writes before the reads below
    // o = sum_j p_j v[j]: thread t takes dims 8 * (t % 8) .. +7 (one 16-byte
    // piece of a V row) over keys j = t / 8, t / 8 + 16, ...; the 16 key
    // groups are then added in group order
    const int dg = t % 8, kg = t / 8;
    float acc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
    for (int j = kg; j < nk; j += 16) {
        const uint4 u = reinterpret_cast<const uint4*>(vb + static_cast<size_t>(j) * HD)[dg];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
        const float pj = p[j];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]));
            acc[2 * e] = fmaf(pj, f.x, acc[2 * e]);
            acc[2 * e + 1] = fmaf(pj, f.y, acc[2 * e + 1]);
        }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) ogrp[kg][dg * 8 + e] = acc[e];
    __syncthreads();
    if (t < HD) {
        const int i = t;
        float o = ogrp[0][i];
#pragma unroll
        for (int g = 1; g < 16; ++g) o += ogrp[g][i];
        if (chunks == 1) {
            out[static_cast<size_t>(b) * d + h * HD + i] = __float2bfloat16(o / l);
        } else {
            float* pp = part + (static_cast<size_t>(bh) * chunks + chunk) * (HD + 2);
            pp[2 + i] = o;
            if (i == 0) {
                pp[0] = m;
                pp[1] = l;
            }
        }
    }
}

// One warp per (b, h): chunks combined in chunk order.
__global__ void decode_attn_combine(const float* __restrict__ part, bf16* __restrict__ out, int d, int heads,
                                    int chunks_arg, int BH, const int* __restrict__ d_len) {
    const int chunks = d_len ? (*d_len + 1 + kChunk - 1) / kChunk : chunks_arg;
    if (chunks <= 1) return;     // the chunk kernel wrote the result
    const int lane = threadIdx.x & 31;
    const int bh = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (bh >= BH) return;
    const float* pp = part + static_cast<size_t>(bh) * chunks * (HD + 2);
    float M = -INFINITY;
    for (int c = 0; c < chunks; ++c) M = fmaxf(M, pp[c * (HD + 2)]);
    float L = 0.0f, o0 = 0.0f, o1 = 0.0f;
    for (int c = 0; c < chunks; ++c) {
        const float* q = pp + c * (HD + 2);
        const float w = __expf(q[0] - M);
        L = fmaf(q[1], w, L);
        o0 = fmaf(q[2 + lane], w, o0);
        o1 = fmaf(q[2 + 32 + lane], w, o1);
    }
    const int b = bh / heads, h = bh % heads;
    bf16* dst = out + static_cast<size_t>(b) * d + h * HD;
    dst[lane] = __float2bfloat16(o0 / L);
    dst[32 + lane] = __float2bfloat16(o1 / L);
}

}  // namespace

// K / V of B*S rows of qkv [B*S, 3d] into caches [max_batch][heads][max_seq][64]
// at positions pos0 .. pos0 + S - 1. d % 64 == 0, pos0 + S <= max_seq.
extern "C" cudaError_t fer_kv_store(const void* qkv, void* k_cache, void* v_cache, int B, int S, int d, int heads,
                                    int max_seq, int pos0, cudaStream_t s) {
    if (B <= 0 || S <= 0 || d != heads * HD || pos0 < 0 || pos0 + S > max_seq) return cudaErrorInvalidValue;
    const size_t total = static_cast<size_t>(B) * S * (2 * d / 8);
    size_t g = (total + 255) / 256;
    if (g > 148 * 16) g = 148 * 16;
    kv_store<<<static_cast<unsigned>(g), 256, 0, s>>>(static_cast<const bf16*>(qkv), static_cast<bf16*>(k_cache),
                                                      static_cast<bf16*>(v_cache), B, S, d, heads, max_seq, pos0);
    return cudaGetLastError();
}

// Floats of scratch fer_attn_decode needs for B sequences and n_keys keys.
extern "C" size_t fer_attn_decode_scratch_floats(int B, int heads, int n_keys) {
    const int chunks = (n_keys + kChunk - 1) / kChunk;
    return chunks > 1 ? static_cast<size_t>(B) * heads * chunks * (HD + 2) : 0;
}

// One query per sequence (row b of qkv_dec [B, 3d], its Q part) against keys
// / values 0 .. n_keys - 1 of the caches; out [B, d] bf16.
extern "C" cudaError_t fer_attn_decode(const void* qkv_dec, const void* k_cache, const void* v_cache, void* out,
                                       float* scratch, int B, int d, int heads, int max_seq, int n_keys,
                                       cudaStream_t s) {
    if (B <= 0 || d != heads * HD || n_keys <= 0 || n_keys > max_seq) return cudaErrorInvalidValue;
    const int chunks = (n_keys + kChunk - 1) / kChunk;
    if (chunks > 1 && !scratch) return cudaErrorInvalidValue;
    const dim3 grid(static_cast<unsigned>(B * heads), static_cast<unsigned>(chunks));
    decode_attn_chunk<<<grid, kThreads, 0, s>>>(static_cast<const bf16*>(qkv_dec), static_cast<const bf16*>(k_cache),
                                                static_cast<const bf16*>(v_cache), static_cast<bf16*>(out), scratch, d,
                                                heads, max_seq, n_keys, nullptr);
    if (chunks > 1) {
        const int BH = B * heads, wpb = 8;
        decode_attn_combine<<<(BH + wpb - 1) / wpb, 32 * wpb, 0, s>>>(scratch, static_cast<bf16*>(out), d, heads,
                                                                      chunks, BH, nullptr);
    }
    return cudaGetLastError();
}

// The same step with the position in device memory (*d_len = position of
// the new token): K / V stored at *d_len, attention over keys 0 .. *d_len
// (grid sized for max_seq; CTAs past the current chunk count return at
// once), then *d_len advances by one. Launch arguments never change between
// steps, so the sequence can be captured in a CUDA graph once and replayed.
// scratch: fer_attn_decode_scratch_floats(B, heads, max_seq) floats.
extern "C" cudaError_t fer_decode_kv_attention(const void* qkv_dec, void* k_cache, void* v_cache, void* out,
                                               float* scratch, int B, int d, int heads, int max_seq, int* d_len,
                                               cudaStream_t s) {
    if (B <= 0 || d != heads * HD || max_seq <= 0 || !d_len) return cudaErrorInvalidValue;
    const int max_chunks = (max_seq + kChunk - 1) / kChunk;
    if (max_chunks > 1 && !scratch) return cudaErrorInvalidValue;
    const int pieces = B * (2 * d / 8);
    kv_store_at<<<(pieces + 255) / 256, 256, 0, s>>>(static_cast<const bf16*>(qkv_dec), static_cast<bf16*>(k_cache),
                                                     static_cast<bf16*>(v_cache), B, d, heads, max_seq, d_len);
    const dim3 grid(static_cast<unsigned>(B * heads), static_cast<unsigned>(max_chunks));
    decode_attn_chunk<<<grid, kThreads, 0, s>>>(static_cast<const bf16*>(qkv_dec), static_cast<const bf16*>(k_cache),
                                                static_cast<const bf16*>(v_cache), static_cast<bf16*>(out), scratch, d,
                                                heads, max_seq, 0, d_len);
    if (max_chunks > 1) {
        const int BH = B * heads, wpb = 8;
        decode_attn_combine<<<(BH + wpb - 1) / wpb, 32 * wpb, 0, s>>>(scratch, static_cast<bf16*>(out), d, heads,
                                                                      max_chunks, BH, d_len);
    }
    return cudaGetLastError();
}

// *d_len += v / *d_len = v on the stream.
extern "C" cudaError_t fer_device_int_add(int* d_len, int v, cudaStream_t s) {
    add_to_int<<<1, 1, 0, s>>>(d_len, v);
    return cudaGetLastError();
}
extern "C" cudaError_t fer_device_int_set(int* d_len, int v, cudaStream_t s) {
    set_int<<<1, 1, 0, s>>>(d_len, v);
    return cudaGetLastError();
}
