// Incremental decoding kernels of the transformer driver: the KV cache store
// and single-query attention over the cache (flash-decoding).
//
// KV cache layout, per layer: K and V each [max_batch][heads][max_seq][64]
// bf16, so the history of one (sequence, head) is one contiguous run of
// 128-byte rows, and one chunk of kChunk positions is one contiguous run of
// kChunk * 128 bytes.
//
// Decode attention for one new query per sequence: positions [0, len] of
// each (sequence, head) are split into chunks of kChunk; one CTA per
// (sequence, head, chunk) computes the scores q.k / 8 (each thread one key,
// a 128-byte row, all its loads in flight at once), their maximum m, p = exp(s - m), l = sum p and o = sum p v
// in f32, in a fixed order, and writes (m, l, o) of the chunk. The last CTA
// of a (sequence, head) to finish (a counter in device memory) combines the
// chunks in chunk order (max, rescale, sum) and writes o / l as bf16; with
// one chunk the CTA writes the result itself. Which CTA combines does not
// change the arithmetic, and every reduction order depends only on len, so
// results are bit-identical run to run.
#include "f32x2.cuh"
#include "pdl.cuh"
#include "sm100_util.cuh"
#include "tmap.cuh"

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace {

using bf16 = __nv_bfloat16;
constexpr int HD = 64;
constexpr int kSub = 32;         // positions per pipeline stage
constexpr int kStages = 3;
constexpr int kRowBytes = HD * 2;                        // one cached position, 128 bytes
constexpr int kStageBytes = 2 * kSub * kRowBytes;        // K rows then V rows, 8 KB
constexpr int kSmemBytes = kStages * kStageBytes + 1024; // + slack for 1024-byte alignment
constexpr int kThreads = 128;                            // 32 key slots x 4 lanes

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

__global__ void add_to_int(int* p, int v) {
    fer::dev::pdl_begin();
    *p += v;
}
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

__device__ __forceinline__ void tma_load_rows(void* dst, const CUtensorMap* map, int row, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            fer::dev::smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(0), "r"(row), "r"(fer::dev::smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ uint4 lds128(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }

// The two bf16 of a 32-bit word as a packed f32 pair (low element first).
__device__ __forceinline__ uint64_t bf16x2_to_f2(uint32_t w) {
    return fer::dev::f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// Address of 16-byte piece c of row r in a 128-byte-swizzled stage.
__device__ __forceinline__ int swz(int r, int c) { return r * kRowBytes + ((c ^ (r & 7)) << 4); }

// Keys [k0, k0 + nk) of one (sequence, head) in stages of kSub positions:
// tmK / tmV are maps over the cache rows (box 64 x kSub, 128-byte swizzle),
// so a stage of K and V is two TMA loads; kStages stages in flight.
// Thread t = 4 * slot + qt owns key slot `slot` of every stage and dims
// 16 qt .. 16 qt + 15: it adds its part of q.k (two 16-byte pieces; even and
// odd dims in two packed f32x2 chains, in dim order, then added), the four
// parts are added by a fixed butterfly (every lane of the
// slot gets the same score), and the slot keeps its own running maximum m,
// sum l and o[16 dims] (online softmax, rescaled when m grows). At the end
// the 32 slots are combined in slot order.
//
// grid (B * heads, G). With G > 1 the keys are split into chunks of
// clen = ceil(n_keys / G) rounded up to kSub (CTAs past the last chunk
// return); each chunk CTA writes (m, l, o[64]) to part, and the last CTA of
// a (sequence, head) to finish (counters, zero before the launch and left
// zero) combines the chunks in chunk order. With one chunk the CTA writes
// the result. d_len given (a decode step): keys 0 .. *d_len, where position
// *d_len is the new token, whose K / V rows come from qkv_dec (stored into
// the caches here, and into the stage in place of the loaded rows); d_len
// null: keys 0 .. n_keys_arg - 1, all from the caches.
__global__ void __launch_bounds__(kThreads) decode_attn(const __grid_constant__ CUtensorMap tmK,
                                                        const __grid_constant__ CUtensorMap tmV,
                                                        const bf16* __restrict__ qkv_dec, bf16* __restrict__ kc,
                                                        bf16* __restrict__ vc, bf16* __restrict__ out,
                                                        float* __restrict__ part, int* __restrict__ counters, int d,
                                                        int heads, int max_seq, int n_keys_arg,
                                                        const int* __restrict__ d_len, uint32_t* err) {
    using namespace fer::dev;
    // A decode step (d_len given) finds *d_len and the cache rows below it
    // written two or more kernels back, so it reads them (and issues the
    // first stage loads) before the programmatic launch wait; q and the new
    // row come from the kernel just before and are read after it.
    const bool early = d_len != nullptr;
    if (threadIdx.x == 0) {
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
    }
    if (!early) pdl_wait();
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full[kStages];
    __shared__ int is_last;
    const int pos = d_len ? *d_len : -1;
    const int n_keys = d_len ? pos + 1 : n_keys_arg;
    if (n_keys <= 0 || n_keys > max_seq) return;          // refused by the host
    const int G = static_cast<int>(gridDim.y);
    const int clen = ((n_keys + G - 1) / G + kSub - 1) / kSub * kSub;
    const int chunks = (n_keys + clen - 1) / clen;
    const int chunk = blockIdx.y;
    if (chunk >= chunks) return;
    const int bh = blockIdx.x, b = bh / heads, h = bh % heads;
    const int k0 = chunk * clen;
    const int nk = n_keys - k0 < clen ? n_keys - k0 : clen;
    const int nsub = (nk + kSub - 1) / kSub;
    const int j_new = d_len ? pos - k0 : -1;              // chunk-local index of the new key, when in [0, nk)
    const int row0 = bh * max_seq + k0;
    uint8_t* st = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int t = threadIdx.x, slot = t >> 2, qt = t & 3;

    if (t == 0) {
        for (int i = 0; i < kStages; ++i) mbar_init(&full[i], 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](int i) {
        uint8_t* sk = st + (i % kStages) * kStageBytes;
        mbar_arrive_expect_tx(&full[i % kStages], kStageBytes);
        tma_load_rows(sk, &tmK, row0 + i * kSub, &full[i % kStages]);
        tma_load_rows(sk + kSub * kRowBytes, &tmV, row0 + i * kSub, &full[i % kStages]);
    };
    if (t == 0)
        for (int i = 0; i < kStages && i < nsub; ++i) issue(i);
    if (early) pdl_wait();
    pdl_trigger();

    const bf16* qrow = qkv_dec + static_cast<size_t>(b) * 3 * d;
    float qr[16];
#pragma unroll
    for (int e = 0; e < 16; e += 2) {
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(qrow + h * HD + 16 * qt + e));
        qr[e] = f.x * 0.125f;
        qr[e + 1] = f.y * 0.125f;
    }
    const bool has_new = j_new >= 0 && j_new < nk;
    uint4 new_piece = make_uint4(0, 0, 0, 0);
    if (has_new && t < 16) {
        // t < 8: K piece t, else V piece t - 8; also stored into the cache
        const int kv = t >> 3, piece = t & 7;
        new_piece = *reinterpret_cast<const uint4*>(qrow + d + kv * d + h * HD + piece * 8);
        *reinterpret_cast<uint4*>((kv ? vc : kc) + (static_cast<size_t>(row0) + j_new) * HD + piece * 8) = new_piece;
    }

    uint64_t q2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) q2[e] = f2_pack(qr[2 * e], qr[2 * e + 1]);
    float m = -INFINITY, l = 0.0f;
    uint64_t acc2[8];   // o[16 dims] as packed pairs
#pragma unroll
    for (int e = 0; e < 8; ++e) acc2[e] = 0ull;
    for (int i = 0; i < nsub; ++i) {
        const int s_i = i % kStages;
        const bool ok = mbar_wait(&full[s_i], static_cast<uint32_t>(i / kStages) & 1u);
        if (!__syncthreads_and(ok)) {
            if (t == 0) {
                report(err, kErrTimeoutLoad);
                // bounded: let the loads this CTA issued (sub-chunks i .. i + kStages - 1) land before it exits
                for (int k = i; k < i + kStages && k < nsub; ++k)
                    mbar_wait(&full[k % kStages], static_cast<uint32_t>(k / kStages) & 1u);
            }
            return;
        }
        uint8_t* sk = st + s_i * kStageBytes;
        uint8_t* sv = sk + kSub * kRowBytes;
        const int jn = j_new - i * kSub;
        if (has_new && jn >= 0 && jn < kSub) {            // the same branch for the whole CTA
            if (t < 16) *reinterpret_cast<uint4*>((t < 8 ? sk : sv) + swz(jn, t & 7)) = new_piece;
            __syncthreads();
        }
        const int j = i * kSub + slot;
        uint64_t s2 = 0ull;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            const uint4 u = lds128(sk + swz(slot, 2 * qt + cc));
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) s2 = f2_fma(q2[4 * cc + e], bf16x2_to_f2(w[e]), s2);
        }
        float s_lo, s_hi;
        f2_unpack(s2, s_lo, s_hi);
        float s = s_lo + s_hi;
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        if (j < nk) {
            if (s > m) {
                const float alpha = __expf(m - s);
                l *= alpha;
                const uint64_t a2 = f2_splat(alpha);
#pragma unroll
                for (int e = 0; e < 8; ++e) acc2[e] = f2_mul(acc2[e], a2);
                m = s;
            }
            const float pj = __expf(s - m);
            l += pj;
            const uint64_t p2 = f2_splat(pj);
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
                const uint4 u = lds128(sv + swz(slot, 2 * qt + cc));
                const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) acc2[4 * cc + e] = f2_fma(p2, bf16x2_to_f2(w[e]), acc2[4 * cc + e]);
            }
        }
        if (has_new) fence_proxy_async_smem();            // a generic write may precede the stage's next load
        __syncthreads();                                  // stage s_i fully read
        if (t == 0 && i + kStages < nsub) issue(i + kStages);
    }

    // combine the 32 slots in slot order (the stage ring is idle now)
    float* so = reinterpret_cast<float*>(st);              // [32][64]
    float* sm = so + 32 * HD;                              // [32]
    float* sl = sm + 32;                                   // [32]
    float acc[16];
#pragma unroll
    for (int e = 0; e < 8; ++e) f2_unpack(acc2[e], acc[2 * e], acc[2 * e + 1]);
#pragma unroll
    for (int e = 0; e < 16; e += 4)
        *reinterpret_cast<float4*>(so + slot * HD + 16 * qt + e) = make_float4(acc[e], acc[e + 1], acc[e + 2], acc[e + 3]);
    if (qt == 0) {
        sm[slot] = m;
        sl[slot] = l;
    }
    __syncthreads();
    bf16* dst = out + static_cast<size_t>(b) * d + h * HD;
    float M = -INFINITY, L = 0.0f, o = 0.0f;
    if (t < HD) {
        for (int k = 0; k < 32; ++k) M = fmaxf(M, sm[k]);
        for (int k = 0; k < 32; ++k) {
            const float w = __expf(sm[k] - M);             // 0 for a slot that saw no key
            L = fmaf(sl[k], w, L);
            o = fmaf(so[k * HD + t], w, o);
        }
    }
    if (chunks == 1) {
        if (t < HD) dst[t] = __float2bfloat16(o / L);
        return;
    }
    float* pp = part + static_cast<size_t>(bh) * chunks * (HD + 2);
    if (t < HD) {
        pp[chunk * (HD + 2) + 2 + t] = o;
        if (t == 0) {
            pp[chunk * (HD + 2)] = M;
            pp[chunk * (HD + 2) + 1] = L;
        }
        __threadfence();
    }
    __syncthreads();
    if (t == 0) is_last = atomicAdd(&counters[bh], 1) == chunks - 1;
    __syncthreads();
    if (!is_last) return;
    // every chunk of (b, h) is written: combine them in chunk order
    __threadfence();
    if (t < HD) {
        float Mc = -INFINITY;
        for (int c = 0; c < chunks; ++c) Mc = fmaxf(Mc, __ldcg(pp + c * (HD + 2)));
        float Lc = 0.0f, oc = 0.0f;
        for (int c = 0; c < chunks; ++c) {
            const float* qc = pp + c * (HD + 2);
            const float w = __expf(__ldcg(qc) - Mc);
            Lc = fmaf(__ldcg(qc + 1), w, Lc);
            oc = fmaf(__ldcg(qc + 2 + t), w, oc);
        }
        dst[t] = __float2bfloat16(oc / Lc);
        if (t == 0) counters[bh] = 0;
    }
}

int sm_count() {
    static int n = [] {
        int dev = 0, v = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v > 0 ? v : 148;
    }();
    return n;
}

// Chunks per (sequence, head): enough CTAs for one full wave when B * heads
// alone does not fill the GPU, never more than one per kSub keys.
int grid_chunks(int BH, int max_keys, int resident_per_sm) {
    const int by_keys = (max_keys + kSub - 1) / kSub;
    int g = sm_count() * resident_per_sm / BH;
    if (g > by_keys) g = by_keys;
    return g < 1 ? 1 : g;
}

int resident_per_sm() {
    static int r = [] {
        int v = 0;
        if (cudaFuncSetAttribute(decode_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, decode_attn, kThreads, kSmemBytes) != cudaSuccess) {
            cudaGetLastError();
            v = 0;
        }
        return v;
    }();
    return r;
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

// Floats of scratch fer_attn_decode needs for B sequences and n_keys keys
// (and fer_decode_kv_attention for any batch up to B): chunk partials of 66
// floats, as many as B' * heads * G can reach for B' <= B (G <= 16 * SMs /
// (B' * heads) when it exceeds one, at most 16 CTAs being resident per SM),
// then one counter per (sequence, head). 0 when no launch splits the keys.
extern "C" size_t fer_attn_decode_scratch_floats(int B, int heads, int n_keys) {
    if (B <= 0 || heads <= 0 || n_keys <= 0) return 0;
    const size_t BH = static_cast<size_t>(B) * heads;
    const size_t by_keys = static_cast<size_t>((n_keys + kSub - 1) / kSub);
    if (by_keys <= 1) return 0;
    size_t parts = static_cast<size_t>(sm_count()) * 16;
    if (parts < BH) parts = BH;
    if (parts > BH * by_keys) parts = BH * by_keys;
    return parts * (HD + 2) + BH;
}

namespace {

cudaError_t launch_decode_attn(const void* qkv_dec, void* k_cache, void* v_cache, void* out, float* scratch,
                               int* counters, int B, int d, int heads, int max_seq, int n_keys, int max_keys,
                               const int* d_len, uint32_t* err, bool pdl, cudaStream_t s) {
    const int res = resident_per_sm();
    if (res <= 0) return cudaErrorInvalidConfiguration;
    const int BH = B * heads;
    const int G = grid_chunks(BH, max_keys, res);
    if (G > 1 && (!scratch || !counters)) return cudaErrorInvalidValue;
    CUtensorMap mk, mv;
    const unsigned long long rows = static_cast<unsigned long long>(BH) * max_seq;
    if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15u ||
        !fer::host::map_rows64_bf16(&mk, k_cache, rows, kSub) || !fer::host::map_rows64_bf16(&mv, v_cache, rows, kSub))
        return cudaErrorInvalidValue;
    const dim3 grid(static_cast<unsigned>(BH), static_cast<unsigned>(G));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl && fer::host::pdl_enabled() ? 1 : 0;
    fer_pdl_note_launch();   // the kernel triggers its dependents either way
    const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_attn, mk, mv, static_cast<const bf16*>(qkv_dec),
                                             static_cast<bf16*>(k_cache), static_cast<bf16*>(v_cache),
                                             static_cast<bf16*>(out), scratch, counters, d, heads, max_seq, n_keys,
                                             d_len, err);
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace

// One query per sequence (row b of qkv_dec [B, 3d], its Q part) against keys
// / values 0 .. n_keys - 1 of the caches; out [B, d] bf16. scratch:
// fer_attn_decode_scratch_floats(B, heads, n_keys) floats (its counters are
// cleared here, on the stream).
extern "C" cudaError_t fer_attn_decode(const void* qkv_dec, const void* k_cache, const void* v_cache, void* out,
                                       float* scratch, int B, int d, int heads, int max_seq, int n_keys,
                                       uint32_t* err, cudaStream_t s) {
    if (B <= 0 || d != heads * HD || n_keys <= 0 || n_keys > max_seq) return cudaErrorInvalidValue;
    const size_t nf = fer_attn_decode_scratch_floats(B, heads, n_keys);
    if (nf && !scratch) return cudaErrorInvalidValue;
    const size_t BH = static_cast<size_t>(B) * heads;
    int* counters = nf ? reinterpret_cast<int*>(scratch + nf - BH) : nullptr;
    if (counters) {
        const cudaError_t e = cudaMemsetAsync(counters, 0, BH * sizeof(int), s);
        if (e != cudaSuccess) return e;
    }
    // the caches are only read on this path (d_len null)
    return launch_decode_attn(qkv_dec, const_cast<void*>(k_cache), const_cast<void*>(v_cache), out, scratch,
                              counters, B, d, heads, max_seq, n_keys, n_keys, nullptr, err, false, s);
}

// The same step with the position in device memory (*d_len = position of
// the new token): attention over keys 0 .. *d_len, the new token's K / V
// taken from qkv_dec and stored at *d_len in the same kernel (the chunk
// count is fixed from max_seq; CTAs past the current chunk count return at
// once). The caller advances *d_len afterwards. Launch arguments never change
// between steps, so the sequence can be captured in a CUDA graph once and
// replayed. scratch: fer_attn_decode_scratch_floats(B, heads, max_seq)
// floats or more; counters: B * heads ints, zero before the first call
// (each call leaves them zero).
extern "C" cudaError_t fer_decode_kv_attention(const void* qkv_dec, void* k_cache, void* v_cache, void* out,
                                               float* scratch, int* counters, int B, int d, int heads, int max_seq,
                                               int* d_len, uint32_t* err, cudaStream_t s) {
    if (B <= 0 || d != heads * HD || max_seq <= 0 || !d_len) return cudaErrorInvalidValue;
    return launch_decode_attn(qkv_dec, k_cache, v_cache, out, scratch, counters, B, d, heads, max_seq, 0, max_seq,
                              d_len, err, true, s);
}

// *d_len += v / *d_len = v on the stream.
extern "C" cudaError_t fer_device_int_add(int* d_len, int v, cudaStream_t s) {
    const cudaError_t e = fer::host::launch_pdl(add_to_int, dim3(1), dim3(1), 0, s, d_len, v);
    return e != cudaSuccess ? e : cudaGetLastError();
}
extern "C" cudaError_t fer_device_int_set(int* d_len, int v, cudaStream_t s) {
    set_int<<<1, 1, 0, s>>>(d_len, v);
    return cudaGetLastError();
}
