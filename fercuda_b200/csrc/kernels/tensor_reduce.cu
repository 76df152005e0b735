// Native tensor-op ABI, everything that is not elementwise: reductions over
// an (outer, reduce, inner) view, row softmax / log-softmax for f64, f16 and
// log f32, cumsum, argmax / argmin, argsort, topk, gather, index_select,
// scatter_add, and the opcode dispatch (reference
// native/core/include/gpu/tensor_ops.h:181-333 with its dispatch,
// native/core/kernels/modules/tensor_kernels_util_dispatch.inl:200-606).
//
// Floating-point results equal the reference kernels bit for bit: each output
// is formed in the reference's order of operations
// (tensor_kernels_ops_core.inl:480-730, 800-860, 960-1140;
// tensor_kernels_indexing_scan.inl), with the data path rearranged:
//   - reductions: the reference gives each output one 256-thread CTA whose
//     thread t folds elements t, t+256, ... and then combines the 256
//     partials with a __shfl_down tree per warp and one over the 8 warp
//     results. Contiguous rows (inner == 1) keep that structure, in
//     persistent CTAs. Strided views (inner > 1) read 32 (f64: 16) adjacent
//     outputs per CTA so every load is a full 128-byte line, keep the 256
//     partials of each output in registers, and replay the same two trees in
//     shared memory;
//   - softmax variants: persistent CTAs over rows, same three passes;
//   - cumsum over contiguous rows: one thread per row as in the reference
//     (the same sequential chain), fed through 32 x 32 shared-memory tiles
//     so every global access is a full 128-byte line; strided views: one
//     thread per column;
//   - argmax / argmin over contiguous rows: one warp per row, first index of
//     the extreme value (the reference's sequential scan) by a combine that
//     prefers the lower index on ties;
//   - argsort: the reference's bitonic network (same compare-exchange
//     steps, so the same permutation, ties included) on the row staged in
//     shared memory, one thread per compare-exchange pair (the reference
//     walks every element and idles half its threads each step);
//   - topk: one warp per output column instead of one thread, the already
//     chosen indices kept in a shared-memory bitmap; each round picks what
//     the reference's scan picks (NaN handling included);
//   - scatter_add: deterministic (one thread per output column, sources
//     added in index order, each add rounded and flushed as the reference's
//     float atomicAdd does) when there are at least 1024 columns; atomics, as
//     the reference, below that.
// The reference's own behaviour is kept where it is unusual: reduce_min_f64
// combines inside each warp with fmax (its k_reduce_min_f64), dispatch's
// WHERE takes its false branch from the output buffer, indices are clamped
// (gather, index_select) or skipped (scatter_add) as there.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "ptx/gpu/tensor_ops.h"

namespace {

constexpr int kThreads = 256;

int sm_count() {
    static const int n = [] {
        int dev = 0, v = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v > 0 ? v : 148;
    }();
    return n;
}

unsigned persistent_grid(size_t items, int per_sm = 8) {
    const size_t cap = static_cast<size_t>(sm_count()) * per_sm;
    return static_cast<unsigned>(items < cap ? (items ? items : 1) : cap);
}

unsigned grid_for(size_t threads) {
    const size_t g = (threads + kThreads - 1) / kThreads;
    return persistent_grid(g);
}

// ---------------------------------------------------------------- reduction ops
// acc: the per-thread fold; tree: the in-warp __shfl_down combine; cross: the
// combine over the 8 warp results; pad: what lanes 8..31 hold in that last
// tree; id: a thread's start value.
template <typename T>
struct RSum {
    __device__ static T id() { return T(0); }
    __device__ static T pad() { return T(0); }
    __device__ static T acc(T a, T x) { return a + x; }
    __device__ static T tree(T a, T b) { return a + b; }
    __device__ static T cross(T a, T b) { return a + b; }
};
template <typename T>
struct RProd {
    __device__ static T id() { return T(1); }
    __device__ static T pad() { return T(1); }
    __device__ static T acc(T a, T x) { return a * x; }
    __device__ static T tree(T a, T b) { return a * b; }
    __device__ static T cross(T a, T b) { return a * b; }
};
struct RMaxF {
    __device__ static float id() { return -INFINITY; }
    __device__ static float pad() { return -INFINITY; }
    __device__ static float acc(float a, float x) { return fmaxf(a, x); }
    __device__ static float tree(float a, float b) { return fmaxf(a, b); }
    __device__ static float cross(float a, float b) { return fmaxf(a, b); }
};
struct RMinF {
    __device__ static float id() { return INFINITY; }
    __device__ static float pad() { return INFINITY; }
    __device__ static float acc(float a, float x) { return fminf(a, x); }
    __device__ static float tree(float a, float b) { return fminf(a, b); }
    __device__ static float cross(float a, float b) { return fminf(a, b); }
};
struct RMaxD {
    __device__ static double id() { return -INFINITY; }
    __device__ static double pad() { return -INFINITY; }
    __device__ static double acc(double a, double x) { return fmax(a, x); }
    __device__ static double tree(double a, double b) { return fmax(a, b); }
    __device__ static double cross(double a, double b) { return fmax(a, b); }
};
// k_reduce_min_f64: fmin per thread, fmax inside each warp, fmin across warps.
struct RMinDRef {
    __device__ static double id() { return INFINITY; }
    __device__ static double pad() { return INFINITY; }
    __device__ static double acc(double a, double x) { return fmin(a, x); }
    __device__ static double tree(double a, double b) { return fmax(a, b); }
    __device__ static double cross(double a, double b) { return fmin(a, b); }
};

template <typename R, typename T>
__device__ __forceinline__ T warp_tree(T v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = R::tree(v, __shfl_down_sync(0xffffffffu, v, off));
    return v;
}
template <typename R, typename T>
__device__ __forceinline__ T warp_cross(T v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v = R::cross(v, __shfl_down_sync(0xffffffffu, v, off));
    return v;
}

// Contiguous rows: one output per CTA pass, thread t folds t, t+256, ...
template <typename R, typename T>
__global__ void __launch_bounds__(kThreads) reduce_rows(const T* __restrict__ in, T* __restrict__ out, size_t rows,
                                                        size_t len, T scale, bool scaled) {
    __shared__ T part[kThreads / 32];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    for (size_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const T* x = in + row * len;
        T v = R::id();
        for (size_t r = threadIdx.x; r < len; r += kThreads) v = R::acc(v, x[r]);
        v = warp_tree<R>(v);
        if (lane == 0) part[wid] = v;
        __syncthreads();
        if (wid == 0) {
            T u = lane < kThreads / 32 ? part[lane] : R::pad();
            u = warp_cross<R>(u);
            if (lane == 0) out[row] = scaled ? u * scale : u;
        }
        __syncthreads();
    }
}

// Strided views: TW adjacent outputs (inner positions) per CTA. Thread
// (g, l), g < 256/TW, l < TW, owns the partials of slots g, g + G, ... of
// output i0 + l; its loads for one slot are TW adjacent elements.
template <typename R, typename T, int TW>
__global__ void __launch_bounds__(kThreads) reduce_strided(const T* __restrict__ in, T* __restrict__ out,
                                                           size_t outer, size_t len, size_t inner, T scale,
                                                           bool scaled) {
    constexpr int G = kThreads / TW;     // thread groups
    constexpr int S = kThreads / G;      // slots per thread (= TW)
    __shared__ T part[kThreads][TW + 1];
    __shared__ T wsum[kThreads / 32][TW];
    const int l = threadIdx.x % TW, g = threadIdx.x / TW;
    const size_t tiles_per_outer = (inner + TW - 1) / TW;
    for (size_t tile = blockIdx.x; tile < outer * tiles_per_outer; tile += gridDim.x) {
        const size_t o = tile / tiles_per_outer;
        const size_t i = (tile % tiles_per_outer) * TW + l;
        T acc[S];
#pragma unroll
        for (int j = 0; j < S; ++j) acc[j] = R::id();
        if (i < inner) {
            const T* base = in + o * len * inner + i;
            const size_t step = static_cast<size_t>(G) * inner;
            size_t k0 = 0;
            // whole rounds of 256 rows: the S loads of a round are issued
            // together, then folded in slot order
            for (; k0 + kThreads <= len; k0 += kThreads) {
                const T* p = base + (k0 + g) * inner;
                T v[S];
#pragma unroll
                for (int j = 0; j < S; ++j) v[j] = p[j * step];
#pragma unroll
                for (int j = 0; j < S; ++j) acc[j] = R::acc(acc[j], v[j]);
            }
            if (k0 < len) {
#pragma unroll
                for (int j = 0; j < S; ++j) {
                    const size_t r = k0 + g + static_cast<size_t>(G) * j;
                    if (r < len) acc[j] = R::acc(acc[j], base[r * inner]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < S; ++j) part[g + G * j][l] = acc[j];
        __syncthreads();
        // the reference's in-warp trees: warp w holds slots 32w .. 32w+31
        for (int t = threadIdx.x; t < (kThreads / 32) * TW; t += kThreads) {
            const int w = t / TW, c = t % TW;
            T v[32];
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] = part[32 * w + k][c];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int k = 0; k < off; ++k) v[k] = R::tree(v[k], v[k + off]);
            wsum[w][c] = v[0];
        }
        __syncthreads();
        if (threadIdx.x < TW) {
            const int c = threadIdx.x;
            T v[32];
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] = k < kThreads / 32 ? wsum[k][c] : R::pad();
#pragma unroll
            for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                for (int k = 0; k < off; ++k) v[k] = R::cross(v[k], v[k + off]);
            const size_t ii = (tile % tiles_per_outer) * TW + c;
            if (ii < inner) out[o * inner + ii] = scaled ? v[0] * scale : v[0];
        }
        __syncthreads();
    }
}

template <typename R, typename T>
void run_reduce(const T* in, T* out, size_t outer, size_t len, size_t inner, cudaStream_t s, T scale = T(1),
                bool scaled = false) {
    const size_t outputs = outer * inner;
    if (outputs == 0) return;
    if (inner == 1) {
        reduce_rows<R><<<persistent_grid(outputs), kThreads, 0, s>>>(in, out, outputs, len, scale, scaled);
    } else {
        constexpr int TW = sizeof(T) == 8 ? 16 : 32;
        const size_t tiles = outer * ((inner + TW - 1) / TW);
        reduce_strided<R, T, TW><<<persistent_grid(tiles, 4), kThreads, 0, s>>>(in, out, outer, len, inner, scale,
                                                                                 scaled);
    }
}

// ---------------------------------------------------------------- argmax / argmin
// First index r with v > best (argmax) / v < best (argmin), best starting at
// -inf / +inf, index 0 when nothing qualifies (k_reduce_argmax_f32).
template <bool MAX>
__device__ __forceinline__ bool beats(float v, float best) {
    return MAX ? v > best : v < best;
}

template <bool MAX>
__global__ void __launch_bounds__(kThreads) arg_rows(const float* __restrict__ in, int32_t* __restrict__ out,
                                                     size_t rows, size_t len) {
    const int lane = threadIdx.x & 31;
    const size_t warp = (static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const size_t warps = (static_cast<size_t>(gridDim.x) * kThreads) >> 5;
    for (size_t row = warp; row < rows; row += warps) {
        const float* x = in + row * len;
        float best = MAX ? -INFINITY : INFINITY;
        int32_t idx = 0;
        for (size_t r = lane; r < len; r += 32) {
            const float v = x[r];
            if (beats<MAX>(v, best)) {
                best = v;
                idx = static_cast<int32_t>(r);
            }
        }
        // lanes hold the first index of their own extreme; ties go to the
        // lower index, which the sequential scan would have met first
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_down_sync(0xffffffffu, best, off);
            const int32_t oi = __shfl_down_sync(0xffffffffu, idx, off);
            const bool take = beats<MAX>(ov, best) || (ov == best && oi < idx);
            if (lane + off < 32 && take) {
                best = ov;
                idx = oi;
            }
        }
        if (lane == 0) out[row] = (best == (MAX ? -INFINITY : INFINITY)) ? 0 : idx;
    }
}

template <bool MAX>
__global__ void __launch_bounds__(kThreads) arg_strided(const float* __restrict__ in, int32_t* __restrict__ out,
                                                        size_t outer, size_t len, size_t inner) {
    const size_t total = outer * inner;
    const size_t stride = static_cast<size_t>(gridDim.x) * kThreads;
    for (size_t lane = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; lane < total; lane += stride) {
        const size_t base = (lane / inner) * len * inner + lane % inner;
        float best = MAX ? -INFINITY : INFINITY;
        int32_t idx = 0;
        for (size_t r = 0; r < len; ++r) {
            const float v = in[base + r * inner];
            if (beats<MAX>(v, best)) {
                best = v;
                idx = static_cast<int32_t>(r);
            }
        }
        out[lane] = idx;
    }
}

template <bool MAX>
void run_arg(const float* in, int32_t* out, size_t outer, size_t len, size_t inner, cudaStream_t s) {
    if (outer * inner == 0) return;
    if (inner == 1)
        arg_rows<MAX><<<persistent_grid((outer + 7) / 8), kThreads, 0, s>>>(in, out, outer, len);
    else
        arg_strided<MAX><<<grid_for(outer * inner), kThreads, 0, s>>>(in, out, outer, len, inner);
}

// ---------------------------------------------------------------- softmax variants
enum class SM { kF64, kF16, kLogF32 };

__device__ __forceinline__ float amax(float a, float b) { return fmaxf(a, b); }
__device__ __forceinline__ double amax(double a, double b) { return fmax(a, b); }

// One row per CTA pass, the reference's three passes and trees
// (k_softmax_f64, k_softmax_f16, k_log_softmax_f32). A = accumulation type.
// The second and third passes re-read the row, which is still in L1 (one
// row per CTA, at most 32 KB); holding rows in registers instead, with or
// without prefetching the next row, measured slower at 4096 columns.
template <SM MODE, typename T, typename A>
__global__ void __launch_bounds__(kThreads) softmax_rows(const T* __restrict__ in, T* __restrict__ out, size_t rows,
                                                         size_t dim) {
    __shared__ A sh[kThreads / 32 + 1];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    constexpr int kWarps = kThreads / 32;
    for (size_t row = blockIdx.x; row < rows; row += gridDim.x) {
        const T* x = in + row * dim;
        T* y = out + row * dim;
        auto load = [&](size_t i) -> A {
            if constexpr (MODE == SM::kF16)
                return __half2float(x[i]);
            else
                return x[i];
        };
        // max
        A m = -INFINITY;
        for (size_t i = threadIdx.x; i < dim; i += kThreads) m = amax(m, load(i));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) m = amax(m, __shfl_down_sync(0xffffffffu, m, off));
        if (lane == 0) sh[wid] = m;
        __syncthreads();
        if (wid == 0) {
            A u = lane < kWarps ? sh[lane] : A(-INFINITY);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) u = amax(u, __shfl_down_sync(0xffffffffu, u, off));
            if (lane == 0) sh[0] = u;
        }
        __syncthreads();
        const A mx = sh[0];
        __syncthreads();
        // exp and sum
        A sum = 0;
        for (size_t i = threadIdx.x; i < dim; i += kThreads) {
            if constexpr (MODE == SM::kF64) {
                const double e = exp(load(i) - mx);
                y[i] = e;
                sum += e;
            } else if constexpr (MODE == SM::kF16) {
                const float e = expf(load(i) - mx);
                y[i] = __float2half(e);
                sum += e;
            } else {
                sum += expf(load(i) - mx);
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) sum += __shfl_down_sync(0xffffffffu, sum, off);
        if (lane == 0) sh[wid] = sum;
        __syncthreads();
        if (wid == 0) {
            A u = lane < kWarps ? sh[lane] : A(0);
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) u += __shfl_down_sync(0xffffffffu, u, off);
            if (lane == 0) sh[0] = u;
        }
        __syncthreads();
        const A total = sh[0];
        __syncthreads();
        if constexpr (MODE == SM::kF64) {
            const double inv = 1.0 / total;
            for (size_t i = threadIdx.x; i < dim; i += kThreads) y[i] *= inv;
        } else if constexpr (MODE == SM::kF16) {
            const float inv = 1.0f / total;
            for (size_t i = threadIdx.x; i < dim; i += kThreads) y[i] = __float2half(__half2float(y[i]) * inv);
        } else {
            const float ls = logf(total);
            for (size_t i = threadIdx.x; i < dim; i += kThreads) y[i] = x[i] - mx - ls;
        }
        __syncthreads();
    }
}

template <SM MODE, typename T, typename A>
void run_softmax(const T* in, T* out, size_t batch, size_t dim, cudaStream_t s) {
    if (batch) softmax_rows<MODE, T, A><<<persistent_grid(batch), kThreads, 0, s>>>(in, out, batch, dim);
}

// ---------------------------------------------------------------- cumsum
// Contiguous rows: one warp per 32 rows, one lane per row as in the
// reference (whose chain acc += x[k], k = 0, 1, ... this keeps), but the
// data moves in 32 x 32 tiles: each row's next 32 elements arrive as one
// coalesced 128-byte load per row (the following tile's loads are issued
// before the current tile is scanned), pass through a padded shared tile so
// lane r can walk row r, and leave the same way.
constexpr int kScanWarps = 4;

__global__ void __launch_bounds__(kScanWarps * 32) cumsum_rows(const float* __restrict__ in, float* __restrict__ out,
                                                               size_t rows, size_t len) {
    __shared__ float tile[kScanWarps][32][33];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    float (*t)[33] = tile[w];
    const size_t groups = (rows + 31) / 32;
    const size_t warps = static_cast<size_t>(gridDim.x) * kScanWarps;
    for (size_t grp = static_cast<size_t>(blockIdx.x) * kScanWarps + w; grp < groups; grp += warps) {
        const size_t row0 = grp * 32;
        const int nr = static_cast<int>(rows - row0 < 32 ? rows - row0 : 32);
        auto load = [&](size_t c0, float (&v)[32]) {
#pragma unroll
            for (int rr = 0; rr < 32; ++rr)
                v[rr] = (rr < nr && c0 + lane < len) ? in[(row0 + rr) * len + c0 + lane] : 0.0f;
        };
        float cur[32], nxt[32];
        load(0, nxt);
        float acc = 0.0f;
        for (size_t c0 = 0; c0 < len; c0 += 32) {
#pragma unroll
            for (int rr = 0; rr < 32; ++rr) cur[rr] = nxt[rr];
            if (c0 + 32 < len) load(c0 + 32, nxt);
#pragma unroll
            for (int rr = 0; rr < 32; ++rr) t[rr][lane] = cur[rr];
            __syncwarp();
            const int m = static_cast<int>(len - c0 < 32 ? len - c0 : 32);
            if (lane < nr) {
                if (m == 32) {
                    float v[32];
#pragma unroll
                    for (int k = 0; k < 32; ++k) v[k] = t[lane][k];
#pragma unroll
                    for (int k = 0; k < 32; ++k) {
                        acc += v[k];
                        t[lane][k] = acc;
                    }
                } else {
                    for (int k = 0; k < m; ++k) {
                        acc += t[lane][k];
                        t[lane][k] = acc;
                    }
                }
            }
            __syncwarp();
#pragma unroll
            for (int rr = 0; rr < 32; ++rr)
                if (rr < nr && c0 + lane < len) out[(row0 + rr) * len + c0 + lane] = t[rr][lane];
            __syncwarp();
        }
    }
}

__global__ void __launch_bounds__(kThreads) cumsum_strided(const float* __restrict__ in, float* __restrict__ out,
                                                           size_t outer, size_t len, size_t inner) {
    const size_t total = outer * inner;
    const size_t stride = static_cast<size_t>(gridDim.x) * kThreads;
    for (size_t lane = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; lane < total; lane += stride) {
        const size_t base = (lane / inner) * len * inner + lane % inner;
        float acc = 0.0f;
        for (size_t k = 0; k < len; ++k) {
            acc += in[base + k * inner];
            out[base + k * inner] = acc;
        }
    }
}

// ---------------------------------------------------------------- argsort
// The reference's bitonic network over the padded index array (pad =
// next power of two >= ncols; indices >= ncols sort last), with the row's
// values staged in shared memory. Same compare-exchange steps, same result.
template <bool ASC>
__global__ void __launch_bounds__(512) argsort_rows(const float* __restrict__ in, unsigned int* __restrict__ out,
                                                    int ncols, int pad) {
    extern __shared__ unsigned char smem[];
    int* idx = reinterpret_cast<int*>(smem);
    float* val = reinterpret_cast<float*>(smem + static_cast<size_t>(pad) * sizeof(int));
    const size_t row = blockIdx.x;
    const float* x = in + row * ncols;
    for (int c = threadIdx.x; c < pad; c += blockDim.x) idx[c] = c;
    for (int c = threadIdx.x; c < ncols; c += blockDim.x) val[c] = x[c];
    __syncthreads();
    const int pairs = pad >> 1;
    for (int k = 2; k <= pad; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            // pair q joins c (bit j clear) and c | j
            for (int q = threadIdx.x; q < pairs; q += blockDim.x) {
                const int c = ((q & ~(j - 1)) << 1) | (q & (j - 1));
                const int p = c | j;
                const int ic = idx[c], ip = idx[p];
                // k_argsort_asc_f32 / k_argsort_desc_f32, first and second
                // half of each k-block
                bool swap;
                if ((c & k) == 0)
                    swap = ic >= ncols || (ip < ncols && (ASC ? val[ic] > val[ip] : val[ic] < val[ip]));
                else
                    swap = ip >= ncols || (ic < ncols && (ASC ? val[ic] < val[ip] : val[ic] > val[ip]));
                if (swap) {
                    idx[c] = ip;
                    idx[p] = ic;
                }
            }
            __syncthreads();
        }
    }
    for (int c = threadIdx.x; c < ncols; c += blockDim.x) out[row * ncols + c] = static_cast<unsigned int>(idx[c]);
}

// ---------------------------------------------------------------- topk
// Round ki picks, among indices not yet chosen, what the reference's scan
// over d = 0, 1, ... picks: the first unchosen element starts as best and a
// later one replaces it only if strictly better; so the result is the first
// unchosen element if that is NaN, else the lowest-index best non-NaN value.
template <bool LARGEST>
__device__ __forceinline__ bool better(float v, float b) {
    return LARGEST ? v > b : v < b;
}

template <bool LARGEST>
__global__ void __launch_bounds__(32) topk_cols(const float* __restrict__ in, float* __restrict__ values,
                                                int32_t* __restrict__ indices, size_t outer, size_t dim,
                                                size_t inner, size_t k) {
    extern __shared__ unsigned int taken[];  // dim bits
    const int lane = threadIdx.x;
    const size_t words = (dim + 31) / 32;
    const size_t kk = k < dim ? k : dim;
    for (size_t col = blockIdx.x; col < outer * inner; col += gridDim.x) {
        const size_t o = col / inner, i = col % inner;
        const float* x = in + o * dim * inner + i;
        const size_t ob = o * k * inner + i;
        for (size_t w = lane; w < words; w += 32) taken[w] = 0u;
        __syncwarp();
        for (size_t r = 0; r < kk; ++r) {
            // per lane: first unchosen index (and its value), best non-NaN
            constexpr unsigned long long kNone = ~0ull;
            unsigned long long first = kNone;
            float first_v = 0.0f;
            unsigned long long bi = kNone;
            float bv = 0.0f;
            for (size_t d = lane; d < dim; d += 32) {
                if (taken[d >> 5] & (1u << (d & 31))) continue;
                const float v = x[d * inner];
                if (first == kNone) {
                    first = d;
                    first_v = v;
                }
                if (v == v && (bi == kNone || better<LARGEST>(v, bv))) {
                    bi = d;
                    bv = v;
                }
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                const unsigned long long of = __shfl_down_sync(0xffffffffu, first, off);
                const float ofv = __shfl_down_sync(0xffffffffu, first_v, off);
                const unsigned long long obi = __shfl_down_sync(0xffffffffu, bi, off);
                const float obv = __shfl_down_sync(0xffffffffu, bv, off);
                if (lane + off < 32) {
                    if (of < first) {
                        first = of;
                        first_v = ofv;
                    }
                    if (obi != kNone && (bi == kNone || better<LARGEST>(obv, bv) || (obv == bv && obi < bi))) {
                        bi = obi;
                        bv = obv;
                    }
                }
            }
            first = __shfl_sync(0xffffffffu, first, 0);
            if (first == kNone) break;   // nothing left (cannot happen while r < min(k, dim))
            unsigned long long pick = 0;
            float pv = 0.0f;
            if (lane == 0) {
                if (first_v != first_v || bi == kNone) {
                    pick = first;
                    pv = first_v;
                } else {
                    pick = bi;
                    pv = bv;
                }
                values[ob + r * inner] = pv;
                if (indices) indices[ob + r * inner] = static_cast<int32_t>(pick);
                taken[pick >> 5] |= 1u << (pick & 31);
            }
            __syncwarp();
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------- gather / index_select / scatter_add
__device__ __forceinline__ int32_t clamp_index(int32_t idx, size_t n) {
    if (idx < 0) idx += static_cast<int32_t>(n);
    if (idx < 0) idx = 0;
    if (idx >= static_cast<int32_t>(n)) idx = static_cast<int32_t>(n) - 1;
    return idx;
}

__global__ void __launch_bounds__(kThreads) gather_kernel(const float* __restrict__ in,
                                                          const int32_t* __restrict__ indices,
                                                          float* __restrict__ out, size_t outer, size_t in_dim,
                                                          size_t idx_dim, size_t inner) {
    const size_t total = outer * idx_dim * inner;
    const size_t stride = static_cast<size_t>(gridDim.x) * kThreads;
    for (size_t e = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; e < total; e += stride) {
        const size_t o = e / (idx_dim * inner), i = e % inner;
        const int32_t idx = clamp_index(indices[e], in_dim);
        out[e] = in[o * in_dim * inner + static_cast<size_t>(idx) * inner + i];
    }
}

__global__ void __launch_bounds__(kThreads) index_select_kernel(const float* __restrict__ in,
                                                                const int32_t* __restrict__ ids,
                                                                float* __restrict__ out, size_t left, size_t src_dim,
                                                                size_t ids_dim, size_t right) {
    const size_t total = left * ids_dim * right;
    const size_t stride = static_cast<size_t>(gridDim.x) * kThreads;
    for (size_t e = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; e < total; e += stride) {
        const size_t l = e / (ids_dim * right), k = (e / right) % ids_dim, r = e % right;
        const int32_t idx = clamp_index(ids[k], src_dim);
        out[e] = in[l * src_dim * right + static_cast<size_t>(idx) * right + r];
    }
}

// f32 add as the reference's atomicAdd performs it (atom.add.f32: round to
// nearest even, subnormal inputs and result flushed to sign-preserving zero).
__device__ __forceinline__ float add_like_atomic(float a, float b) {
    float r;
    asm("add.rn.ftz.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}

// Deterministic: column (l, r) adds its sources in k order.
__global__ void __launch_bounds__(kThreads) scatter_add_cols(const int32_t* __restrict__ ids,
                                                             const float* __restrict__ src, float* __restrict__ out,
                                                             size_t left, size_t src_dim, size_t dst_dim,
                                                             size_t right) {
    const size_t cols = left * right;
    const size_t stride = static_cast<size_t>(gridDim.x) * kThreads;
    for (size_t c = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; c < cols; c += stride) {
        const size_t l = c / right, r = c % right;
        for (size_t k = 0; k < src_dim; ++k) {
            int32_t idx = ids[k];
            if (idx < 0) idx += static_cast<int32_t>(dst_dim);
            if (idx >= 0 && idx < static_cast<int32_t>(dst_dim))
            {
                float* d = out + l * dst_dim * right + static_cast<size_t>(idx) * right + r;
                *d = add_like_atomic(*d, src[(l * src_dim + k) * right + r]);
            }
        }
    }
}

__global__ void __launch_bounds__(kThreads) scatter_add_atomic(const int32_t* __restrict__ ids,
                                                               const float* __restrict__ src, float* out, size_t left,
                                                               size_t src_dim, size_t dst_dim, size_t right) {
    const size_t total = left * src_dim * right;
    const size_t stride = static_cast<size_t>(gridDim.x) * kThreads;
    for (size_t e = static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x; e < total; e += stride) {
        const size_t l = e / (src_dim * right), k = (e / right) % src_dim, r = e % right;
        int32_t idx = ids[k];
        if (idx < 0) idx += static_cast<int32_t>(dst_dim);
        if (idx >= 0 && idx < static_cast<int32_t>(dst_dim))
            atomicAdd(&out[l * dst_dim * right + static_cast<size_t>(idx) * right + r], src[e]);
    }
}

}  // namespace

extern "C" {

// ---- reductions (ops_core.inl:480-720, launchers :1519-1565; f64 :990-1090) ----------
void ptx_tensor_reduce_sum_f32(float* in, float* out, size_t outer, size_t reduce, size_t inner, cudaStream_t s) {
    run_reduce<RSum<float>>(in, out, outer, reduce, inner, s);
}
void ptx_tensor_reduce_mean_f32(float* in, float* out, size_t outer, size_t reduce, size_t inner, cudaStream_t s) {
    // sum, then times 1/reduce (the reference's second kernel, fused)
    run_reduce<RSum<float>>(in, out, outer, reduce, inner, s, 1.0f / static_cast<float>(reduce), true);
}
void ptx_tensor_reduce_max_f32(float* in, float* out, size_t outer, size_t reduce, size_t inner, cudaStream_t s) {
    run_reduce<RMaxF>(in, out, outer, reduce, inner, s);
}
void ptx_tensor_reduce_min_f32(float* in, float* out, size_t outer, size_t reduce, size_t inner, cudaStream_t s) {
    run_reduce<RMinF>(in, out, outer, reduce, inner, s);
}
void ptx_tensor_reduce_prod_f32(float* in, float* out, size_t outer, size_t reduce, size_t inner, cudaStream_t s) {
    run_reduce<RProd<float>>(in, out, outer, reduce, inner, s);
}
void ptx_tensor_reduce_sum_f64(double* in, double* out, size_t outer, size_t reduce, size_t inner, cudaStream_t s) {
    run_reduce<RSum<double>>(in, out, outer, reduce, inner, s);
}
void ptx_tensor_reduce_max_f64(double* in, double* out, size_t outer, size_t reduce, size_t inner, cudaStream_t s) {
    run_reduce<RMaxD>(in, out, outer, reduce, inner, s);
}
void ptx_tensor_reduce_min_f64(double* in, double* out, size_t outer, size_t reduce, size_t inner, cudaStream_t s) {
    run_reduce<RMinDRef>(in, out, outer, reduce, inner, s);
}
void ptx_tensor_reduce_argmax_f32(float* in, int32_t* out, size_t outer, size_t reduce, size_t inner, cudaStream_t s) {
    run_arg<true>(in, out, outer, reduce, inner, s);
}
void ptx_tensor_reduce_argmin_f32(float* in, int32_t* out, size_t outer, size_t reduce, size_t inner, cudaStream_t s) {
    run_arg<false>(in, out, outer, reduce, inner, s);
}

// ---- softmax variants (ops_core.inl:809-860, 1050-1110, 1180-1230) ----------------------
void ptx_tensor_log_softmax_f32(float* in, float* out, size_t batch, size_t dim, cudaStream_t s) {
    run_softmax<SM::kLogF32, float, float>(in, out, batch, dim, s);
}
void ptx_tensor_softmax_f64(double* in, double* out, size_t batch, size_t dim, cudaStream_t s) {
    run_softmax<SM::kF64, double, double>(in, out, batch, dim, s);
}
void ptx_tensor_softmax_f16(__half* in, __half* out, size_t batch, size_t dim, cudaStream_t s) {
    run_softmax<SM::kF16, __half, float>(in, out, batch, dim, s);
}

// ---- scan, sort, select (indexing_scan.inl) ---------------------------------------------
void ptx_tensor_cumsum_f32(float* in, float* out, size_t outer, size_t dim, size_t inner, cudaStream_t s) {
    if (outer * inner == 0) return;
    if (inner == 1)
        cumsum_rows<<<persistent_grid((outer + 32 * kScanWarps - 1) / (32 * kScanWarps), 16), kScanWarps * 32, 0,
                      s>>>(in, out, outer, dim);
    else
        cumsum_strided<<<grid_for(outer * inner), kThreads, 0, s>>>(in, out, outer, dim, inner);
}

void ptx_tensor_argsort_f32(float* in, uint32_t* out, size_t nrows, size_t ncols, int ascending, cudaStream_t s) {
    if (nrows == 0 || ncols == 0) return;
    int pad = 1;
    while (pad < static_cast<int>(ncols)) pad <<= 1;
    const size_t smem = static_cast<size_t>(pad) * sizeof(int) + ncols * sizeof(float);
    const int block = pad < 2 ? 1 : (pad / 2 < 512 ? pad / 2 : 512);
    auto kern = ascending ? argsort_rows<true> : argsort_rows<false>;
    if (smem > (48u << 10)) {
        if (smem > (227u << 10) ||
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
                cudaSuccess)
            return;
    }
    kern<<<static_cast<unsigned>(nrows), block, smem, s>>>(in, out, static_cast<int>(ncols), pad);
}

void ptx_tensor_topk_f32(float* in, float* values_out, int32_t* indices_out, size_t outer, size_t dim_size,
                         size_t inner, size_t k, int largest, cudaStream_t s) {
    const size_t cols = outer * inner;
    if (cols == 0 || k == 0 || dim_size == 0) return;
    const size_t smem = ((dim_size + 31) / 32) * sizeof(unsigned int);
    auto kern = largest ? topk_cols<true> : topk_cols<false>;
    if (smem > (48u << 10)) {
        if (smem > (227u << 10) ||
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
                cudaSuccess)
            return;
    }
    kern<<<persistent_grid(cols, 16), 32, smem, s>>>(in, values_out, indices_out, outer, dim_size, inner, k);
}

void ptx_tensor_gather_f32(float* in, int32_t* indices, float* out, size_t outer, size_t input_dim_size,
                           size_t idx_dim_size, size_t inner, cudaStream_t s) {
    const size_t total = outer * idx_dim_size * inner;
    if (total && input_dim_size) gather_kernel<<<grid_for(total), kThreads, 0, s>>>(in, indices, out, outer, input_dim_size,
                                                                  idx_dim_size, inner);
}

void ptx_tensor_index_select_f32(float* in, int32_t* ids, float* out, size_t left_size, size_t src_dim_size,
                                 size_t ids_dim_size, size_t right_size, cudaStream_t s) {
    const size_t total = left_size * ids_dim_size * right_size;
    if (total && src_dim_size) index_select_kernel<<<grid_for(total), kThreads, 0, s>>>(in, ids, out, left_size, src_dim_size,
                                                                        ids_dim_size, right_size);
}

void ptx_tensor_scatter_add_f32(int32_t* ids, float* src, float* out, size_t left_size, size_t src_dim_size,
                                size_t dst_dim_size, size_t right_size, cudaStream_t s) {
    const size_t total = left_size * src_dim_size * right_size;
    if (total == 0) return;
    const size_t cols = left_size * right_size;
    if (cols >= 1024)
        scatter_add_cols<<<grid_for(cols), kThreads, 0, s>>>(ids, src, out, left_size, src_dim_size, dst_dim_size,
                                                             right_size);
    else
        scatter_add_atomic<<<grid_for(total), kThreads, 0, s>>>(ids, src, out, left_size, src_dim_size,
                                                                dst_dim_size, right_size);
}

// ---- opcode dispatch (util_dispatch.inl:200-606) ------------------------------------------
cudaError_t ptx_tensor_dispatch(const PTXTensorOp* op) {
    if (!op) return cudaErrorInvalidValue;
    cudaStream_t s = op->stream;
    void* a = op->input_a;
    void* b = op->input_b;
    void* o = op->output;
    const size_t n = op->elem_count;
    const bool f32 = op->dtype == PTX_DTYPE_F32, f64 = op->dtype == PTX_DTYPE_F64, f16 = op->dtype == PTX_DTYPE_F16;
    auto F = [](void* p) { return static_cast<float*>(p); };
    auto D = [](void* p) { return static_cast<double*>(p); };
    auto H = [](void* p) { return static_cast<__half*>(p); };
    auto U8 = [](void* p) { return static_cast<uint8_t*>(p); };
    auto I32 = [](void* p) { return static_cast<int32_t*>(p); };
    const size_t outer = op->outer_size, red = op->reduce_size, inner = op->inner_size;
    switch (op->opcode) {
#define BIN3(OPC, FF, DD, HH)                      \
    case OPC:                                      \
        if (f32) FF(F(a), F(b), F(o), n, s);       \
        else if (f64) DD(D(a), D(b), D(o), n, s);  \
        else if (f16) HH(H(a), H(b), H(o), n, s);  \
        break;
        BIN3(PTX_OP_ADD, ptx_tensor_add_f32, ptx_tensor_add_f64, ptx_tensor_add_f16)
        BIN3(PTX_OP_SUB, ptx_tensor_sub_f32, ptx_tensor_sub_f64, ptx_tensor_sub_f16)
        BIN3(PTX_OP_MUL, ptx_tensor_mul_f32, ptx_tensor_mul_f64, ptx_tensor_mul_f16)
        BIN3(PTX_OP_DIV, ptx_tensor_div_f32, ptx_tensor_div_f64, ptx_tensor_div_f16)
#undef BIN3
#define UN2(OPC, FF, DD)                      \
    case OPC:                                 \
        if (f32) FF(F(a), F(o), n, s);        \
        else if (f64) DD(D(a), D(o), n, s);   \
        break;
        UN2(PTX_OP_NEG, ptx_tensor_neg_f32, ptx_tensor_neg_f64)
        UN2(PTX_OP_EXP, ptx_tensor_exp_f32, ptx_tensor_exp_f64)
        UN2(PTX_OP_LOG, ptx_tensor_log_f32, ptx_tensor_log_f64)
        UN2(PTX_OP_SQRT, ptx_tensor_sqrt_f32, ptx_tensor_sqrt_f64)
        UN2(PTX_OP_TANH, ptx_tensor_tanh_f32, ptx_tensor_tanh_f64)
#undef UN2
#define UN1(OPC, FF)                   \
    case OPC:                          \
        if (f32) FF(F(a), F(o), n, s); \
        break;
        UN1(PTX_OP_SIN, ptx_tensor_sin_f32)
        UN1(PTX_OP_COS, ptx_tensor_cos_f32)
        UN1(PTX_OP_ABS, ptx_tensor_abs_f32)
        UN1(PTX_OP_SQR, ptx_tensor_sqr_f32)
        UN1(PTX_OP_RECIP, ptx_tensor_recip_f32)
        UN1(PTX_OP_CEIL, ptx_tensor_ceil_f32)
        UN1(PTX_OP_FLOOR, ptx_tensor_floor_f32)
        UN1(PTX_OP_ROUND, ptx_tensor_round_f32)
        UN1(PTX_OP_SIGN, ptx_tensor_sign_f32)
        UN1(PTX_OP_LOG2, ptx_tensor_log2_f32)
        UN1(PTX_OP_LOG10, ptx_tensor_log10_f32)
        UN1(PTX_OP_TAN, ptx_tensor_tan_f32)
        UN1(PTX_OP_SINH, ptx_tensor_sinh_f32)
        UN1(PTX_OP_COSH, ptx_tensor_cosh_f32)
        UN1(PTX_OP_ERF, ptx_tensor_erf_f32)
        UN1(PTX_OP_SILU, ptx_tensor_silu_f32)
        UN1(PTX_OP_SELU, ptx_tensor_selu_f32)
        UN1(PTX_OP_SOFTPLUS, ptx_tensor_softplus_f32)
        UN1(PTX_OP_MISH, ptx_tensor_mish_f32)
        UN1(PTX_OP_GELU_TANH, ptx_tensor_gelu_tanh_f32)
        UN1(PTX_OP_HARDSWISH, ptx_tensor_hardswish_f32)
        UN1(PTX_OP_HARDSIGMOID, ptx_tensor_hardsigmoid_f32)
        UN1(PTX_OP_COPY, ptx_tensor_copy_f32)
#undef UN1
        case PTX_OP_MOD:
            if (f32) ptx_tensor_mod_f32(F(a), F(b), F(o), n, s);
            break;
#define ACT3(OPC, FF, DD, HH)                 \
    case OPC:                                 \
        if (f32) FF(F(a), F(o), n, s);        \
        else if (f64) DD(D(a), D(o), n, s);   \
        else if (f16) HH(H(a), H(o), n, s);   \
        break;
        ACT3(PTX_OP_RELU, ptx_tensor_relu_f32, ptx_tensor_relu_f64, ptx_tensor_relu_f16)
        ACT3(PTX_OP_GELU, ptx_tensor_gelu_f32, ptx_tensor_gelu_f64, ptx_tensor_gelu_f16)
        ACT3(PTX_OP_SIGMOID, ptx_tensor_sigmoid_f32, ptx_tensor_sigmoid_f64, ptx_tensor_sigmoid_f16)
#undef ACT3
        case PTX_OP_ELU:
            if (f32) ptx_tensor_elu_f32(F(a), F(o), n, op->scalar_a, s);
            break;
        case PTX_OP_LEAKY_RELU:
            if (f32) ptx_tensor_leaky_relu_f32(F(a), F(o), n, op->scalar_a, s);
            break;
        case PTX_OP_REDUCE_SUM:
            if (f32) ptx_tensor_reduce_sum_f32(F(a), F(o), outer, red, inner, s);
            else if (f64) ptx_tensor_reduce_sum_f64(D(a), D(o), outer, red, inner, s);
            break;
        case PTX_OP_REDUCE_MEAN:
            if (f32) ptx_tensor_reduce_mean_f32(F(a), F(o), outer, red, inner, s);
            break;
        case PTX_OP_REDUCE_MAX:
            if (f32) ptx_tensor_reduce_max_f32(F(a), F(o), outer, red, inner, s);
            else if (f64) ptx_tensor_reduce_max_f64(D(a), D(o), outer, red, inner, s);
            break;
        case PTX_OP_REDUCE_MIN:
            if (f32) ptx_tensor_reduce_min_f32(F(a), F(o), outer, red, inner, s);
            else if (f64) ptx_tensor_reduce_min_f64(D(a), D(o), outer, red, inner, s);
            break;
        case PTX_OP_REDUCE_PROD:
            if (f32) ptx_tensor_reduce_prod_f32(F(a), F(o), outer, red, inner, s);
            break;
        case PTX_OP_REDUCE_ARGMAX:
            if (f32) ptx_tensor_reduce_argmax_f32(F(a), I32(o), outer, red, inner, s);
            break;
        case PTX_OP_REDUCE_ARGMIN:
            if (f32) ptx_tensor_reduce_argmin_f32(F(a), I32(o), outer, red, inner, s);
            break;
        case PTX_OP_SOFTMAX:
            if (f32) ptx_tensor_softmax_f32(F(a), F(o), outer, red, s);
            else if (f64) ptx_tensor_softmax_f64(D(a), D(o), outer, red, s);
            else if (f16) ptx_tensor_softmax_f16(H(a), H(o), outer, red, s);
            break;
        case PTX_OP_LOG_SOFTMAX:
            if (f32) ptx_tensor_log_softmax_f32(F(a), F(o), outer, red, s);
            break;
        case PTX_OP_AFFINE:
            if (f32) ptx_tensor_affine_f32(F(a), F(o), n, op->scalar_a, op->scalar_b, s);
            else if (f64)
                ptx_tensor_affine_f64(D(a), D(o), n, static_cast<double>(op->scalar_a),
                                      static_cast<double>(op->scalar_b), s);
            break;
        case PTX_OP_CLAMP:
            if (f32) ptx_tensor_clamp_f32(F(a), F(o), n, op->scalar_a, op->scalar_b, s);
            break;
        case PTX_OP_POW:
            if (f32) ptx_tensor_powf_f32(F(a), F(o), n, op->scalar_a, s);
            break;
#define CMPD(OPC, FF)                              \
    case OPC:                                      \
        if (f32) FF(F(a), F(b), U8(o), n, s);      \
        break;
        CMPD(PTX_OP_CMP_EQ, ptx_tensor_cmp_eq_f32)
        CMPD(PTX_OP_CMP_NE, ptx_tensor_cmp_ne_f32)
        CMPD(PTX_OP_CMP_LT, ptx_tensor_cmp_lt_f32)
        CMPD(PTX_OP_CMP_LE, ptx_tensor_cmp_le_f32)
        CMPD(PTX_OP_CMP_GT, ptx_tensor_cmp_gt_f32)
        CMPD(PTX_OP_CMP_GE, ptx_tensor_cmp_ge_f32)
#undef CMPD
        case PTX_OP_WHERE:
            // out = cond ? input_b : out (the reference passes the output as
            // both the false branch and the destination)
            if (f32) ptx_tensor_where_f32(U8(a), F(b), F(o), F(o), n, s);
            break;
        case PTX_OP_FILL:
            if (f32) ptx_tensor_fill_f32(F(o), n, op->scalar_a, s);
            break;
        case PTX_OP_GATHER:
            // outer, input dim (reduce_size), index dim (inner_size), inner (elem_count)
            if (f32) ptx_tensor_gather_f32(F(a), I32(b), F(o), outer, red, inner, n, s);
            break;
        case PTX_OP_CUMSUM:
            if (f32) ptx_tensor_cumsum_f32(F(a), F(o), outer, red, inner, s);
            break;
        case PTX_OP_TOPK:
            // k = elem_count, largest = scalar_a > 0.5, indices to input_b
            if (f32) ptx_tensor_topk_f32(F(a), F(o), I32(b), outer, red, inner, n, op->scalar_a > 0.5f ? 1 : 0, s);
            break;
        case PTX_OP_INDEX_SELECT:
            if (f32) ptx_tensor_index_select_f32(F(a), I32(b), F(o), outer, red, inner, n, s);
            break;
        case PTX_OP_SCATTER_ADD:
            if (f32) ptx_tensor_scatter_add_f32(I32(b), F(a), F(o), outer, red, inner, n, s);
            break;
        case PTX_OP_ARGSORT:
            if (f32)
                ptx_tensor_argsort_f32(F(a), static_cast<uint32_t*>(o), outer, red, op->scalar_a > 0.5f ? 1 : 0, s);
            break;
        default:
            return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

cudaError_t ptx_tensor_dispatch_sync(const PTXTensorOp* op) {
    const cudaError_t e = ptx_tensor_dispatch(op);
    if (e != cudaSuccess) return e;
    return op->stream ? cudaStreamSynchronize(op->stream) : cudaDeviceSynchronize();
}

}  // extern "C"
