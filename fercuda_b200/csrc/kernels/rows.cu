// Row kernels: softmax, layer norm, and softmax followed by layer norm, f32.
//
// Numerics follow the reference kernels operation for operation, so results
// are bit-identical to them on the same GPU:
//   softmax    k_softmax_f32   native/core/kernels/modules/tensor_kernels_ops_core.inl:733-808
//              (256 threads; thread t owns elements t, t+256, ...; warp
//              __shfl_down trees, then warp 0 over the 8 warp results)
//   layer norm k_layer_norm_f32 src/runtime/ops_bridge.cu:33-59
//              (T = min(cols, 256) threads, strided per-thread sums, shared
//              halving tree, mean = sum/n, rsqrtf(var/n + eps))
// Both were built by the reference with -fmad=false; so is this file.
//
// Data movement is B200-first instead of the reference's one-CTA-per-row,
// three-reads-two-writes pattern:
//   - persistent CTAs, rows assigned round-robin, each row read once from HBM
//     by a 1-D bulk copy (cp.async.bulk, TMA engine) into a shared-memory ring
//     of `stages` row buffers guarded by mbarriers, so the next rows stream in
//     while the current one is reduced;
//   - every value lives in registers from the shared-memory read to the
//     store; softmax and layer norm fuse into one pass (8 bytes of HBM
//     traffic per element instead of 8 per element per kernel);
//   - the reference's 8-step shared halving tree is evaluated as one shared
//     read of the 256 partials by warp 0 in the same association order,
//     followed by the matching __shfl_down tree.
// Shapes the bulk-copy path cannot take (cols < 256, cols % 4 != 0, a
// misaligned base, cols > 16384) run a multi-pass kernel with the same
// arithmetic.
#include "elem.cuh"
#include "f32x2.cuh"
#include "pdl.cuh"
#include "sm100_util.cuh"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <mutex>

namespace {

using namespace fer::dev;

constexpr int kThreads = 256;
constexpr int kMaxStages = 8;

// kSoftmaxTree: softmax reduced with the shared halving tree of the
// reference's JIT softmax intent (intent_runtime.cpp:72-118: max starts at
// -1e30f, both reductions `for (s = T/2; s > 0; s >>= 1)`), instead of the
// warp-shuffle order of the native k_softmax_f32.
enum : uint32_t { kSoftmax = 1u, kLayerNorm = 2u, kSoftmaxTree = 4u };

struct RowsArgs {
    const float* x;
    float* y;
    const float* gamma;  // optional, [cols]
    const float* beta;   // optional, [cols]
    int rows;
    int cols;
    float eps;
    uint32_t flags;
    int stages;
    uint32_t* err;
    // Bulk kernel only: work before the programmatic launch wait (cleared by
    // the host against the kernel just before on the stream): 0 none, 1 the
    // first ring fill, 2 everything (the wait then only orders completion).
    uint32_t early;
};

__device__ __forceinline__ float warp_down_max(float v) {
    for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_down_sync(0xffffffffu, v, off));
    return v;
}

__device__ __forceinline__ float warp_down_sum(float v) {
    for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
    return v;
}

struct Scratch {
    float warp_max[8];
    float warp_sum[8];
    float part[kThreads];
    float fin[4];
};

// Shared slots for the single-barrier reductions of the bulk kernel: each
// reduction of a row has its own slots, and every warp finishes the
// reduction itself from them (same association order as the reference, so
// the same bits), which needs one barrier per reduction instead of two. A
// slot is rewritten only three barriers after its last read.
struct RowSlots {
    float warp_max[8];
    float warp_sum[8];
    float ln_sum[kThreads];
    float ln_var[kThreads];
};

// Block max / sum in the k_softmax_f32 order. All 256 threads call it.
__device__ __forceinline__ float softmax_block_max(float m, Scratch& sc) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    m = warp_down_max(m);
    if (lane == 0) sc.warp_max[wid] = m;
    __syncthreads();
    if (wid == 0) {
        float w = lane < 8 ? sc.warp_max[lane] : -INFINITY;
        w = warp_down_max(w);
        if (lane == 0) sc.fin[0] = w;
    }
    __syncthreads();
    return sc.fin[0];
}

__device__ __forceinline__ float softmax_block_sum(float s, Scratch& sc) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    s = warp_down_sum(s);
    if (lane == 0) sc.warp_sum[wid] = s;
    __syncthreads();
    if (wid == 0) {
        float w = lane < 8 ? sc.warp_sum[lane] : 0.0f;
        w = warp_down_sum(w);
        if (lane == 0) sc.fin[1] = w;
    }
    __syncthreads();
    return sc.fin[1];
}

// --- single-barrier variants (every warp finishes the reduction) -----------

// Warp maximum in one instruction. max is exact and order-independent
// (a NaN operand yields the other operand, as fmaxf does), so this equals
// the reference's __shfl_down / fmaxf tree bit for bit.
__device__ __forceinline__ float warp_max_redux(float v) {
    float r;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
    return r;
}

// k_softmax_f32 order: warp tree, then a tree over the 8 warp results padded
// to 32 lanes. `abort_in` joins the barrier as a vote (__syncthreads_or).
__device__ __forceinline__ float sb_softmax_max(float m, float* slot8, int abort_in, int* abort_out) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    m = warp_max_redux(m);
    if (lane == 0) slot8[wid] = m;
    *abort_out = __syncthreads_or(abort_in);
    return warp_max_redux(lane < 8 ? slot8[lane] : -INFINITY);
}

__device__ __forceinline__ float sb_softmax_sum(float s, float* slot8) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    s = warp_down_sum(s);
    if (lane == 0) slot8[wid] = s;
    __syncthreads();
    float w = lane < 8 ? slot8[lane] : 0.0f;
    return __shfl_sync(0xffffffffu, warp_down_sum(w), 0);
}

// Sum of 256 per-thread partials in the order of the reference's
// `for (s = 128; s > 0; s >>= 1) sdata[t] += sdata[t + s]` tree: steps
// s = 128, 64, 32 as one expression per lane, then s = 16 .. 1 as the
// __shfl_down tree.
__device__ __forceinline__ float sb_halving_sum(float p, float* slot256, int abort_in, int* abort_out) {
    const int lane = threadIdx.x & 31;
    slot256[threadIdx.x] = p;
    *abort_out = __syncthreads_or(abort_in);
    const float* q = slot256;
    float u = ((q[lane] + q[lane + 128]) + (q[lane + 64] + q[lane + 192])) +
              ((q[lane + 32] + q[lane + 160]) + (q[lane + 96] + q[lane + 224]));
    return __shfl_sync(0xffffffffu, warp_down_sum(u), 0);
}

__device__ __forceinline__ float sb_halving_max(float p, float* slot256, int abort_in, int* abort_out) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    // max is order-independent: reduce each warp first, then the 8 results.
    p = warp_max_redux(p);
    if (lane == 0) slot256[wid] = p;
    *abort_out = __syncthreads_or(abort_in);
    return warp_max_redux(lane < 8 ? slot256[lane] : -INFINITY);
}

// One row held in registers (thread t owns columns t + 256 j). The first
// barrier of the row carries the load-timeout vote and is also the point
// after which every thread has finished reading the row's ring buffer; the
// caller's `after_first_barrier` issues the refill there. Returns false if
// any thread reported a timeout.
// FULL: cols == 256 * VPT, so no per-element bounds checks.
template <int VPT, bool FULL, typename Hook>
__device__ __forceinline__ bool process_row_sb(float (&v)[VPT], const RowsArgs& a, RowSlots& sl, int cols,
                                               int timed_out, Hook after_first_barrier) {
    const int t = threadIdx.x;
    int abort_any = 0;
    bool first = true;
    if (a.flags & kSoftmax) {
        const bool tree = (a.flags & kSoftmaxTree) != 0;
        float m = tree ? -1e30f : -INFINITY;
#pragma unroll
        for (int j = 0; j < VPT; ++j)
            if (FULL || t + kThreads * j < cols) m = fmaxf(m, v[j]);
        const float mx = tree ? sb_halving_max(m, sl.ln_var, timed_out, &abort_any)
                              : sb_softmax_max(m, sl.warp_max, timed_out, &abort_any);
        if (abort_any) return false;
        after_first_barrier();
        first = false;
        float s = 0.0f;
        if constexpr (FULL && VPT % 2 == 0) {
            // the subtractions and scalings in packed pairs (same bits)
#pragma unroll
            for (int j = 0; j < VPT; j += 2) {
                f2_unpack(f2_sub(f2_pack(v[j], v[j + 1]), f2_splat(mx)), v[j], v[j + 1]);
                v[j] = expf(v[j]);
                s += v[j];
                v[j + 1] = expf(v[j + 1]);
                s += v[j + 1];
            }
        } else {
#pragma unroll
            for (int j = 0; j < VPT; ++j)
                if (FULL || t + kThreads * j < cols) {
                    v[j] = expf(v[j] - mx);
                    s += v[j];
                }
        }
        int dummy = 0;
        const float sum = tree ? sb_halving_sum(s, sl.ln_sum, 0, &dummy) : sb_softmax_sum(s, sl.warp_sum);
        const float inv = 1.0f / sum;
        if constexpr (VPT % 2 == 0) {
#pragma unroll
            for (int j = 0; j < VPT; j += 2) f2_unpack(f2_mul(f2_pack(v[j], v[j + 1]), f2_splat(inv)), v[j], v[j + 1]);
        } else {
#pragma unroll
            for (int j = 0; j < VPT; ++j) v[j] *= inv;
        }
    }
    if (a.flags & kLayerNorm) {
        const float n = static_cast<float>(cols);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < VPT; ++j)
            if (FULL || t + kThreads * j < cols) s += v[j];
        // With the tree-order softmax the ln_sum / ln_var slots were used by
        // its reductions; the barriers in between keep the reuse safe.
        const float mean = sb_halving_sum(s, (a.flags & kSoftmaxTree) ? sl.ln_var : sl.ln_sum,
                                          first ? timed_out : 0, &abort_any) / n;
        if (first) {
            if (abort_any) return false;
            after_first_barrier();
        }
        float q = 0.0f;
        if constexpr (FULL && VPT % 2 == 0) {
            // v - mean and its square in packed pairs; the sum stays in
            // element order (same bits); v keeps v - mean
#pragma unroll
            for (int j = 0; j < VPT; j += 2) {
                const uint64_t d = f2_sub(f2_pack(v[j], v[j + 1]), f2_splat(mean));
                float d0, d1;
                f2_unpack(f2_mul(d, d), d0, d1);
                q += d0;
                q += d1;
                f2_unpack(d, v[j], v[j + 1]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < VPT; ++j)
                if (FULL || t + kThreads * j < cols) {
                    const float d = v[j] - mean;
                    q += d * d;
                }
        }
        int dummy = 0;
        const float var = sb_halving_sum(q, (a.flags & kSoftmaxTree) ? sl.ln_sum : sl.ln_var, 0, &dummy) / n;
        const float inv_std = rsqrtf(var + a.eps);
        if constexpr (FULL && VPT % 2 == 0) {
#pragma unroll
            for (int j = 0; j < VPT; j += 2)
                f2_unpack(f2_mul(f2_pack(v[j], v[j + 1]), f2_splat(inv_std)), v[j], v[j + 1]);
        } else {
#pragma unroll
            for (int j = 0; j < VPT; ++j) v[j] = (v[j] - mean) * inv_std;
        }
        if (a.gamma || a.beta) {
#pragma unroll
            for (int j = 0; j < VPT; ++j) {
                const int c = t + kThreads * j;
                if (FULL || c < cols) {
                    if (a.gamma) v[j] = v[j] * a.gamma[c];
                    if (a.beta) v[j] = v[j] + a.beta[c];
                }
            }
        }
    }
    return true;
}

// Persistent bulk-copy kernel. Requires 256 <= cols <= 256*VPT, cols % 4 == 0,
// x 16-byte aligned, dynamic shared memory = stages * cols * 4 bytes.
template <int VPT, bool FULL>
__global__ void __launch_bounds__(kThreads) rows_bulk_kernel(RowsArgs a) {
    extern __shared__ __align__(128) float ring[];
    __shared__ __align__(8) uint64_t full[kMaxStages];
    __shared__ RowSlots sl;

    const int t = threadIdx.x;
    const int cols = a.cols;
    const uint32_t row_bytes = static_cast<uint32_t>(cols) * 4u;
    const int stages = a.stages;
    const int my_rows = (blockIdx.x < static_cast<unsigned>(a.rows))
                            ? (a.rows - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                            : 0;
    if (t == 0) {
        for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (a.early == 0) pdl_begin();
    if (t == 0) {
        const int pre = my_rows < stages ? my_rows : stages;
        for (int i = 0; i < pre; ++i) {
            const size_t r = blockIdx.x + static_cast<size_t>(i) * gridDim.x;
            mbar_arrive_expect_tx(&full[i], row_bytes);
            bulk_g2s(ring + static_cast<size_t>(i) * cols, a.x + r * cols, row_bytes, &full[i]);
        }
    }
    if (a.early == 1) pdl_begin();
    for (int i = 0; i < my_rows; ++i) {
        const int s = i % stages;
        const uint32_t parity = static_cast<uint32_t>(i / stages) & 1u;
        const size_t r = blockIdx.x + static_cast<size_t>(i) * gridDim.x;
        const int timed_out = mbar_wait(&full[s], parity) ? 0 : 1;
        float v[VPT];
        const float* buf = ring + static_cast<size_t>(s) * cols;
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
            const int c = t + kThreads * j;
            v[j] = (FULL || c < cols) ? buf[c] : 0.0f;
        }
        // Refill of ring slot s with the row `stages` ahead, issued once every
        // thread is past the row's first barrier (all reads of slot s done).
        auto refill = [&]() {
            if (t == 0 && i + stages < my_rows) {
                fence_proxy_async_smem();
                const size_t rn = r + static_cast<size_t>(stages) * gridDim.x;
                mbar_arrive_expect_tx(&full[s], row_bytes);
                bulk_g2s(ring + static_cast<size_t>(s) * cols, a.x + rn * cols, row_bytes, &full[s]);
            }
        };
        if (!process_row_sb<VPT, FULL>(v, a, sl, cols, timed_out, refill)) {
            if (t == 0) report(a.err, kErrTimeoutLoad);
            return;
        }
        float* out = a.y + r * cols;
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
            const int c = t + kThreads * j;
            if (FULL || c < cols) st_global_cs(out + c, v[j]);
        }
    }
    if (a.early == 2) pdl_begin();   // every thread waits before it exits
}

// Any shape: one CTA per row, values re-read from global memory per pass,
// same arithmetic. The layer-norm tree uses T = min(cols, 256) threads like
// the reference (including its behaviour for T not a power of two).
__global__ void __launch_bounds__(kThreads) rows_generic_kernel(RowsArgs a) {
    __shared__ Scratch sc;
    __shared__ float sdata[kThreads];
    const int t = threadIdx.x;
    const int cols = a.cols;
    for (int r = blockIdx.x; r < a.rows; r += gridDim.x) {
        const float* in = a.x + static_cast<size_t>(r) * cols;
        float* out = a.y + static_cast<size_t>(r) * cols;
        const float* src = in;
        if ((a.flags & kSoftmax) && (a.flags & kSoftmaxTree)) {
            // T = min(cols, 256) threads, shared halving trees.
            const int T = cols < kThreads ? cols : kThreads;
            float m = -1e30f;
            if (t < T)
                for (int c = t; c < cols; c += T) m = fmaxf(m, in[c]);
            sdata[t] = m;
            __syncthreads();
            for (int h = T / 2; h > 0; h >>= 1) {
                if (t < h) sdata[t] = fmaxf(sdata[t], sdata[t + h]);
                __syncthreads();
            }
            const float mx = sdata[0];
            __syncthreads();
            float s = 0.0f;
            if (t < T)
                for (int c = t; c < cols; c += T) {
                    const float e = expf(in[c] - mx);
                    out[c] = e;
                    s += e;
                }
            sdata[t] = s;
            __syncthreads();
            for (int h = T / 2; h > 0; h >>= 1) {
                if (t < h) sdata[t] += sdata[t + h];
                __syncthreads();
            }
            const float inv = 1.0f / sdata[0];
            __syncthreads();
            if (t < T)
                for (int c = t; c < cols; c += T) out[c] *= inv;
            src = out;
            __syncthreads();
        } else if (a.flags & kSoftmax) {
            float m = -INFINITY;
            for (int c = t; c < cols; c += kThreads) m = fmaxf(m, in[c]);
            const float mx = softmax_block_max(m, sc);
            float s = 0.0f;
            for (int c = t; c < cols; c += kThreads) {
                const float e = expf(in[c] - mx);
                out[c] = e;
                s += e;
            }
            const float sum = softmax_block_sum(s, sc);
            const float inv = 1.0f / sum;
            for (int c = t; c < cols; c += kThreads) out[c] *= inv;
            src = out;
            __syncthreads();
        }
        if (a.flags & kLayerNorm) {
            const int T = cols < kThreads ? cols : kThreads;
            const float n = static_cast<float>(cols);
            float s = 0.0f;
            if (t < T)
                for (int c = t; c < cols; c += T) s += src[c];
            sdata[t] = s;
            __syncthreads();
            for (int h = T / 2; h > 0; h >>= 1) {
                if (t < h) sdata[t] += sdata[t + h];
                __syncthreads();
            }
            const float mean = sdata[0] / n;
            __syncthreads();
            float q = 0.0f;
            if (t < T)
                for (int c = t; c < cols; c += T) {
                    const float d = src[c] - mean;
                    q += d * d;
                }
            sdata[t] = q;
            __syncthreads();
            for (int h = T / 2; h > 0; h >>= 1) {
                if (t < h) sdata[t] += sdata[t + h];
                __syncthreads();
            }
            const float inv_std = rsqrtf(sdata[0] / n + a.eps);
            __syncthreads();
            if (t < T)
                for (int c = t; c < cols; c += T) {
                    float v = (src[c] - mean) * inv_std;
                    if (a.gamma) v = v * a.gamma[c];
                    if (a.beta) v = v + a.beta[c];
                    out[c] = v;
                }
            __syncthreads();
        }
    }
}

// Layer norm of f16 / bf16 / i8 / u8 rows, one CTA per row: each value is
// widened to f32 on load, normalised with the arithmetic of the layer-norm
// pass above (the reference's k_layer_norm_f32 order), and rounded back with
// the reference's cast. That is what the reference computes through f32
// temporaries (exec_planner.cu:304-387: cast, normalise, cast back), bit for
// bit, in one launch and without the temporaries. In place (x == y) is
// allowed: a row is written only after its last read.
template <uint32_t DT>
__global__ void __launch_bounds__(kThreads) ln_typed_kernel(const typename Elem<DT>::T* x, typename Elem<DT>::T* y,
                                                            int rows, int cols, float eps) {
    __shared__ float sdata[kThreads];
    const int t = threadIdx.x;
    const int T = cols < kThreads ? cols : kThreads;
    const float n = static_cast<float>(cols);
    for (int r = blockIdx.x; r < rows; r += gridDim.x) {
        const size_t base = static_cast<size_t>(r) * cols;
        float s = 0.0f;
        if (t < T)
            for (int c = t; c < cols; c += T) s += Elem<DT>::load(x, base + c);
        sdata[t] = s;
        __syncthreads();
        for (int h = T / 2; h > 0; h >>= 1) {
            if (t < h) sdata[t] += sdata[t + h];
            __syncthreads();
        }
        const float mean = sdata[0] / n;
        __syncthreads();
        float q = 0.0f;
        if (t < T)
            for (int c = t; c < cols; c += T) {
                const float d = Elem<DT>::load(x, base + c) - mean;
                q += d * d;
            }
        sdata[t] = q;
        __syncthreads();
        for (int h = T / 2; h > 0; h >>= 1) {
            if (t < h) sdata[t] += sdata[t + h];
            __syncthreads();
        }
        const float inv_std = rsqrtf(sdata[0] / n + eps);
        __syncthreads();
        if (t < T)
            for (int c = t; c < cols; c += T)
                Elem<DT>::store(y, base + c, (Elem<DT>::load(x, base + c) - mean) * inv_std);
    }
}

int num_sms() {
    static const int n = [] {
        int dev = 0, v = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v > 0 ? v : 148;
    }();
    return n;
}

// The bulk kernel triggers its dependents, so every launch is counted; with
// `pdl` it is launched with the programmatic-serialization attribute.
template <int VPT, bool FULL>
cudaError_t go_bulk(const RowsArgs& a, int grid, size_t smem, bool pdl, cudaStream_t stream) {
    if (pdl) {
        const cudaError_t e = fer::host::launch_pdl(rows_bulk_kernel<VPT, FULL>, dim3(grid), dim3(kThreads), smem, stream, a);
        return e != cudaSuccess ? e : cudaGetLastError();
    }
    fer_pdl_note_launch();
    rows_bulk_kernel<VPT, FULL><<<grid, kThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

template <int VPT, bool FULL>
cudaError_t launch_bulk(RowsArgs a, bool pdl, cudaStream_t stream) {
    const size_t row_bytes = static_cast<size_t>(a.cols) * 4;
    // Ring depth: the deepest ring among those that keep the most CTAs
    // resident per SM (2..8 row buffers). FERCUDA_ROWS_STAGES overrides it.
    static const int override_stages = [] {
        const char* e = std::getenv("FERCUDA_ROWS_STAGES");
        return e ? std::atoi(e) : 0;
    }();
    // Decision cache per (device, cols) for this instantiation.
    struct Choice { int dev, cols, stages, per_sm; };
    static Choice cache[8] = {};
    static int cache_n = 0;
    static std::mutex cache_mu;
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lk(cache_mu);
        for (int k = 0; k < cache_n; ++k)
            if (cache[k].dev == dev && cache[k].cols == a.cols) {
                a.stages = cache[k].stages;
                int grid = num_sms() * cache[k].per_sm;
                if (grid > a.rows) grid = a.rows;
                return go_bulk<VPT, FULL>(a, grid, row_bytes * a.stages, pdl, stream);
            }
    }
    // The attribute is only an upper bound; occupancy follows the smem each
    // launch passes, so it is set once to the largest ring used.
    cudaError_t e = cudaFuncSetAttribute(rows_bulk_kernel<VPT, FULL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(200u << 10));
    if (e != cudaSuccess) return e;
    int best_stages = 2, best_per_sm = 0;
    for (int st = kMaxStages; st >= 2; --st) {
        if (override_stages >= 2 && st != override_stages) continue;
        const size_t smem = row_bytes * st;
        if (smem > (200u << 10)) continue;
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rows_bulk_kernel<VPT, FULL>, kThreads, smem);
        if (e != cudaSuccess) return e;
        if (per_sm > best_per_sm) {
            best_per_sm = per_sm;
            best_stages = st;
        }
    }
    if (best_per_sm < 1) best_per_sm = 1;
    a.stages = best_stages;
    const size_t smem = row_bytes * best_stages;
    {
        std::lock_guard<std::mutex> lk(cache_mu);
        if (cache_n < 8) cache[cache_n++] = Choice{dev, a.cols, best_stages, best_per_sm};
    }
    int grid = num_sms() * best_per_sm;
    if (grid > a.rows) grid = a.rows;
    return go_bulk<VPT, FULL>(a, grid, smem, pdl, stream);
}

cudaError_t rows_launch(const float* x, float* y, const float* gamma, const float* beta, int rows, int cols, float eps,
                        uint32_t flags, uint32_t early, bool pdl, uint32_t* err, cudaStream_t stream) {
    if (rows <= 0 || cols <= 0) return cudaSuccess;
    if (early > 2) return cudaErrorInvalidValue;
    RowsArgs a{x, y, gamma, beta, rows, cols, eps, flags, 2, err, pdl ? early : 0u};
    const bool bulk_ok = cols >= kThreads && cols <= 64 * kThreads && (cols % 4) == 0 &&
                         (reinterpret_cast<uintptr_t>(x) % 16) == 0 && x != y;
    if (bulk_ok) {
        const int vpt = (cols + kThreads - 1) / kThreads;
        const bool full = cols % kThreads == 0;
        if (full) {
            switch (vpt) {
                case 1: return launch_bulk<1, true>(a, pdl, stream);
                case 2: return launch_bulk<2, true>(a, pdl, stream);
                case 4: return launch_bulk<4, true>(a, pdl, stream);
                case 8: return launch_bulk<8, true>(a, pdl, stream);
                case 16: return launch_bulk<16, true>(a, pdl, stream);
                case 32: return launch_bulk<32, true>(a, pdl, stream);
                case 64: return launch_bulk<64, true>(a, pdl, stream);
                default: break;
            }
        }
        if (vpt <= 2) return launch_bulk<2, false>(a, pdl, stream);
        if (vpt <= 4) return launch_bulk<4, false>(a, pdl, stream);
        if (vpt <= 8) return launch_bulk<8, false>(a, pdl, stream);
        if (vpt <= 16) return launch_bulk<16, false>(a, pdl, stream);
        if (vpt <= 32) return launch_bulk<32, false>(a, pdl, stream);
        return launch_bulk<64, false>(a, pdl, stream);
    }
    // any other shape: the multi-pass kernel, plain launch, never triggers
    int grid = rows < num_sms() * 8 ? rows : num_sms() * 8;
    rows_generic_kernel<<<grid, kThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace

// Host launcher shared by the native ABI and the session layer.
// flags: 1 = softmax, 2 = layer norm, 3 = softmax then layer norm.
extern "C" cudaError_t fer_rows_f32(const float* x, float* y, const float* gamma, const float* beta, int rows,
                                    int cols, float eps, uint32_t flags, uint32_t* err, cudaStream_t stream) {
    return rows_launch(x, y, gamma, beta, rows, cols, eps, flags, 0, false, err, stream);
}

// The same with programmatic dependent launch where the bulk kernel applies;
// `early` as fer_rows_fast_f32_pdl (1: the first ring fill, 2: the whole
// kernel before the wait; the caller's promise about the kernel before).
extern "C" cudaError_t fer_rows_f32_pdl(const float* x, float* y, const float* gamma, const float* beta, int rows,
                                        int cols, float eps, uint32_t flags, uint32_t early, uint32_t* err,
                                        cudaStream_t stream) {
    return rows_launch(x, y, gamma, beta, rows, cols, eps, flags, early, true, err, stream);
}

// Layer norm of each row of a [rows, cols] buffer of dtype `dtype`
// (fer_buffer_dtype_t: 0 f32, 1 f16, 2 bf16, 3 i8, 4 u8), no affine.
extern "C" cudaError_t fer_layer_norm_typed(const void* x, void* y, int rows, int cols, float eps, uint32_t dtype,
                                            uint32_t* err, cudaStream_t stream) {
    if (rows <= 0 || cols <= 0) return cudaSuccess;
    if (dtype == kF32)
        return fer_rows_f32(static_cast<const float*>(x), static_cast<float*>(y), nullptr, nullptr, rows, cols, eps,
                            kLayerNorm, err, stream);
    const int grid = rows < num_sms() * 8 ? rows : num_sms() * 8;
    switch (dtype) {
        case kF16:
            ln_typed_kernel<kF16><<<grid, kThreads, 0, stream>>>(static_cast<const __half*>(x),
                                                                 static_cast<__half*>(y), rows, cols, eps);
            break;
        case kBF16:
            ln_typed_kernel<kBF16><<<grid, kThreads, 0, stream>>>(static_cast<const __nv_bfloat16*>(x),
                                                                  static_cast<__nv_bfloat16*>(y), rows, cols, eps);
            break;
        case kI8:
            ln_typed_kernel<kI8><<<grid, kThreads, 0, stream>>>(static_cast<const int8_t*>(x),
                                                                static_cast<int8_t*>(y), rows, cols, eps);
            break;
        case kU8:
            ln_typed_kernel<kU8><<<grid, kThreads, 0, stream>>>(static_cast<const uint8_t*>(x),
                                                                static_cast<uint8_t*>(y), rows, cols, eps);
            break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// ---- native ABI: reference-compatible launcher -------------------------------
// ptx_tensor_softmax_f32, reference tensor_kernels_indexing_scan.inl:391-394.
extern "C" void ptx_tensor_softmax_f32(float* in, float* out, size_t batch, size_t dim, cudaStream_t stream) {
    fer_rows_f32(in, out, nullptr, nullptr, static_cast<int>(batch), static_cast<int>(dim), 0.0f, kSoftmax,
                 nullptr, stream);
}

// Additive: fused row softmax -> layer norm (optional gamma/beta, may be null).
extern "C" void ptx_tensor_softmax_layer_norm_f32(float* in, float* out, const float* gamma, const float* beta,
                                                  size_t rows, size_t cols, float eps, cudaStream_t stream) {
    fer_rows_f32(in, out, gamma, beta, static_cast<int>(rows), static_cast<int>(cols), eps, kSoftmax | kLayerNorm,
                 nullptr, stream);
}

// Additive: row-batched layer norm, each row normalised like a rank-1
// fer_submit_layer_norm of that row.
extern "C" void ptx_tensor_layer_norm_rows_f32(float* in, float* out, const float* gamma, const float* beta,
                                               size_t rows, size_t cols, float eps, cudaStream_t stream) {
    fer_rows_f32(in, out, gamma, beta, static_cast<int>(rows), static_cast<int>(cols), eps, kLayerNorm, nullptr,
                 stream);
}
