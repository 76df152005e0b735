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
#include "sm100_util.cuh"

#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

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

// Sum of 256 per-thread partials in the order of the reference's
// `for (s = 128; s > 0; s >>= 1) sdata[t] += sdata[t + s]` tree.
__device__ __forceinline__ float halving_sum_256(float p, Scratch& sc, int slot) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    sc.part[threadIdx.x] = p;
    __syncthreads();
    if (wid == 0) {
        const float* q = sc.part;
        // steps s = 128, 64, 32
        float u = ((q[lane] + q[lane + 128]) + (q[lane + 64] + q[lane + 192])) +
                  ((q[lane + 32] + q[lane + 160]) + (q[lane + 96] + q[lane + 224]));
        // steps s = 16 .. 1
        u = warp_down_sum(u);
        if (lane == 0) sc.fin[slot] = u;
    }
    __syncthreads();
    return sc.fin[slot];
}

__device__ __forceinline__ float halving_max_256(float p, Scratch& sc, int slot) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    sc.part[threadIdx.x] = p;
    __syncthreads();
    if (wid == 0) {
        const float* q = sc.part;
        float u = fmaxf(fmaxf(fmaxf(q[lane], q[lane + 128]), fmaxf(q[lane + 64], q[lane + 192])),
                        fmaxf(fmaxf(q[lane + 32], q[lane + 160]), fmaxf(q[lane + 96], q[lane + 224])));
        u = warp_down_max(u);
        if (lane == 0) sc.fin[slot] = u;
    }
    __syncthreads();
    return sc.fin[slot];
}

template <int VPT>
__device__ __forceinline__ void process_row(float (&v)[VPT], const RowsArgs& a, Scratch& sc, int cols) {
    const int t = threadIdx.x;
    if (a.flags & kSoftmax) {
        const bool tree = (a.flags & kSoftmaxTree) != 0;
        float m = tree ? -1e30f : -INFINITY;
#pragma unroll
        for (int j = 0; j < VPT; ++j)
            if (t + kThreads * j < cols) m = fmaxf(m, v[j]);
        const float mx = tree ? halving_max_256(m, sc, 0) : softmax_block_max(m, sc);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < VPT; ++j)
            if (t + kThreads * j < cols) {
                v[j] = expf(v[j] - mx);
                s += v[j];
            }
        const float sum = tree ? halving_sum_256(s, sc, 1) : softmax_block_sum(s, sc);
        const float inv = 1.0f / sum;
#pragma unroll
        for (int j = 0; j < VPT; ++j) v[j] *= inv;
    }
    if (a.flags & kLayerNorm) {
        const float n = static_cast<float>(cols);
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < VPT; ++j)
            if (t + kThreads * j < cols) s += v[j];
        const float mean = halving_sum_256(s, sc, 2) / n;
        float q = 0.0f;
#pragma unroll
        for (int j = 0; j < VPT; ++j)
            if (t + kThreads * j < cols) {
                const float d = v[j] - mean;
                q += d * d;
            }
        const float var = halving_sum_256(q, sc, 3) / n;
        const float inv_std = rsqrtf(var + a.eps);
#pragma unroll
        for (int j = 0; j < VPT; ++j) v[j] = (v[j] - mean) * inv_std;
        if (a.gamma || a.beta) {
#pragma unroll
            for (int j = 0; j < VPT; ++j) {
                const int c = t + kThreads * j;
                if (c < cols) {
                    if (a.gamma) v[j] = v[j] * a.gamma[c];
                    if (a.beta) v[j] = v[j] + a.beta[c];
                }
            }
        }
    }
}

// Persistent bulk-copy kernel. Requires 256 <= cols <= 256*VPT, cols % 4 == 0,
// x 16-byte aligned, dynamic shared memory = stages * cols * 4 bytes.
template <int VPT>
__global__ void __launch_bounds__(kThreads) rows_bulk_kernel(RowsArgs a) {
    extern __shared__ __align__(128) float ring[];
    __shared__ __align__(8) uint64_t full[kMaxStages];
    __shared__ Scratch sc;
    __shared__ int abort_flag;

    const int t = threadIdx.x;
    const int cols = a.cols;
    const uint32_t row_bytes = static_cast<uint32_t>(cols) * 4u;
    const int stages = a.stages;
    const int my_rows = (blockIdx.x < static_cast<unsigned>(a.rows))
                            ? (a.rows - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                            : 0;
    if (t == 0) {
        abort_flag = 0;
        for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (t == 0) {
        const int pre = my_rows < stages ? my_rows : stages;
        for (int i = 0; i < pre; ++i) {
            const size_t r = blockIdx.x + static_cast<size_t>(i) * gridDim.x;
            mbar_arrive_expect_tx(&full[i], row_bytes);
            bulk_g2s(ring + static_cast<size_t>(i) * cols, a.x + r * cols, row_bytes, &full[i]);
        }
    }
    for (int i = 0; i < my_rows; ++i) {
        const int s = i % stages;
        const uint32_t parity = static_cast<uint32_t>(i / stages) & 1u;
        const size_t r = blockIdx.x + static_cast<size_t>(i) * gridDim.x;
        if (!mbar_wait(&full[s], parity)) abort_flag = 1;
        __syncthreads();
        if (abort_flag) {
            if (t == 0) report(a.err, kErrTimeoutLoad);
            return;
        }
        float v[VPT];
        const float* buf = ring + static_cast<size_t>(s) * cols;
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
            const int c = t + kThreads * j;
            v[j] = c < cols ? buf[c] : 0.0f;
        }
        // Every thread has read buffer s once it reaches this barrier; the
        // refill is issued behind it.
        __syncthreads();
        if (t == 0 && i + stages < my_rows) {
            fence_proxy_async_smem();
            const size_t rn = r + static_cast<size_t>(stages) * gridDim.x;
            mbar_arrive_expect_tx(&full[s], row_bytes);
            bulk_g2s(ring + static_cast<size_t>(s) * cols, a.x + rn * cols, row_bytes, &full[s]);
        }
        process_row<VPT>(v, a, sc, cols);
        float* out = a.y + r * cols;
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
            const int c = t + kThreads * j;
            if (c < cols) st_global_cs(out + c, v[j]);
        }
    }
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

int g_num_sms = 0;

int num_sms() {
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

template <int VPT>
cudaError_t launch_bulk(RowsArgs a, cudaStream_t stream) {
    const size_t row_bytes = static_cast<size_t>(a.cols) * 4;
    // Ring: as many row buffers as fit in 48 KiB (2..8), so three or more
    // CTAs share an SM and keep >100 KiB of reads in flight per SM.
    int stages = static_cast<int>((48u << 10) / row_bytes);
    if (stages < 2) stages = 2;
    if (stages > kMaxStages) stages = kMaxStages;
    a.stages = stages;
    const size_t smem = row_bytes * stages;
    cudaError_t e = cudaFuncSetAttribute(rows_bulk_kernel<VPT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, rows_bulk_kernel<VPT>, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) per_sm = 1;
    int grid = num_sms() * per_sm;
    if (grid > a.rows) grid = a.rows;
    rows_bulk_kernel<VPT><<<grid, kThreads, smem, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace

// Host launcher shared by the native ABI and the session layer.
// flags: 1 = softmax, 2 = layer norm, 3 = softmax then layer norm.
extern "C" cudaError_t fer_rows_f32(const float* x, float* y, const float* gamma, const float* beta, int rows,
                                    int cols, float eps, uint32_t flags, uint32_t* err, cudaStream_t stream) {
    if (rows <= 0 || cols <= 0) return cudaSuccess;
    RowsArgs a{x, y, gamma, beta, rows, cols, eps, flags, 2, err};
    const bool bulk_ok = cols >= kThreads && cols <= 64 * kThreads && (cols % 4) == 0 &&
                         (reinterpret_cast<uintptr_t>(x) % 16) == 0 && x != y;
    if (bulk_ok) {
        const int vpt = (cols + kThreads - 1) / kThreads;
        if (vpt <= 2) return launch_bulk<2>(a, stream);
        if (vpt <= 4) return launch_bulk<4>(a, stream);
        if (vpt <= 8) return launch_bulk<8>(a, stream);
        if (vpt <= 16) return launch_bulk<16>(a, stream);
        if (vpt <= 32) return launch_bulk<32>(a, stream);
        return launch_bulk<64>(a, stream);
    }
    int grid = rows < num_sms() * 8 ? rows : num_sms() * 8;
    rows_generic_kernel<<<grid, kThreads, 0, stream>>>(a);
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
