// Deterministic bf16 GEMM on the 5th-generation tensor cores (tcgen05).
//
// C[M,N] = A[M,K] . B[K,N], A and B row-major bf16, f32 accumulation in
// tensor memory, C f32 or bf16 (round to nearest even).
//
// Replaces the reference's CUDA-core GEMM for bf16 operands
// (k_matmul_f32, src/runtime/ops_bridge.cu:13-31, reached through the f32
// cast staging of exec_planner.cu:189-302). Each output tile is produced by
// one CTA that walks K in a fixed order; there is no split-K and no atomic,
// so results are bit-identical run to run (they differ from the reference's
// sequential-FMA chain only by summation order).
//
// Structure (one CTA per SM, persistent over 128x256 output tiles):
//   warp 0      TMA producer: A tile [128 x 64] (K-major) and B tile
//               [64 x 256] (N-major, as four 64-column boxes), 128-byte
//               swizzle, into a 4-stage shared-memory ring (48 KiB / stage)
//   warp 1      allocates all 512 tensor-memory columns (two 128x256 f32
//               accumulators) and issues tcgen05.mma (M=128, N=256, K=16)
//               from one thread; tcgen05.commit releases ring slots and
//               hands finished accumulators to the epilogue
//   warps 2..9  epilogue, two warps per 32-lane TMEM quarter (one per
//               128-column half): tcgen05.ld, convert (bf16 / GELU), write a
//               32-row x 128-byte box into a swizzled shared staging buffer,
//               and one lane issues a TMA tensor store of the box (or, for
//               the in-place residual x += A.B, a TMA reduce-add, which adds
//               each element exactly once in L2). Runs while the MMA warp
//               fills the other accumulator.
// Tile order: groups of 16 M-blocks, N-blocks inside a group, so a wave of
// 148 CTAs touches ~16 A row-panels and ~9 B column-panels (fits in L2).
// Every wait is bounded (about one second); on timeout the kernel records an
// error bit, stops issuing work, releases tensor memory and returns.
// No TMA multicast is used anywhere.
#include "f32x2.cuh"
#include "pdl.cuh"
#include "sm100_util.cuh"
#include "tmap.cuh"

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>

namespace {

using namespace fer::dev;

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;              // 16 KiB
constexpr int B_BYTES = BK * BN * 2;              // 32 KiB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;    // 48 KiB
constexpr int EPI_WARPS = 8;
constexpr int STAGING_BYTES = 32 * 128;           // one 32-row x 128-byte output box per epilogue warp
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + EPI_WARPS * STAGING_BYTES + 1024;
constexpr int kThreads = 64 + 32 * EPI_WARPS;
constexpr int GROUP_M = 16;
constexpr uint32_t TMEM_COLS = 512;

struct Bars {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];
    uint32_t tmem_base;
    int abort_flag;
};

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2),
// descriptor version 1, base offset 0 (tiles are 1024-byte aligned).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;          // version
    d |= 2ull << 61;          // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: f32 accumulator, bf16 A and B,
// A K-major, B N-major, M = 128, N = n (a multiple of 16, <= 256).
constexpr uint32_t idesc_n(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(BM >> 4) << 24);
}
constexpr uint32_t kIdesc = idesc_n(BN);

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate,
                                         uint32_t idesc = kIdesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive f32 columns of this thread's TMEM lane; the wait sits in the
// same asm statement, so no use of the registers is scheduled before it.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int* mb, int* nb) {
    const int per_group = GROUP_M * num_n;
    const int g = t / per_group;
    const int first_m = g * GROUP_M;
    const int gm = (num_m - first_m) < GROUP_M ? (num_m - first_m) : GROUP_M;
    const int r = t - g * per_group;
    *mb = first_m + r % gm;
    *nb = r / gm;
}

// Epilogue modes.
enum : int { kEpiF32 = 0, kEpiBF16 = 1, kEpiGeluBF16 = 2, kEpiResidF32 = 3 };

// GELU, x * Phi(x) with Phi(x) = (1 + erf(x / sqrt 2)) / 2 (the erf form the
// block's FFN uses), branch-free. erf comes from Abramowitz & Stegun 7.1.26
// (C. Hastings' approximation, |error| <= 1.5e-7 for x >= 0):
//   1 - erf(z) = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) exp(-z^2), t = 1 / (1 + p z),
// so with s = 1 - erf(|x| / sqrt 2): 1 + erf(x / sqrt 2) = s for x < 0 (no
// cancellation) and 2 - s otherwise. Max error against the exact function is
// ~4e-7 absolute, far below the bf16 rounding of the result.
// Every step is an explicitly rounded operation (no contraction), so the
// scalar form and the paired form below give the same bits.
__device__ __forceinline__ float gelu_erf(float x) {
    const float z = __fmul_rn(fabsf(x), 0.70710678118654752f);
    float t, e;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(__fmaf_rn(0.3275911f, z, 1.0f)));
    float h = __fmaf_rn(t, 1.061405429f, -1.453152027f);
    h = __fmaf_rn(t, h, 1.421413741f);
    h = __fmaf_rn(t, h, -0.284496736f);
    h = __fmaf_rn(t, h, 0.254829592f);
    const float poly = __fmul_rn(t, h);
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(__fmul_rn(__fmul_rn(z, z), -1.4426950408889634f)));
    const float s = __fmul_rn(poly, e);
    return __fmul_rn(__fmul_rn(0.5f, x), x < 0.0f ? s : __fsub_rn(2.0f, s));
}


// gelu_erf of a pair, the same operations on packed f32x2 (bit-identical
// to two scalar calls; about half the instructions in the epilogue).
__device__ __forceinline__ void gelu_erf2(float& x0, float& x1) {
    const uint64_t x = f2_pack(x0, x1);
    const uint64_t z = f2_mul(x & 0x7fffffff7fffffffull, f2_splat(0.70710678118654752f));
    float d0, d1, t0, t1;
    f2_unpack(f2_fma(f2_splat(0.3275911f), z, f2_splat(1.0f)), d0, d1);
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t0) : "f"(d0));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t1) : "f"(d1));
    const uint64_t t = f2_pack(t0, t1);
    uint64_t h = f2_fma(t, f2_splat(1.061405429f), f2_splat(-1.453152027f));
    h = f2_fma(t, h, f2_splat(1.421413741f));
    h = f2_fma(t, h, f2_splat(-0.284496736f));
    h = f2_fma(t, h, f2_splat(0.254829592f));
    const uint64_t poly = f2_mul(t, h);
    float a0, a1, e0, e1;
    f2_unpack(f2_mul(f2_mul(z, z), f2_splat(-1.4426950408889634f)), a0, a1);
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(a0));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(a1));
    const uint64_t s = f2_mul(poly, f2_pack(e0, e1));
    const uint64_t q = f2_sub(f2_splat(2.0f), s);
    float s0, s1, q0, q1;
    f2_unpack(s, s0, s1);
    f2_unpack(q, q0, q1);
    const uint64_t r = f2_pack(x0 < 0.0f ? s0 : q0, x1 < 0.0f ? s1 : q1);
    f2_unpack(f2_mul(f2_mul(f2_splat(0.5f), x), r), x0, x1);
}

// bf16 pair {lo, hi} (round to nearest even), lo in the low half.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t u;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(u) : "f"(hi), "f"(lo));
    return u;
}

// One 128-byte row of a staging box: 16-byte chunk j of row r lives at
// r*128 + ((j ^ (r & 7)) * 16), the layout a SWIZZLE_128B tensor map expects
// of a 1024-byte aligned box (and 8 distinct banks groups per 8 lanes).
__device__ __forceinline__ void stage_row(uint32_t sbase, int r, const uint32_t (&w)[32]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t a = sbase + static_cast<uint32_t>(r * 128 + ((j ^ (r & 7)) << 4));
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(w[4 * j]), "r"(w[4 * j + 1]),
                     "r"(w[4 * j + 2]), "r"(w[4 * j + 3])
                     : "memory");
    }
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t ssrc, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(ssrc), "r"(x), "r"(y)
                 : "memory");
}

// out[box] += staged[box], element by element in L2 (one add per element).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, uint32_t ssrc, int x, int y) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(ssrc), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t nclusters_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// 16 bytes of another CTA's shared memory (address from map_to_rank).
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

// Split-K epilogue for four consecutive outputs (float4 index i4 of the
// row-major M x N output; N % 4 == 0): the sum over splits, already added
// in split order, through the epilogue of fer_gemm_bf16_tc_ex.
__device__ __forceinline__ void splitk_store4(float4 acc, void* __restrict__ out, size_t i4, int epi) {
    if (epi == kEpiF32) {
        reinterpret_cast<float4*>(out)[i4] = acc;
    } else if (epi == kEpiResidF32) {
        float4 r = reinterpret_cast<float4*>(out)[i4];
        r.x += acc.x;
        r.y += acc.y;
        r.z += acc.z;
        r.w += acc.w;
        reinterpret_cast<float4*>(out)[i4] = r;
    } else {
        if (epi == kEpiGeluBF16) {
            acc.x = gelu_erf(acc.x);
            acc.y = gelu_erf(acc.y);
            acc.z = gelu_erf(acc.z);
            acc.w = gelu_erf(acc.w);
        }
        uint2 w;
        w.x = pack_bf16x2(acc.x, acc.y);
        w.y = pack_bf16x2(acc.z, acc.w);
        reinterpret_cast<uint2*>(out)[i4] = w;
    }
}

__device__ __forceinline__ void add4(float4& a, const float4& v) {
    a.x += v.x;
    a.y += v.y;
    a.z += v.z;
    a.w += v.w;
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// f32 partial tile of the cluster split-K mode: row stride in floats (the
// 4-float pad puts 8 consecutive rows' 16-byte pieces in distinct banks).
constexpr int part_stride(int bn) { return bn + 4; }
static_assert(BM * part_stride(BN) * 4 <= STAGES * STAGE_BYTES, "partial tile must fit the stage ring");

// kCluster: split-K through distributed shared memory. The grid is launched
// in clusters of `splits` CTAs; the CTAs of one cluster share one output tile
// (job t: tile t / splits, split t % splits = rank in the cluster), each
// computes its K range into TMEM and copies it to its shared memory, and
// after a cluster barrier CTA r adds the partials of all splits, in split
// order, for its 1/splits share of the tile and stores them through the
// epilogue directly to `out` (row-major M x N). No workspace, no second
// kernel; the same bits as the workspace form with the same split count.
// kBN: output tile width. 256 everywhere but in the narrow cluster form
// (128, or 64, for one M-block of at most 128 rows, the decode GEMMs): the
// cluster reduction moves rows x kBN x 4 bytes of partials between the SMs
// of a cluster per CTA, and that traffic, not the loads or the MMAs, is the
// longest phase of a decode GEMM with 256-wide tiles. Each stage keeps its
// 48 KiB slot; a narrow tile fills A plus kBN / 64 of the four B panels.
template <bool kCluster, int kBN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, int M, int N, int K, int epi, int splits, int kps,
                        void* __restrict__ out, int b_static, uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ Bars bars;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    static_assert(kBN == 64 || kBN == 128 || kBN == BN, "tile width 64, 128 or 256");
    static_assert(kBN == BN || kCluster, "narrow tiles only in the cluster form");
    constexpr int kStageTx = A_BYTES + BK * kBN * 2;     // bytes the TMA loads of one stage deliver
    constexpr int kPS = part_stride(kBN);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int num_m = (M + BM - 1) / BM, num_n = (N + kBN - 1) / kBN;
    const int num_tiles = num_m * num_n;
    const int num_k = (K + BK - 1) / BK;
    if (threadIdx.x == 32) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if (!kCluster) prefetch_tmap(&tmC);
    }
    // Split-K (splits > 1): job t covers k-blocks [kps * split, ...) of tile
    // t % num_tiles and stores its f32 partial at rows split * num_m * BM +
    // ... of C; splits == 1 is the plain GEMM (one job per tile, all of K).
    const int num_jobs = num_tiles * splits;
    auto job_tile = [&](int t) { return kCluster ? t / splits : t % num_tiles; };
    auto job_split = [&](int t) { return kCluster ? t % splits : t / num_tiles; };
    auto job_k = [&](int t, int* kb0, int* nk) {
        const int split = job_split(t);
        *kb0 = split * kps;
        const int left = num_k - *kb0;
        *nk = left < kps ? left : kps;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&bars.full[s], 1);
            mbar_init(&bars.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars.acc_full[b], 1);
            mbar_init(&bars.acc_empty[b], EPI_WARPS);   // one arrival per epilogue warp
        }
        bars.abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_addr(&bars.tmem_base)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars.tmem_base;
    // Setup above touches no global memory; under programmatic launch it
    // overlaps the previous kernel. The producer waits below, after it has
    // fetched what does not depend on that kernel.
    if (warp != 0) fer::dev::pdl_begin();

    volatile int* abort_flag = &bars.abort_flag;
    // Each role loop is run by its whole warp (waits voted across the warp,
    // issue from lane 0) so every warp reaches the final barrier converged.
    if (warp == 0) {
        // ---------------- TMA producer
        auto load_b = [&](int s, int nb, int kblock) {
            uint8_t* sb = smem + s * STAGE_BYTES + A_BYTES;
#pragma unroll
            for (int c = 0; c < kBN / 64; ++c)
                tma_load_2d(sb + c * (BK * 128), &tmB, nb * kBN + c * 64, kblock * BK, &bars.full[s]);
        };
        // b_static: B (weights) is not written by the previous kernel, so
        // the first job's first STAGES B tiles are fetched before the wait.
        int pre = 0;
        if (b_static && static_cast<int>(blockIdx.x) < num_jobs) {
            int mb, nb, kb0, nk;
            tile_coords(job_tile(blockIdx.x), num_m, num_n, &mb, &nb);
            job_k(blockIdx.x, &kb0, &nk);
            pre = nk < STAGES ? nk : STAGES;
            if (lane == 0)
                for (int kt = 0; kt < pre; ++kt) {
                    mbar_arrive_expect_tx(&bars.full[kt], kStageTx);
                    load_b(kt, nb, kb0 + kt);
                }
            __syncwarp();
        }
        fer::dev::pdl_begin();
        int it = 0;
        for (int t = blockIdx.x; t < num_jobs && !warp_flag(abort_flag); t += gridDim.x) {
            int mb, nb, kb0, nk;
            tile_coords(job_tile(t), num_m, num_n, &mb, &nb);
            job_k(t, &kb0, &nk);
            for (int kt = 0; kt < nk; ++kt, ++it) {
                const int s = it % STAGES;
                const uint32_t ph = static_cast<uint32_t>(it / STAGES) & 1u;
                if (it < pre) {
                    // slot armed and its B in flight since before the wait
                    if (lane == 0) tma_load_2d(smem + s * STAGE_BYTES, &tmA, (kb0 + kt) * BK, mb * BM, &bars.full[s]);
                    __syncwarp();
                    continue;
                }
                if (!__all_sync(0xffffffffu, mbar_wait(&bars.empty[s], ph ^ 1u))) {
                    if (lane == 0) report(err, kErrTimeoutSync);
                    *abort_flag = 1;
                    break;
                }
                if (lane == 0) {
                    mbar_arrive_expect_tx(&bars.full[s], kStageTx);
                    tma_load_2d(smem + s * STAGE_BYTES, &tmA, (kb0 + kt) * BK, mb * BM, &bars.full[s]);
                    load_b(s, nb, kb0 + kt);
                }
                __syncwarp();
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (lane 0 issues)
        int it = 0, local = 0;
        for (int t = blockIdx.x; t < num_jobs && !warp_flag(abort_flag); t += gridDim.x, ++local) {
            int kb0, nk;
            job_k(t, &kb0, &nk);
            const int buf = local & 1;
            const uint32_t acc_ph = static_cast<uint32_t>(local >> 1) & 1u;
            if (!__all_sync(0xffffffffu, mbar_wait(&bars.acc_empty[buf], acc_ph ^ 1u))) {
                if (lane == 0) report(err, kErrTimeoutSync);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            const uint32_t d = tmem + static_cast<uint32_t>(buf * kBN);
            bool ok = true;
            for (int kt = 0; kt < nk; ++kt, ++it) {
                const int s = it % STAGES;
                const uint32_t ph = static_cast<uint32_t>(it / STAGES) & 1u;
                if (!__all_sync(0xffffffffu, mbar_wait(&bars.full[s], ph))) {
                    if (lane == 0) report(err, kErrTimeoutLoad);
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t sa = smem_addr(smem + s * STAGE_BYTES);
                    const uint32_t sb = sa + A_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        // A: K-major, +32 bytes per 16 elements of K inside the swizzle atom.
                        const uint64_t ad = smem_desc(sa + k * 32, 16, 1024);
                        // B: N-major, 16 K-rows of 128 bytes per step; 64-column panels 8 KiB apart.
                        const uint64_t bd = smem_desc(sb + k * 16 * 128, BK * 128, 1024);
                        mma_bf16(d, ad, bd, (kt | k) ? 1u : 0u, idesc_n(kBN));
                    }
                    mma_commit(&bars.empty[s]);   // ring slot free once these MMAs finish
                }
                __syncwarp();
            }
            if (!ok) break;
            if (lane == 0) mma_commit(&bars.acc_full[buf]);   // accumulator complete
            __syncwarp();
        }
    } else {
        // ---------------- epilogue warps 2..9: TMEM lanes 32*(warp%4) .., columns half*128 ..
        const int q = warp & 3;
        const int half = (warp - 2) >> 2;
        const uint32_t stage = smem_addr(smem + STAGES * STAGE_BYTES + (warp - 2) * STAGING_BYTES);
        const bool f32_out = epi == kEpiF32 || epi == kEpiResidF32;
        const int chunk_cols = f32_out ? 32 : 64;            // one 128-byte box row
        const int n_chunks = (kBN / 2) / chunk_cols;
        int local = 0;
        for (int t = blockIdx.x; t < num_jobs; t += gridDim.x, ++local) {
            const int buf = local & 1;
            const uint32_t acc_ph = static_cast<uint32_t>(local >> 1) & 1u;
            const bool got = __all_sync(0xffffffffu, mbar_wait(&bars.acc_full[buf], acc_ph));
            if (!got || warp_flag(abort_flag)) {
                if (lane == 0 && !got) report(err, kErrTimeoutMma);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            int mb, nb;
            tile_coords(job_tile(t), num_m, num_n, &mb, &nb);
            const int row_in = mb * BM + q * 32;                          // row within this job's M rows
            const int row0 = job_split(t) * num_m * BM + row_in;          // row of C (split block offset)
            const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(buf * kBN + half * (kBN / 2));
            if constexpr (kCluster) {
                // f32 partial rows -> this CTA's shared memory (the stage
                // ring is idle: every load of the one job has been consumed
                // by MMAs that completed before acc_full)
                const int r = q * 32 + lane;
                const bool live = row_in + lane < M;
                const uint32_t prow = smem_addr(smem) + static_cast<uint32_t>((r * kPS + half * (kBN / 2)) * 4);
#pragma unroll 1
                for (int c = 0; c < (kBN / 2) / 32; ++c) {
                    uint32_t w[32];
                    tmem_ld32(tbase + c * 32, w);
                    if (c == (kBN / 2) / 32 - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&bars.acc_empty[buf]);
                    }
                    if (live) {
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(prow + (c * 32 + 4 * j) * 4),
                                         "r"(w[4 * j]), "r"(w[4 * j + 1]), "r"(w[4 * j + 2]), "r"(w[4 * j + 3])
                                         : "memory");
                    }
                }
                continue;
            }
#pragma unroll 1
            for (int c = 0; c < n_chunks; ++c) {
                uint32_t w[32];
                if (f32_out) {
                    tmem_ld32(tbase + c * 32, w);
                } else {
                    const bool gelu = epi == kEpiGeluBF16;
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2) {
                        uint32_t r[32];
                        tmem_ld32(tbase + c * 64 + h2 * 32, r);
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            float a0 = __uint_as_float(r[2 * j]), a1 = __uint_as_float(r[2 * j + 1]);
                            if (gelu) gelu_erf2(a0, a1);
                            w[16 * h2 + j] = pack_bf16x2(a0, a1);
                        }
                    }
                }
                if (c == n_chunks - 1) {
                    // every TMEM read of this accumulator is done: hand it back
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&bars.acc_empty[buf]);
                }
                // the previous box has been read out of the staging buffer
                if (lane == 0) bulk_wait_read0();
                __syncwarp();
                stage_row(stage, lane, w);
                fence_proxy_async_smem();
                __syncwarp();
                const int col0 = nb * kBN + half * (kBN / 2) + c * chunk_cols;
                if (lane == 0 && row_in < M && col0 < N) {
                    if (epi == kEpiResidF32) tma_reduce_add_2d(&tmC, stage, col0, row0);
                    else tma_store_2d(&tmC, stage, col0, row0);
                    bulk_commit();
                }
                __syncwarp();
            }
        }
        if (lane == 0) bulk_wait0();
        __syncwarp();
    }

    if constexpr (kCluster) {
        cluster_sync_all();   // every split's partial is in its CTA's shared memory
        const int t = blockIdx.x;
        int mb, nb;
        tile_coords(job_tile(t), num_m, num_n, &mb, &nb);
        const int rank = job_split(t);
        const int rows = M - mb * BM < BM ? M - mb * BM : BM;
        const int total = rows * (kBN / 4);                    // float4 pieces of the tile's live rows
        const int per = (total + splits - 1) / splits;
        const int f_end = (rank + 1) * per < total ? (rank + 1) * per : total;
        const uint32_t pbase = smem_addr(smem);
        for (int f = rank * per + static_cast<int>(threadIdx.x); f < f_end; f += kThreads) {
            const int r = f / (kBN / 4), c4 = f % (kBN / 4);
            const int col = nb * kBN + c4 * 4;
            if (col >= N) continue;
            const uint32_t off = pbase + static_cast<uint32_t>((r * kPS + c4 * 4) * 4);
            // every split's load in flight at once (splits <= 16), then the
            // additions in split order
            float4 v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u)
                if (u < splits) v[u] = ld_cluster_f4(map_to_rank(off, static_cast<uint32_t>(u)));
            float4 acc = v[0];
#pragma unroll
            for (int u = 1; u < 16; ++u)
                if (u < splits) add4(acc, v[u]);
            splitk_store4(acc, out, (static_cast<size_t>(mb * BM + r) * N + col) / 4, epi);
        }
        cluster_sync_all();   // no CTA exits while its partial is still being read
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ================================================================ 2-CTA version
//
// A cluster of two CTAs (two SMs) computes a 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256): CTA r holds A rows [128r, 128r+128) of
// the tile and B columns [128r, 128r+128), so each SM fetches 32 KiB per
// 64-deep k-block instead of 48 KiB, and six stages fit where four did.
// Both CTAs' TMA loads complete on the leader's (rank 0) full barrier; the
// leader's MMA thread issues for the pair and its commits arrive on both
// CTAs' barriers (tcgen05.commit multicast). Each CTA's epilogue drains its
// own TMEM rows (same code path as above) and releases the accumulator with
// an arrive on the leader's acc_empty barrier. No TMA multicast is used.
constexpr int STAGES2 = 6;
constexpr int A2_BYTES = 128 * BK * 2;            // 16 KiB: this CTA's 128 rows
constexpr int B2_BYTES = BK * 128 * 2;            // 16 KiB: this CTA's 128 columns (two 64-column panels)
constexpr int STAGE2_BYTES = A2_BYTES + B2_BYTES;
constexpr int SMEM2_BYTES = STAGES2 * STAGE2_BYTES + EPI_WARPS * STAGING_BYTES + 1024;
constexpr int GROUP_M2 = 8;                       // default 256-row blocks per raster group
// kind::f16, f32 accumulator, bf16 A/B, A K-major, B N-major, N = 256, M = 256.
constexpr uint32_t kIdesc2 = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | (static_cast<uint32_t>(256 >> 3) << 17) |
                             (static_cast<uint32_t>(256 >> 4) << 24);

struct Bars2 {
    uint64_t full[STAGES2];     // leader's copy is the one used
    uint64_t empty[STAGES2];
    uint64_t acc_full[2];
    uint64_t acc_empty[2];      // leader's copy: 2 x EPI_WARPS arrivals per phase
    uint32_t tmem_base;
    int abort_flag;
};

__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc2), "r"(accumulate)
        : "memory");
}
// Arrives on the barrier at this offset in both CTAs once the MMAs issued so far complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_addr(bar)),
        "h"(static_cast<uint16_t>(3))
        : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

__device__ __forceinline__ void tile_coords2(int t, int num_m2, int num_n, int group_m, int* mb, int* nb) {
    const int per_group = group_m * num_n;
    const int g = t / per_group;
    const int first_m = g * group_m;
    const int gm = (num_m2 - first_m) < group_m ? (num_m2 - first_m) : group_m;
    const int r = t - g * per_group;
    *mb = first_m + r % gm;
    *nb = r / gm;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm_bf16_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmC, int M, int N, int K, int epi, int group_m,
                         uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ Bars2 bars;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const bool leader = rank == 0;
    const int cid = static_cast<int>(cluster_id_x()), ncl = static_cast<int>(nclusters_x());
    const int num_m2 = (M + 255) / 256, num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m2 * num_n;
    const int num_k = (K + BK - 1) / BK;
    if (threadIdx.x == 32) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        prefetch_tmap(&tmC);
    }

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES2; ++s) {
            mbar_init(&bars.full[s], 1);
            mbar_init(&bars.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars.acc_full[b], 1);
            mbar_init(&bars.acc_empty[b], 2 * EPI_WARPS);
        }
        bars.abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&bars.tmem_base)),
                     "r"(TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync_all();   // barriers initialised and TMEM allocated in both CTAs
    tc_fence_after();
    const uint32_t tmem = bars.tmem_base;
    volatile int* abort_flag = &bars.abort_flag;
    // Set-up above touches no global memory: under programmatic launch it
    // overlaps the previous kernel's tail. Every thread waits for that kernel
    // here and then lets the next kernel be scheduled (no-ops under a plain
    // launch).
    fer::dev::pdl_begin();

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs): own A rows, own B columns
        const uint32_t full0 = map_to_rank(smem_addr(&bars.full[0]), 0);
        int it = 0;
        for (int t = cid; t < num_tiles && !warp_flag(abort_flag); t += ncl) {
            int mb, nb;
            tile_coords2(t, num_m2, num_n, group_m, &mb, &nb);
            const int row = mb * 256 + static_cast<int>(rank) * 128;
            const int col = nb * BN + static_cast<int>(rank) * 128;
            for (int kt = 0; kt < num_k; ++kt, ++it) {
                const int s = it % STAGES2;
                const uint32_t ph = static_cast<uint32_t>(it / STAGES2) & 1u;
                if (!__all_sync(0xffffffffu, mbar_wait(&bars.empty[s], ph ^ 1u))) {
                    if (lane == 0) report(err, kErrTimeoutSync);
                    *abort_flag = 1;
                    break;
                }
                if (lane == 0) {
                    const uint32_t fb = full0 + static_cast<uint32_t>(s * sizeof(uint64_t));
                    if (leader) mbar_arrive_expect_tx(&bars.full[s], 2 * STAGE2_BYTES);
                    const uint32_t sa = smem_addr(smem + s * STAGE2_BYTES);
                    tma_load_2d_pair(sa, &tmA, kt * BK, row, fb);
                    tma_load_2d_pair(sa + A2_BYTES, &tmB, col, kt * BK, fb);
                    tma_load_2d_pair(sa + A2_BYTES + BK * 128, &tmB, col + 64, kt * BK, fb);
                }
                __syncwarp();
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: the leader's warp 1 issues for the pair
        if (leader) {
            int it = 0, local = 0;
            for (int t = cid; t < num_tiles && !warp_flag(abort_flag); t += ncl, ++local) {
                const int buf = local & 1;
                const uint32_t acc_ph = static_cast<uint32_t>(local >> 1) & 1u;
                if (!__all_sync(0xffffffffu, mbar_wait(&bars.acc_empty[buf], acc_ph ^ 1u))) {
                    if (lane == 0) report(err, kErrTimeoutSync);
                    *abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + static_cast<uint32_t>(buf * BN);
                bool ok = true;
                for (int kt = 0; kt < num_k; ++kt, ++it) {
                    const int s = it % STAGES2;
                    const uint32_t ph = static_cast<uint32_t>(it / STAGES2) & 1u;
                    if (!__all_sync(0xffffffffu, mbar_wait(&bars.full[s], ph))) {
                        if (lane == 0) report(err, kErrTimeoutLoad);
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    if (lane == 0) {
                        const uint32_t sa = smem_addr(smem + s * STAGE2_BYTES);
                        const uint32_t sb = sa + A2_BYTES;
#pragma unroll
                        for (int k = 0; k < BK / 16; ++k) {
                            const uint64_t ad = smem_desc(sa + k * 32, 16, 1024);
                            const uint64_t bd = smem_desc(sb + k * 16 * 128, BK * 128, 1024);
                            mma_bf16_pair(d, ad, bd, (kt | k) ? 1u : 0u);
                        }
                        mma_commit_pair(&bars.empty[s]);
                    }
                    __syncwarp();
                }
                if (!ok) break;
                if (lane == 0) mma_commit_pair(&bars.acc_full[buf]);
                __syncwarp();
            }
        }
    } else {
        // ---------------- epilogue warps 2..9 (both CTAs): this CTA's 128 rows
        const int q = warp & 3;
        const int half = (warp - 2) >> 2;
        const uint32_t stage = smem_addr(smem + STAGES2 * STAGE2_BYTES + (warp - 2) * STAGING_BYTES);
        const uint32_t acc_empty0 = map_to_rank(smem_addr(&bars.acc_empty[0]), 0);
        const bool f32_out = epi == kEpiF32 || epi == kEpiResidF32;
        const int chunk_cols = f32_out ? 32 : 64;
        const int n_chunks = (BN / 2) / chunk_cols;
        int local = 0;
        for (int t = cid; t < num_tiles; t += ncl, ++local) {
            const int buf = local & 1;
            const uint32_t acc_ph = static_cast<uint32_t>(local >> 1) & 1u;
            const bool got = __all_sync(0xffffffffu, mbar_wait(&bars.acc_full[buf], acc_ph));
            if (!got || warp_flag(abort_flag)) {
                if (lane == 0 && !got) report(err, kErrTimeoutMma);
                *abort_flag = 1;
                break;
            }
            tc_fence_after();
            int mb, nb;
            tile_coords2(t, num_m2, num_n, group_m, &mb, &nb);
            const int row0 = mb * 256 + static_cast<int>(rank) * 128 + q * 32;
            const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16) +
                                   static_cast<uint32_t>(buf * BN + half * (BN / 2));
#pragma unroll 1
            for (int c = 0; c < n_chunks; ++c) {
                uint32_t w[32];
                if (f32_out) {
                    tmem_ld32(tbase + c * 32, w);
                } else {
                    const bool gelu = epi == kEpiGeluBF16;
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2) {
                        uint32_t r[32];
                        tmem_ld32(tbase + c * 64 + h2 * 32, r);
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            float a0 = __uint_as_float(r[2 * j]), a1 = __uint_as_float(r[2 * j + 1]);
                            if (gelu) gelu_erf2(a0, a1);
                            w[16 * h2 + j] = pack_bf16x2(a0, a1);
                        }
                    }
                }
                if (c == n_chunks - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(acc_empty0 + static_cast<uint32_t>(buf * sizeof(uint64_t)));
                }
                if (lane == 0) bulk_wait_read0();
                __syncwarp();
                stage_row(stage, lane, w);
                fence_proxy_async_smem();
                __syncwarp();
                const int col0 = nb * BN + half * (BN / 2) + c * chunk_cols;
                if (lane == 0 && row0 < M && col0 < N) {
                    if (epi == kEpiResidF32) tma_reduce_add_2d(&tmC, stage, col0, row0);
                    else tma_store_2d(&tmC, stage, col0, row0);
                    bulk_commit();
                }
                __syncwarp();
            }
        }
        if (lane == 0) bulk_wait0();
        __syncwarp();
    }

    tc_fence_before();
    cluster_sync_all();   // no CTA leaves while its peer's MMAs or arrivals may still touch it
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

// ---------------------------------------------------------------- host side

using fer::host::EncodeTiledFn;

EncodeTiledFn encode_fn() { return fer::host::encode_tiled_fn(); }

// Tuning knobs read once per process: FERCUDA_GEMM_GROUP (256-row blocks
// per raster group of the 2-CTA kernel) and FERCUDA_GEMM_L2_PROMOTION
// (0 none, 1 64 B, 2 128 B, 3 256 B for the TMA loads).
// Default: GROUP_M2, or twice that for wide outputs (64 or more 256-column
// tiles, e.g. an LM head), where a taller group re-reads the wide B operand
// fewer times.
int gemm_group_m(int num_n) {
    static const int g = [] {
        const char* e = std::getenv("FERCUDA_GEMM_GROUP");
        const int v = e ? std::atoi(e) : 0;
        return v < 1 ? 0 : v;
    }();
    if (g) return g;
    return num_n >= 64 ? 2 * GROUP_M2 : GROUP_M2;
}

int l2_promotion() {
    static const int p = [] {
        const char* e = std::getenv("FERCUDA_GEMM_L2_PROMOTION");
        const int v = e ? std::atoi(e) : static_cast<int>(CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
        return (v < 0 || v > 3) ? static_cast<int>(CU_TENSOR_MAP_L2_PROMOTION_L2_256B) : v;
    }();
    return p;
}

// 2-D tensor map over a row-major [rows, cols] matrix of 2- or 4-byte
// elements, box [box_rows, 128 bytes], 128-byte swizzle.
bool make_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
              CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const uint32_t esize = dt == CU_TENSOR_MAP_DATA_TYPE_FLOAT32 ? 4u : 2u;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * esize};
    const cuuint32_t box[2] = {128u / esize, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, static_cast<CUtensorMapL2promotion>(l2_promotion()),
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
    static const int n = [] {
        int dev = 0, v = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v > 0 ? v : 148;
    }();
    return n;
}

// Programmatic launch of the 2-CTA kernel (its set-up overlaps the tail of
// the kernel before; at 4096 tokens per GPU the forward takes 2-3% less
// time, at 32768 the same): on unless FERCUDA_GEMM_PDL=0 or FERCUDA_PDL=0.
bool tc2_pdl() {
    static const bool on = [] {
        const char* e = std::getenv("FERCUDA_GEMM_PDL");
        return !(e && e[0] == '0') && fer::host::pdl_enabled();
    }();
    return on;
}

int g_gemm_mode = 0;        // 0: 2-CTA kernel where it applies, 1: always the 1-CTA kernel
std::atomic<int> g_gemm_clusters{-1};   // co-resident 2-CTA clusters (queried once; same value from any thread)

}  // namespace

// Selects the GEMM kernel: 0 (default) the 2-CTA cluster kernel for M > 128,
// 1 the single-CTA kernel everywhere. Both give bit-identical results.
extern "C" void fer_gemm_tc_set_mode(int mode) { g_gemm_mode = mode; }

// Number of 2-CTA clusters the persistent kernel launches at most (-1 before
// the first 2-CTA GEMM on this device).
extern "C" int fer_gemm_tc_clusters() { return g_gemm_clusters.load(std::memory_order_relaxed); }

// epi: 0 f32 out, 1 bf16 out, 2 bf16(gelu(acc)), 3 f32 out = resid + acc.
// With resid == c the residual add happens in place (TMA reduce-add); any
// other resid is first copied into c (it must not partly overlap c).
// Requires K % 8 == 0 and N % 8 == 0 (16-byte row pitches for the tensor
// maps) and 16-byte aligned operands; returns cudaErrorInvalidValue otherwise.
namespace {

cudaError_t gemm_ex(const void* a, const void* b, void* c, const float* resid, int M, int N, int K, int epi,
                    int b_static, uint32_t* err, cudaStream_t stream) {
    if (M <= 0 || N <= 0 || K <= 0 || (K % 8) || (N % 8)) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c)) & 15u)
        return cudaErrorInvalidValue;
    if (epi < kEpiF32 || epi > kEpiResidF32 || (epi == kEpiResidF32 && (!resid || (reinterpret_cast<uintptr_t>(resid) & 15u))))
        return cudaErrorInvalidValue;
    const bool f32_out = epi == kEpiF32 || epi == kEpiResidF32;
    CUtensorMap ma, mb, mc;
    if (!make_map(&ma, a, static_cast<uint64_t>(M), static_cast<uint64_t>(K), BM) ||
        !make_map(&mb, b, static_cast<uint64_t>(K), static_cast<uint64_t>(N), BK) ||
        !make_map(&mc, c, static_cast<uint64_t>(M), static_cast<uint64_t>(N), 32,
                  f32_out ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16))
        return cudaErrorInvalidValue;
    if (epi == kEpiResidF32 && resid != c) {
        const size_t bytes = static_cast<size_t>(M) * N * sizeof(float);
        const uintptr_t r0 = reinterpret_cast<uintptr_t>(resid), c0 = reinterpret_cast<uintptr_t>(c);
        if (r0 < c0 + bytes && c0 < r0 + bytes) return cudaErrorInvalidValue;
        cudaError_t e = cudaMemcpyAsync(c, resid, bytes, cudaMemcpyDeviceToDevice, stream);
        if (e != cudaSuccess) return e;
    }
    if (g_gemm_mode != 1 && M > BM) {
        // 2-CTA kernel: A boxes of 128 rows per CTA, one 256-row tile per cluster
        int clusters = g_gemm_clusters.load(std::memory_order_relaxed);
        if (clusters < 0) {
            cudaError_t e = cudaFuncSetAttribute(gemm_bf16_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 SMEM2_BYTES);
            if (e != cudaSuccess) return e;
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
            cfg.blockDim = dim3(kThreads, 1, 1);
            cfg.dynamicSmemBytes = SMEM2_BYTES;
            int n = 0;
            e = cudaOccupancyMaxActiveClusters(&n, gemm_bf16_tc2_kernel, &cfg);
            clusters = (e == cudaSuccess && n > 0) ? n : 0;
            if (e != cudaSuccess) cudaGetLastError();
            g_gemm_clusters.store(clusters, std::memory_order_relaxed);
        }
        if (clusters > 0) {
            const int tiles2 = ((M + 255) / 256) * ((N + BN - 1) / BN);
            const int ncl = tiles2 < clusters ? tiles2 : clusters;
            const int gm = gemm_group_m((N + BN - 1) / BN);
            fer_pdl_note_launch();   // the kernel triggers its dependents under either launch
            if (tc2_pdl()) {
                cudaLaunchConfig_t cfg{};
                cfg.gridDim = dim3(2 * ncl);
                cfg.blockDim = dim3(kThreads);
                cfg.dynamicSmemBytes = SMEM2_BYTES;
                cfg.stream = stream;
                cudaLaunchAttribute at[1];
                at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
                at[0].val.programmaticStreamSerializationAllowed = 1;
                cfg.attrs = at;
                cfg.numAttrs = 1;
                const cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_bf16_tc2_kernel, ma, mb, mc, M, N, K, epi, gm, err);
                return e != cudaSuccess ? e : cudaGetLastError();
            }
            gemm_bf16_tc2_kernel<<<2 * ncl, kThreads, SMEM2_BYTES, stream>>>(ma, mb, mc, M, N, K, epi, gm, err);
            return cudaGetLastError();
        }
    }
    static const cudaError_t attr_rc = cudaFuncSetAttribute(gemm_bf16_tc_kernel<false, BN>,
                                                            cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (attr_rc != cudaSuccess) return attr_rc;
    const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    const int grid = tiles < sm_count() ? tiles : sm_count();
    const cudaError_t e = fer::host::launch_pdl(gemm_bf16_tc_kernel<false, BN>, dim3(grid), dim3(kThreads), SMEM_BYTES,
                                                stream, ma, mb, mc, M, N, K, epi, 1, (K + BK - 1) / BK,
                                                static_cast<void*>(nullptr), b_static, err);
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace

extern "C" cudaError_t fer_gemm_bf16_tc_ex(const void* a, const void* b, void* c, const float* resid, int M, int N,
                                           int K, int epi, uint32_t* err, cudaStream_t stream) {
    return gemm_ex(a, b, c, resid, M, N, K, epi, 0, err, stream);
}

namespace {

// out = epilogue(sum over splits s = 0, 1, ... of part[s * mpad + m][n]) for
// m < M: the partials are added in split order, so the result is the same
// bits on every run.
__global__ void __launch_bounds__(256) splitk_reduce(const float* __restrict__ part, void* __restrict__ out, int M,
                                                     int N, int mpad, int splits, int epi) {
    fer::dev::pdl_begin();
    const size_t total4 = static_cast<size_t>(M) * N / 4;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total4; i += stride) {
        const size_t e = i * 4;
        const size_t m = e / N, n = e % N;
        const size_t slab = static_cast<size_t>(mpad) * N;   // floats between consecutive splits
        const float4* src = reinterpret_cast<const float4*>(part + m * N + n);
        float4 acc = src[0];
        int sp = 1;
        // four splits' loads in flight, added in split order
        for (; sp + 3 < splits; sp += 4) {
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = src[(sp + u) * slab / 4];
#pragma unroll
            for (int u = 0; u < 4; ++u) add4(acc, v[u]);
        }
        for (; sp < splits; ++sp) add4(acc, src[sp * slab / 4]);
        splitk_store4(acc, out, i, epi);
    }
}

}  // namespace

namespace {

size_t splitk_bytes(int M, int N, int splits) {
    const size_t mpad = static_cast<size_t>((M + BM - 1) / BM) * BM;
    return static_cast<size_t>(splits) * mpad * N * sizeof(float);
}

// Splits actually used: `want` (<= 0: enough jobs for one per SM), at most
// one per 64-deep k-block, reduced until the partials fit ws_bytes; every
// split gets at least one block. 0 when even one split does not fit.
int splitk_plan(int M, int N, int K, int want, size_t ws_bytes, int* kps_out) {
    const int num_k = (K + BK - 1) / BK;
    const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
    int splits = want > 0 ? want : (sm_count() + tiles - 1) / tiles;
    if (splits > num_k) splits = num_k;
    if (splits < 1) splits = 1;
    while (splits > 1 && splitk_bytes(M, N, splits) > ws_bytes) --splits;
    if (splitk_bytes(M, N, splits) > ws_bytes) return 0;
    const int kps = (num_k + splits - 1) / splits;
    *kps_out = kps;
    return (num_k + kps - 1) / kps;
}

}  // namespace

// Workspace bytes for fer_gemm_bf16_tc_splitk with the automatic split count.
extern "C" size_t fer_gemm_splitk_workspace_bytes(int M, int N, int K) {
    int kps = 0;
    const int splits = splitk_plan(M, N, K, 0, static_cast<size_t>(-1), &kps);
    return splitk_bytes(M, N, splits);
}

namespace {

// Largest cluster of split-K CTAs allowed (FERCUDA_SPLITK_CLUSTER: 0 turns
// the cluster form off, 2..16 caps the cluster size; default 16).
int csplit_cap() {
    static const int cap = [] {
        const char* e = std::getenv("FERCUDA_SPLITK_CLUSTER");
        if (!e || !*e) return 16;
        const int v = std::atoi(e);
        return v < 2 ? 0 : (v > 16 ? 16 : v);
    }();
    return cap;
}

// Output tile width of the cluster form for M rows: 128 for a single
// M-block (the decode GEMMs: half the partial traffic of a 256-wide tile per
// CTA, twice the tiles to spread the weights over), 256 otherwise. Measured
// at M = 64 (d 1024, ffn 4096), microseconds per launch for widths 256 / 128
// / 64: QKV 7.96 / 7.06 / 7.65, out-proj 8.28 / 6.69 / 6.78, W1 8.42 / 7.51 /
// 7.93, W2 9.54 / 8.77 / 8.78 (64 leaves room for fewer splits, so each CTA
// walks more of K). FERCUDA_SPLITK_BN = 64, 128 or 256 fixes the width.
int csplit_bn(int M) {
    static const int env = [] {
        const char* e = std::getenv("FERCUDA_SPLITK_BN");
        const int v = e ? std::atoi(e) : 0;
        return (v == 64 || v == 128 || v == BN) ? v : 0;
    }();
    if (env) return env;
    return M <= BM ? 128 : BN;
}

using ClusterKernel = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, int, int, int, int, int, int, void*, int,
                               uint32_t*);
ClusterKernel cluster_kernel(int bn) {
    return bn == 64 ? gemm_bf16_tc_kernel<true, 64> : bn == 128 ? gemm_bf16_tc_kernel<true, 128>
                                                                : gemm_bf16_tc_kernel<true, BN>;
}

// Clusters of `size` CTAs of the cluster split-K kernel with tile width bn
// that can be resident at once (0: none), queried once per (width, size);
// also sets the kernel's shared-memory and cluster-size attributes.
int csplit_max_clusters(int size, int bn) {
    static std::atomic<int> cache[3][17] = {};
    const int wi = bn == 64 ? 0 : bn == 128 ? 1 : 2;
    const ClusterKernel kern = cluster_kernel(bn);
    if (cache[wi][size].load(std::memory_order_relaxed) == 0) {
        int n = 0;
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
        if (e == cudaSuccess && size > 8)
            e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e == cudaSuccess) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(static_cast<unsigned>(size * 16));
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = SMEM_BYTES;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = static_cast<unsigned>(size);
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = 1;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
        }
        if (e != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        cache[wi][size].store(n > 0 ? n : -1, std::memory_order_relaxed);
    }
    const int v = cache[wi][size].load(std::memory_order_relaxed);
    return v > 0 ? v : 0;
}

// Cluster split-K plan: the largest split count S <= 16 (each split whole
// 64-deep k-blocks, S = ceil(num_k / ceil(num_k / S))) whose clusters of S
// CTAs all fit on the GPU at once, one cluster per output tile of width
// *bn_out (csplit_bn). 1: no split fits (the plain kernel runs); 0: the
// cluster form is off.
int csplit_plan(int M, int N, int K, int* kps_out, int* bn_out) {
    const int cap = csplit_cap();
    const int num_k = (K + BK - 1) / BK;
    const int bn = csplit_bn(M);
    *kps_out = num_k;
    *bn_out = bn;
    if (cap == 0) return 0;
    const int tiles = ((M + BM - 1) / BM) * ((N + bn - 1) / bn);
    for (int S = num_k < cap ? num_k : cap; S >= 2; --S) {
        const int kps = (num_k + S - 1) / S;
        if ((num_k + kps - 1) / kps != S) continue;
        if (tiles <= csplit_max_clusters(S, bn)) {
            *kps_out = kps;
            return S;
        }
    }
    return 1;
}

}  // namespace

// Split count the automatic fer_gemm_bf16_tc_splitk uses in its cluster
// form: >= 2 clusters of that many CTAs, 1 the single-pass kernel, 0 the
// cluster form is switched off (FERCUDA_SPLITK_CLUSTER=0).
extern "C" int fer_gemm_splitk_cluster_splits(int M, int N, int K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    int kps = 0, bn = 0;
    return csplit_plan(M, N, K, &kps, &bn);
}

// Split-K tensor-core GEMM for short M (decode steps): K is divided into
// ranges of whole 64-deep blocks computed by separate CTAs, and the f32
// partials are added in range order before the epilogue (epi as
// fer_gemm_bf16_tc_ex; for epi 3 the residual is c itself). Deterministic,
// but the additions are grouped differently from fer_gemm_bf16_tc_ex, so the
// low bits differ from it.
// splits <= 0 (automatic): the cluster form (fer_gemm_splitk_cluster_splits)
// adds the partials through distributed shared memory inside one kernel, or
// the single-pass kernel runs when no split fits; ws is not touched.
// splits > 0, or the cluster form switched off: the partials go to the f32
// workspace ws and one more kernel adds them; the count is reduced until the
// partials fit ws_bytes (cudaErrorInvalidValue if one split does not), and
// with the cluster form off, splits <= 0 gives every SM one job. Both forms
// give the same bits for the same split count.
// flags bit 0: b is not written by the kernel just before this call on the
// stream (weights), so its first tiles are fetched before the programmatic
// launch wait, overlapping that kernel's tail.
extern "C" cudaError_t fer_gemm_bf16_tc_splitk(const void* a, const void* b, void* c, int M, int N, int K, int epi,
                                               int splits, float* ws, size_t ws_bytes, int flags, uint32_t* err,
                                               cudaStream_t stream) {
    const int b_static = flags & 1;
    if (M <= 0 || N <= 0 || K <= 0 || (K % 8) || (N % 8) || epi < kEpiF32 || epi > kEpiResidF32 || !ws)
        return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c) |
         reinterpret_cast<uintptr_t>(ws)) & 15u)
        return cudaErrorInvalidValue;
    int kps = 0;
    if (splits <= 0) {
        int bn = BN;
        const int cs = csplit_plan(M, N, K, &kps, &bn);
        if (cs == 1) return gemm_ex(a, b, c, epi == kEpiResidF32 ? static_cast<const float*>(c) : nullptr, M, N, K,
                                    epi, b_static, err, stream);
        if (cs >= 2) {
            CUtensorMap ma, mb;
            if (!make_map(&ma, a, static_cast<uint64_t>(M), static_cast<uint64_t>(K), BM) ||
                !make_map(&mb, b, static_cast<uint64_t>(K), static_cast<uint64_t>(N), BK))
                return cudaErrorInvalidValue;
            const int tiles = ((M + BM - 1) / BM) * ((N + bn - 1) / bn);
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(static_cast<unsigned>(tiles * cs));
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = SMEM_BYTES;
            cfg.stream = stream;
            cudaLaunchAttribute at[2];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = static_cast<unsigned>(cs);
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = 1;
            at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            at[1].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = at;
            cfg.numAttrs = fer::host::pdl_enabled() ? 2 : 1;
            fer_pdl_note_launch();   // the kernel triggers its dependents either way
            // the C map is not used by the cluster form
            const cudaError_t e = cudaLaunchKernelEx(&cfg, cluster_kernel(bn), ma, mb, ma, M, N, K, epi, cs, kps, c,
                                                     b_static, err);
            return e != cudaSuccess ? e : cudaGetLastError();
        }
    }
    splits = splitk_plan(M, N, K, splits, ws_bytes, &kps);
    if (splits == 0) return cudaErrorInvalidValue;
    const int num_m = (M + BM - 1) / BM;
    const int tiles = num_m * ((N + BN - 1) / BN);
    const int mpad = num_m * BM;
    CUtensorMap ma, mb, mc;
    if (!make_map(&ma, a, static_cast<uint64_t>(M), static_cast<uint64_t>(K), BM) ||
        !make_map(&mb, b, static_cast<uint64_t>(K), static_cast<uint64_t>(N), BK) ||
        !make_map(&mc, ws, static_cast<uint64_t>(splits) * mpad, static_cast<uint64_t>(N), 32,
                  CU_TENSOR_MAP_DATA_TYPE_FLOAT32))
        return cudaErrorInvalidValue;
    static const cudaError_t attr_rc = cudaFuncSetAttribute(gemm_bf16_tc_kernel<false, BN>,
                                                            cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (attr_rc != cudaSuccess) return attr_rc;
    const int jobs = tiles * splits;
    const int grid = jobs < sm_count() ? jobs : sm_count();
    cudaError_t e = fer::host::launch_pdl(gemm_bf16_tc_kernel<false, BN>, dim3(grid), dim3(kThreads), SMEM_BYTES, stream,
                                          ma, mb, mc, M, N, K, static_cast<int>(kEpiF32), splits, kps,
                                          static_cast<void*>(nullptr), b_static, err);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t total4 = static_cast<size_t>(M) * N / 4;
    size_t g = (total4 + 255) / 256;
    if (g > static_cast<size_t>(sm_count()) * 8) g = static_cast<size_t>(sm_count()) * 8;
    e = fer::host::launch_pdl(splitk_reduce, dim3(static_cast<unsigned>(g)), dim3(256), 0, stream,
                              static_cast<const float*>(ws), c, M, N, mpad, splits, epi);
    return e != cudaSuccess ? e : cudaGetLastError();
}

// out_dtype: 0 = f32, 2 = bf16 (fer_buffer_dtype_t codes).
extern "C" cudaError_t fer_gemm_bf16_tc(const void* a, const void* b, void* c, int M, int N, int K,
                                        uint32_t out_dtype, uint32_t* err, cudaStream_t stream) {
    if (out_dtype != 0 && out_dtype != 2) return cudaErrorInvalidValue;
    return fer_gemm_bf16_tc_ex(a, b, c, nullptr, M, N, K, out_dtype == 2 ? kEpiBF16 : kEpiF32, err, stream);
}
