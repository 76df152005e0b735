// Causal multi-head attention, head_dim 64, on the 5th-generation tensor
// cores (tcgen05), straight out of the fused QKV activation.
//
// qkv: [B*S, 3*d] bf16 row-major (q | k | v; head h at columns h*64 of each
// third); out: [B*S, d] bf16. S must be a multiple of 128.
//
// One CTA per (128-query tile, head, sequence), three CTAs per SM (64 KB of
// shared memory and 128 tensor-memory columns each). Per key block j (64
// keys, j = 0 .. 2 * query tile + 1):
//   warp 0      TMA: Q once ([128 rows x 64 bf16]), K_j and V_j into 2-deep
//               rings ([64 rows x 64 bf16]), all 128-byte swizzled boxes
//   warp 1      tcgen05.mma from one thread: S = Q K_j^T (M128 N64, f32 in
//               tensor memory), issued for block j+1 as soon as the softmax
//               threads have read block j's scores, then O += P_j V_j (M128
//               N64, K = 64 keys) once P_j is written
//   warps 2..5  one query row per thread: scores from tensor memory
//               (tcgen05.ld), causal mask on the two diagonal blocks, running
//               max in the log2 domain, p = 2^(s*scale - m) (ex2.approx), row
//               sum in f32, P rounded to bf16 into swizzled shared memory (the
//               A operand of the P.V MMA). O accumulates in tensor memory
//               across key blocks; the max a row subtracts is raised only
//               when a block's max exceeds it by more than 2^8, and then the
//               softmax thread rescales its O row in place (tcgen05.ld / st)
//               before the next P.V lands on it.
// Finally o / l is rounded to bf16 and stored. The arithmetic is the same
// online softmax as the mma.sync kernel in xfmr_kernels.cu (and the oracle's
// exp(s - max) / sum with P rounded to bf16 before P.V).
// Every wait is bounded (about one second): on timeout the kernel records an
// error bit, stops, releases tensor memory and returns. No TMA multicast.
#include "f32x2.cuh"
#include "pdl.cuh"
#include "sm100_util.cuh"
#include "tmap.cuh"

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>

namespace {

using namespace fer::dev;

constexpr int TQ = 128;                   // queries per CTA
constexpr int TK = 64;                    // keys per block
constexpr int Q_BYTES = TQ * 128;         // [128 rows x 64 bf16], 16 KiB
constexpr int KV_BYTES = TK * 128;        // [64 rows x 64 bf16], 8 KiB
constexpr int P_BYTES = TQ * TK * 2;      // [128 rows x 64 keys bf16], 16 KiB
constexpr int OFF_Q = 0;
constexpr int OFF_K = Q_BYTES;            // two K buffers
constexpr int OFF_V = OFF_K + 2 * KV_BYTES;   // two V buffers
constexpr int OFF_P = OFF_V + 2 * KV_BYTES;
constexpr int SMEM_BYTES = OFF_P + P_BYTES + 1024;
constexpr int kThreads = 192;
constexpr int kCtasPerSm = 3;
constexpr uint32_t TMEM_COLS = 128;       // S at columns [0, 64), O at [64, 128)
constexpr uint32_t COL_O = 64;
constexpr float kRescaleSlack = 8.0f;     // log2 units the subtracted max may lag the row max
static_assert(kCtasPerSm * TMEM_COLS <= 512, "tensor memory per SM");

// kind::f16 instruction descriptors: f32 accumulate, bf16 A and B, M = 128.
// S = Q K^T: A and B K-major, N = 64. O = P V: A K-major, B (V) N-major, N = 64.
constexpr uint32_t kIdescS = (1u << 4) | (1u << 7) | (1u << 10) | ((64u >> 3) << 17) | ((128u >> 4) << 24);
constexpr uint32_t kIdescPV =
    (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((64u >> 3) << 17) | ((128u >> 4) << 24);

struct Bars {
    uint64_t q_full;
    uint64_t k_full[2];
    uint64_t k_empty[2];
    uint64_t v_full[2];
    uint64_t v_empty[2];
    uint64_t s_full;
    uint64_t s_free;
    uint64_t p_full;
    uint64_t o_full;
    uint32_t tmem_base;
    int abort_flag;
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle, version 1.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= 1ull << 46;
    d |= 2ull << 61;
    return d;
}

__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

__device__ __forceinline__ void commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 64 consecutive f32 columns of this thread's TMEM lane; the wait is in the
// same asm statement, so no use of the registers can be scheduled before it.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float* v) {
    uint32_t r[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Stores 32 f32 columns to this thread's TMEM lane and waits for the store.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n\t"
        "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
        "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
        "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
        "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
        "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
        : "memory");
}

// max of three floats in one instruction (sm_100 `max.f32` with three inputs)
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t u;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(u) : "f"(hi), "f"(lo));
    return u;
}

__device__ __forceinline__ void st_shared_v4(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

// Whole-warp bounded wait: every lane polls, the warp agrees on the outcome.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity));
}

__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    attn_causal_tc(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmkv,
                   __nv_bfloat16* __restrict__ out, int S, int d, int heads, int tile_major, float scale_log2,
                   uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ Bars bars;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_addr(smem);

    // Work item of this CTA (1-D grid). Head-major (the tiles of one head on
    // consecutive CTAs, longest first, so they share K/V in L2), or, when the
    // grid is under about two waves, tile-major (every head's longest tile in
    // the first wave, the shortest ones last, so the tail is a short tile).
    const int n_qt = S / TQ;
    const int bid = static_cast<int>(blockIdx.x);
    int qt, h, bseq;
    if (tile_major) {
        const int per = static_cast<int>(gridDim.x) / n_qt;     // heads * sequences
        qt = n_qt - 1 - bid / per;
        h = (bid % per) % heads;
        bseq = (bid % per) / heads;
    } else {
        qt = n_qt - 1 - bid % n_qt;
        h = (bid / n_qt) % heads;
        bseq = (bid / n_qt) / heads;
    }
    const int seq_row0 = bseq * S;
    const int n_k = (qt + 1) * (TQ / TK);                                               // keys 0 .. end of tile
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 32) {
        prefetch_tmap(&tmq);
        prefetch_tmap(&tmkv);
    }

    if (threadIdx.x == 0) {
        mbar_init(&bars.q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars.k_full[i], 1);
            mbar_init(&bars.k_empty[i], 1);
            mbar_init(&bars.v_full[i], 1);
            mbar_init(&bars.v_empty[i], 1);
        }
        mbar_init(&bars.s_full, 1);
        mbar_init(&bars.s_free, 4);
        mbar_init(&bars.p_full, 4);
        mbar_init(&bars.o_full, 1);
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
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = bars.tmem_base;
    volatile int* abort_flag = &bars.abort_flag;
    // set-up above touches no global memory (overlaps the previous kernel
    // under programmatic launch)
    fer::dev::pdl_begin();

    if (warp == 0) {
        // ---------------- TMA producer
        if (lane == 0) {
            mbar_arrive_expect_tx(&bars.q_full, Q_BYTES);
            tma_load_2d(sbase + OFF_Q, &tmq, h * 64, seq_row0 + qt * TQ, &bars.q_full);
        }
        __syncwarp();
        for (int j = 0; j < n_k && !warp_flag(abort_flag); ++j) {
            const int st = j & 1;
            const uint32_t use = static_cast<uint32_t>(j >> 1);
            if (!warp_wait(&bars.k_empty[st], (use & 1u) ^ 1u)) {
                if (lane == 0) report(err, kErrTimeoutSync);
                *abort_flag = 1;
                break;
            }
            if (lane == 0) {
                mbar_arrive_expect_tx(&bars.k_full[st], KV_BYTES);
                tma_load_2d(sbase + OFF_K + st * KV_BYTES, &tmkv, d + h * 64, seq_row0 + j * TK, &bars.k_full[st]);
            }
            __syncwarp();
            if (!warp_wait(&bars.v_empty[st], (use & 1u) ^ 1u)) {
                if (lane == 0) report(err, kErrTimeoutSync);
                *abort_flag = 1;
                break;
            }
            if (lane == 0) {
                mbar_arrive_expect_tx(&bars.v_full[st], KV_BYTES);
                tma_load_2d(sbase + OFF_V + st * KV_BYTES, &tmkv, 2 * d + h * 64, seq_row0 + j * TK,
                            &bars.v_full[st]);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: S_{j+1} goes in as soon as the softmax
        // threads have read S_j, so it runs under their exponentials; P_j V_j
        // follows once P_j is written.
        auto issue_s = [&](int j) -> bool {
            const int st = j & 1;
            if (!warp_wait(&bars.k_full[st], static_cast<uint32_t>(j >> 1) & 1u)) return false;
            if (j > 0 && !warp_wait(&bars.s_free, static_cast<uint32_t>(j - 1) & 1u)) return false;
            fence_after();
            if (lane == 0) {
                const uint32_t q = sbase + OFF_Q, k = sbase + OFF_K + st * KV_BYTES;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk)
                    mma(tmem, sdesc(q + kk * 32, 16, 1024), sdesc(k + kk * 32, 16, 1024), kIdescS, kk ? 1u : 0u);
                commit(&bars.k_empty[st]);
                commit(&bars.s_full);
            }
            __syncwarp();
            return true;
        };
        bool ok = warp_wait(&bars.q_full, 0) && issue_s(0);
        for (int j = 0; j < n_k && ok && !warp_flag(abort_flag); ++j) {
            const uint32_t ph = static_cast<uint32_t>(j) & 1u;
            if (j + 1 < n_k && !(ok = issue_s(j + 1))) break;
            const int st = j & 1;
            ok = warp_wait(&bars.p_full, ph) && warp_wait(&bars.v_full[st], static_cast<uint32_t>(j >> 1) & 1u);
            if (!ok) break;
            fence_after();
            if (lane == 0) {
                const uint32_t p = sbase + OFF_P, v = sbase + OFF_V + st * KV_BYTES;
#pragma unroll
                for (int kk = 0; kk < TK / 16; ++kk)
                    mma(tmem + COL_O, sdesc(p + kk * 32, 16, 1024), sdesc(v + kk * 2048, KV_BYTES, 1024), kIdescPV,
                        (j | kk) ? 1u : 0u);
                commit(&bars.v_empty[st]);
                commit(&bars.o_full);
            }
            __syncwarp();
        }
        if (!ok) {
            if (lane == 0) report(err, kErrTimeoutLoad);
            *abort_flag = 1;
        }
    } else {
        // ---------------- softmax warps: one query row per thread
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;                      // row in the query tile
        const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        float m = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int j = 0; j < n_k; ++j) {
            const uint32_t ph = static_cast<uint32_t>(j) & 1u;
            if (warp_flag(abort_flag) || !warp_wait(&bars.s_full, ph)) {
                ok = false;
                break;
            }
            fence_after();
            float sv[TK];
            tmem_ld64(trow, sv);
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.s_free);   // S_{j+1} may overwrite S now
            const int kb = j * TK - qt * TQ;            // first key of the block, relative to the tile's first query
            if (kb + TK - 1 > 0) {
#pragma unroll
                for (int e = 0; e < TK; ++e)
                    if (kb + e > r) sv[e] = -INFINITY;          // causal mask on the diagonal blocks
            }
            // block max with the three-input max of sm_100 (exact, so the
            // grouping does not matter): 31 instructions for 64 scores
            float mx[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) mx[e] = sv[e];
#pragma unroll
            for (int e = 8; e < TK; e += 2) mx[(e >> 1) & 7] = max3f(mx[(e >> 1) & 7], sv[e], sv[e + 1]);
            const float smax = max3f(max3f(mx[0], mx[1], mx[2]), max3f(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
            // The subtracted max is raised only when the block's max exceeds
            // it by more than kRescaleSlack (log2 units, so p <= 256):
            // softmax does not depend on the constant subtracted, and O is
            // then rescaled a few times per row instead of whenever the max
            // grows (always on the first block with a key).
            const float bmax = smax * scale_log2;
            const bool raise = bmax > m + kRescaleSlack;
            const float m_new = raise ? bmax : m;
            const float alpha = raise ? ex2(m - m_new) : 1.0f;   // 0 while m is -inf
            // P_{j-1} V_{j-1} done: P's buffer is free and O holds every
            // earlier block
            if (j > 0 && !warp_wait(&bars.o_full, ph ^ 1u)) {
                ok = false;
                break;
            }
            fence_after();
            // p = 2^(s*scale - m_new), row sum, P (bf16) into shared memory
            // on packed pairs: s*scale - m_new is one fma per element and the
            // eight row-sum accumulators are four pairs, each element added
            // to the same accumulator in the same order as the scalar form,
            // so the bits are those of fmaf / scalar adds
            uint64_t sm2[4] = {0, 0, 0, 0};
            const uint64_t sc2 = f2_splat(scale_log2), nm2 = f2_splat(-m_new);
#pragma unroll
            for (int c = 0; c < TK / 32; ++c) {
                uint32_t w[16];
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    float t0, t1;
                    f2_unpack(f2_fma(f2_pack(sv[c * 32 + e], sv[c * 32 + e + 1]), sc2, nm2), t0, t1);
                    const float p0 = ex2(t0), p1 = ex2(t1);
                    sm2[(e >> 1) & 3] = f2_add(sm2[(e >> 1) & 3], f2_pack(p0, p1));
                    w[e >> 1] = pack_bf16x2(p0, p1);
                }
                const uint32_t prow = sbase + OFF_P + r * 128;
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const int chunk = (c & 1) * 4 + q4;
                    st_shared_v4(prow + ((chunk ^ (r & 7)) << 4), w[4 * q4], w[4 * q4 + 1], w[4 * q4 + 2],
                                 w[4 * q4 + 3]);
                }
            }
            float sm[8];
#pragma unroll
            for (int k = 0; k < 4; ++k) f2_unpack(sm2[k], sm[2 * k], sm[2 * k + 1]);
            const float sum = ((sm[0] + sm[1]) + (sm[2] + sm[3])) + ((sm[4] + sm[5]) + (sm[6] + sm[7]));
            // O holds sum_{i<j} P_i V_i scaled by 2^-m: rescale it in place
            // before P_j V_j accumulates on it.
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
                for (int c = 0; c < 2; ++c) {
                    float ov[32];
                    tmem_ld32(trow + COL_O + c * 32, ov);
                    const uint64_t a2 = f2_splat(alpha);
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        float o0, o1;
                        f2_unpack(f2_mul(f2_pack(ov[e], ov[e + 1]), a2), o0, o1);
                        ov[e] = o0;
                        ov[e + 1] = o1;
                    }
                    tmem_st32(trow + COL_O + c * 32, ov);
                }
            }
            l = l * alpha + sum;
            m = m_new;
            fence_proxy_async_smem();   // P is read by the tensor core (async proxy)
            fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.p_full);
        }
        if (ok && !warp_wait(&bars.o_full, static_cast<uint32_t>(n_k - 1) & 1u)) ok = false;
        if (!ok) {
            if (lane == 0) report(err, kErrTimeoutMma);
            *abort_flag = 1;
        } else {
            fence_after();
            float o[64];
            tmem_ld64(trow + COL_O, o);
            const float inv = 1.0f / l;
            uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(seq_row0 + qt * TQ + r) * d + h * 64);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint4 u;
                u.x = pack_bf16x2(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
                u.y = pack_bf16x2(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
                u.z = pack_bf16x2(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
                u.w = pack_bf16x2(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
                dst[c] = u;
            }
        }
    }

    fence_before();
    __syncthreads();
    if (warp == 1) {
        fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
    }
}

using fer::host::EncodeTiledFn;

EncodeTiledFn encode_fn() { return fer::host::encode_tiled_fn(); }

}  // namespace

// Returns cudaErrorNotSupported (launching nothing) for shapes this kernel
// does not take: head_dim != 64, S % 128 != 0, misaligned qkv / out.
extern "C" cudaError_t fer_attn_causal_tc(const void* qkv, void* out, int B, int S, int d, int heads, uint32_t* err,
                                          cudaStream_t stream) {
    if (B <= 0 || S <= 0 || heads <= 0 || d != heads * 64 || (S % TQ) != 0) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(out)) & 15u) return cudaErrorNotSupported;
    EncodeTiledFn fn = encode_fn();
    if (!fn) return cudaErrorNotSupported;
    // two maps over qkv [B*S, 3d]: Q boxes of 128 rows, K / V boxes of 64
    CUtensorMap tmq, tmkv;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(3) * d, static_cast<cuuint64_t>(B) * S};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(3) * d * 2};
    const cuuint32_t boxq[2] = {64, TQ}, boxkv[2] = {64, TK};
    const cuuint32_t estr[2] = {1, 1};
    if (fn(&tmq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(qkv), dims, strides, boxq, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
        fn(&tmkv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(qkv), dims, strides, boxkv, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return cudaErrorNotSupported;
    static const cudaError_t attr_rc =
        cudaFuncSetAttribute(attn_causal_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (attr_rc != cudaSuccess) return attr_rc;
    const float scale_log2 = 1.4426950408889634f / 8.0f;   // log2(e) / sqrt(64)
    const long long ctas = static_cast<long long>(S / TQ) * heads * B;
    if (ctas > 0x7fffffffll) return cudaErrorNotSupported;
    static const int sms = [] {
        int dev = 0, v = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v > 0 ? v : 148;
    }();
    const int tile_major = ctas <= 2ll * kCtasPerSm * sms ? 1 : 0;
    const dim3 grid(static_cast<unsigned>(ctas));
    static const bool pdl = [] {   // as the GEMM: off with FERCUDA_GEMM_PDL=0 (launch_pdl honours FERCUDA_PDL)
        const char* e = std::getenv("FERCUDA_GEMM_PDL");
        return !(e && e[0] == '0');
    }();
    if (pdl) {
        const cudaError_t e = fer::host::launch_pdl(attn_causal_tc, grid, dim3(kThreads), SMEM_BYTES, stream, tmq, tmkv,
                                                    static_cast<__nv_bfloat16*>(out), S, d, heads, tile_major,
                                                    scale_log2, err);
        return e != cudaSuccess ? e : cudaGetLastError();
    }
    fer_pdl_note_launch();   // the kernel triggers its dependents under either launch
    attn_causal_tc<<<grid, kThreads, SMEM_BYTES, stream>>>(tmq, tmkv, static_cast<__nv_bfloat16*>(out), S, d, heads,
                                                           tile_major, scale_log2, err);
    return cudaGetLastError();
}
