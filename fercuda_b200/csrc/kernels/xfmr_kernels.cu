// Kernels of the decoder-only transformer forward (pre-LN block: LN -> QKV ->
// causal attention -> out-proj + residual -> LN -> W1 + GELU -> W2 + residual;
// final LN and LM head). The block structure follows the reference's
// transformer (rust/deps/ferrite-torch/examples/transformer_demo.rs:18-70,
// computed there by libtorch); the GEMMs run on gemm_tc.cu.
//
//   fill_normal_bf16   seeded weight init on the device (counter-based
//                      splitmix64 + Box-Muller, bit-identical to the host
//                      generator), so a 333 MB model is made in milliseconds
//                      and only rank 0's copy is broadcast
//   embed_f32          token rows of the bf16 embedding -> f32 residual stream
//   embed_ln_bf16      the same rows and, in the same pass, the first layer's
//                      layer norm of them (one launch instead of two)
//   ln_bf16            per-token layer norm, f32 in, bf16 out (GEMM operand)
//   attn_causal        causal multi-head attention for head_dim 64 straight out
//                      of the fused QKV activation [tokens, 3*d]; flash-style
//                      (online softmax, no score matrix in HBM), one CTA per
//                      (128 queries, head, sequence), bf16 tensor-core MMAs
//                      (mma.sync m16n8k16) fed by ldmatrix from swizzled
//                      shared tiles, K/V double-buffered with cp.async
#include "pdl.cuh"
#include "sm100_util.cuh"

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace {

using bf16 = __nv_bfloat16;

// ------------------------------------------------------------------ init

__device__ __forceinline__ uint64_t splitmix_draw(uint64_t seed, uint64_t k) {
    uint64_t z = seed + k * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Box-Muller on draws 2i+1 and 2i+2 of the seed's stream for element i, with
// ln and cos as fixed series evaluated by IEEE double +, -, *, /, sqrt, each
// an explicit round-to-nearest intrinsic (no contraction into FMA), so the
// bits equal the host generator's (fercuda_b200/synth.py normal_bf16) on any
// IEEE machine that takes the same steps.
//   ln(k 2^-53), 1 <= k <= 2^53: k = f 2^b, f in [sqrt(1/2), sqrt(2));
//     ln = (b - 53) ln2 + 2 s P(s^2), s = (f - 1) / (f + 1), P the atanh series
//   cos(2 pi k 2^-53), 0 <= k < 2^53: octant q = k >> 50, offset r (exact),
//     odd octants take 1/8 - r; x = 2 pi r in [0, pi/4]; sin or cos series
__constant__ double kLnSeries[11] = {
    0x1.0000000000000p+0, 0x1.5555555555555p-2, 0x1.999999999999ap-3, 0x1.2492492492492p-3,
    0x1.c71c71c71c71cp-4, 0x1.745d1745d1746p-4, 0x1.3b13b13b13b14p-4, 0x1.1111111111111p-4,
    0x1.e1e1e1e1e1e1ep-5, 0x1.af286bca1af28p-5, 0x1.8618618618618p-5};
__constant__ double kSinSeries[9] = {
    0x1.0000000000000p+0, -0x1.5555555555555p-3, 0x1.1111111111111p-7, -0x1.a01a01a01a01ap-13,
    0x1.71de3a556c734p-19, -0x1.ae64567f544e4p-26, 0x1.6124613a86d09p-33, -0x1.ae7f3e733b81fp-41,
    0x1.952c77030ad4ap-49};
__constant__ double kCosSeries[10] = {
    0x1.0000000000000p+0, -0x1.0000000000000p-1, 0x1.5555555555555p-5, -0x1.6c16c16c16c17p-10,
    0x1.a01a01a01a01ap-16, -0x1.27e4fb7789f5cp-22, 0x1.1eed8eff8d898p-29, -0x1.93974a8c07c9dp-37,
    0x1.ae7f3e733b81fp-45, -0x1.6827863b97d97p-53};
constexpr double kLn2 = 0x1.62e42fefa39efp-1;
constexpr double kTwoPi = 0x1.921fb54442d18p+2;
constexpr double kSqrtHalf = 0x1.6a09e667f3bcdp-1;

template <int N>
__device__ __forceinline__ double horner(const double (&c)[N], double t) {
    double p = c[N - 1];
#pragma unroll
    for (int k = N - 2; k >= 0; --k) p = __dadd_rn(__dmul_rn(p, t), c[k]);
    return p;
}

__device__ __forceinline__ double portable_ln(uint64_t k) {
    const long long bits = __double_as_longlong(__ull2double_rn(k));      // exact: k <= 2^53
    double e = static_cast<double>(static_cast<int>((bits >> 52) & 0x7ff) - 1075);
    double f = __longlong_as_double((bits & 0x000fffffffffffffll) | (1022ll << 52));   // [0.5, 1)
    if (f < kSqrtHalf) {
        f = __dmul_rn(f, 2.0);
        e = __dadd_rn(e, -1.0);
    }
    const double s = __ddiv_rn(__dadd_rn(f, -1.0), __dadd_rn(f, 1.0));
    const double p = horner(kLnSeries, __dmul_rn(s, s));
    return __dadd_rn(__dmul_rn(e, kLn2), __dmul_rn(__dmul_rn(2.0, s), p));
}

__device__ __forceinline__ double portable_cos_turns(uint64_t k) {
    const int q = static_cast<int>(k >> 50);
    double r = __dmul_rn(__ull2double_rn(k & ((1ull << 50) - 1)), 0x1p-53);
    if (q & 1) r = __dadd_rn(0.125, -r);
    const double x = __dmul_rn(kTwoPi, r);
    const double x2 = __dmul_rn(x, x);
    const bool use_cos = q == 0 || q == 3 || q == 4 || q == 7;
    const double v = use_cos ? horner(kCosSeries, x2) : __dmul_rn(x, horner(kSinSeries, x2));
    return (q >= 2 && q <= 5) ? -v : v;
}

__global__ void fill_normal_bf16(bf16* out, size_t n, uint64_t seed, float stddev) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const double sd = static_cast<double>(stddev);
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t d0 = splitmix_draw(seed, 2 * i + 1), d1 = splitmix_draw(seed, 2 * i + 2);
        const double z = __dmul_rn(__dsqrt_rn(__dmul_rn(-2.0, portable_ln((d0 >> 11) + 1))),
                                   portable_cos_turns(d1 >> 11));
        // mean 0 added as the host does (turns a -0 product into +0)
        out[i] = __float2bfloat16_rn(__double2float_rn(__dadd_rn(0.0, __dmul_rn(sd, z))));
    }
}

__global__ void fill_f32(float* out, size_t n, float v) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) out[i] = v;
}

// ------------------------------------------------------------------ embedding

// One warp per token; d % 256 == 0.
__global__ void embed_f32(const int* __restrict__ tok, const bf16* __restrict__ emb, float* __restrict__ x, int T,
                          int d, int vocab, uint32_t* err) {
    fer::dev::pdl_begin();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const int id = tok[warp];
    float* row = x + static_cast<size_t>(warp) * d;
    if (id < 0 || id >= vocab) {
        if (lane == 0) fer::dev::report(err, fer::dev::kErrBadShape);
        for (int c = lane * 4; c < d; c += 128) *reinterpret_cast<float4*>(row + c) = make_float4(0.f, 0.f, 0.f, 0.f);
        return;
    }
    const bf16* src = emb + static_cast<size_t>(id) * d;
    for (int c = lane * 8; c < d; c += 256) {
        const uint4 v = *reinterpret_cast<const uint4*>(src + c);
        const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
        float2 f0 = __bfloat1622float2(p[0]), f1 = __bfloat1622float2(p[1]);
        float2 f2 = __bfloat1622float2(p[2]), f3 = __bfloat1622float2(p[3]);
        *reinterpret_cast<float4*>(row + c) = make_float4(f0.x, f0.y, f1.x, f1.y);
        *reinterpret_cast<float4*>(row + c + 4) = make_float4(f2.x, f2.y, f3.x, f3.y);
    }
}

// ------------------------------------------------------------------ layer norm

// One warp per row, d % 128 == 0 and d <= 4096: two-pass mean / variance
// over values held in registers, out = (x - mean) * rsqrt(var + eps) * g + b.
template <int VPL>   // float4 vectors per lane = d / 128
__global__ void ln_bf16(const float* __restrict__ x, const float* __restrict__ g, const float* __restrict__ b,
                        bf16* __restrict__ out, int T, int d, float eps) {
    fer::dev::pdl_begin();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const float* row = x + static_cast<size_t>(warp) * d;
    float4 v[VPL];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        v[i] = *reinterpret_cast<const float4*>(row + (i * 32 + lane) * 4);
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / static_cast<float>(d);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, e = v[i].w - mean;
        q += (a * a + bb * bb) + (c * c + e * e);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float inv = rsqrtf(q / static_cast<float>(d) + eps);
    bf16* orow = out + static_cast<size_t>(warp) * d;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c = (i * 32 + lane) * 4;
        const float4 gg = *reinterpret_cast<const float4*>(g + c);
        const float4 bb = *reinterpret_cast<const float4*>(b + c);
        __nv_bfloat162 p0 = __floats2bfloat162_rn((v[i].x - mean) * inv * gg.x + bb.x, (v[i].y - mean) * inv * gg.y + bb.y);
        __nv_bfloat162 p1 = __floats2bfloat162_rn((v[i].z - mean) * inv * gg.z + bb.z, (v[i].w - mean) * inv * gg.w + bb.w);
        uint2 w;
        w.x = *reinterpret_cast<uint32_t*>(&p0);
        w.y = *reinterpret_cast<uint32_t*>(&p1);
        *reinterpret_cast<uint2*>(orow + c) = w;
    }
}

// Token embedding and the first layer's layer norm in one pass: one warp per
// token writes the f32 residual row (the bf16 embedding row upcast, exactly
// what embed_f32 writes) and its layer norm (the arithmetic of ln_bf16, on
// the same values in the same lanes, so the same bits).
template <int VPL>
__global__ void embed_ln_bf16(const int* __restrict__ tok, const bf16* __restrict__ emb, float* __restrict__ x,
                              const float* __restrict__ g, const float* __restrict__ b, bf16* __restrict__ out, int T,
                              int d, int vocab, float eps, uint32_t* err) {
    fer::dev::pdl_begin();
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= T) return;
    const int id = tok[warp];
    const bool bad = id < 0 || id >= vocab;
    if (bad && lane == 0) fer::dev::report(err, fer::dev::kErrBadShape);
    const bf16* src = emb + static_cast<size_t>(bad ? 0 : id) * d;
    float* row = x + static_cast<size_t>(warp) * d;
    float4 v[VPL];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c = (i * 32 + lane) * 4;
        const uint2 u = *reinterpret_cast<const uint2*>(src + c);
        const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
        const float2 f0 = __bfloat1622float2(p[0]), f1 = __bfloat1622float2(p[1]);
        v[i] = bad ? make_float4(0.f, 0.f, 0.f, 0.f) : make_float4(f0.x, f0.y, f1.x, f1.y);
        *reinterpret_cast<float4*>(row + c) = v[i];
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / static_cast<float>(d);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, e = v[i].w - mean;
        q += (a * a + bb * bb) + (c * c + e * e);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float inv = rsqrtf(q / static_cast<float>(d) + eps);
    bf16* orow = out + static_cast<size_t>(warp) * d;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c = (i * 32 + lane) * 4;
        const float4 gg = *reinterpret_cast<const float4*>(g + c);
        const float4 bb = *reinterpret_cast<const float4*>(b + c);
        __nv_bfloat162 p0 = __floats2bfloat162_rn((v[i].x - mean) * inv * gg.x + bb.x, (v[i].y - mean) * inv * gg.y + bb.y);
        __nv_bfloat162 p1 = __floats2bfloat162_rn((v[i].z - mean) * inv * gg.z + bb.z, (v[i].w - mean) * inv * gg.w + bb.w);
        uint2 w;
        w.x = *reinterpret_cast<uint32_t*>(&p0);
        w.y = *reinterpret_cast<uint32_t*>(&p1);
        *reinterpret_cast<uint2*>(orow + c) = w;
    }
}

// ------------------------------------------------------------------ attention

constexpr int AM = 128;   // queries per CTA (8 warps x 16)
constexpr int AN = 64;    // keys per block
constexpr int HD = 64;    // head dim
constexpr int kAttnThreads = 256;

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in a [rows][64 bf16]
// tile; the chunk index is XOR-swizzled with the row so that ldmatrix reads
// of 8 rows at one column hit 8 different bank groups.
__device__ __forceinline__ uint32_t swz(int r, int c) { return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    const int n = valid ? 16 : 0;   // 0 source bytes: the 16 destination bytes are zero-filled
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&p);
}

// qkv: [B*S, 3*d] bf16 (q | k | v, head h at columns h*64 of each third);
// out: [B*S, d] bf16. grid = (ceil(S/128), heads, B).
__global__ void __launch_bounds__(kAttnThreads) attn_causal(const bf16* __restrict__ qkv, bf16* __restrict__ out, int S,
                                                           int d, float scale_log2) {
    __shared__ __align__(128) uint8_t sQ[AM * 128];
    __shared__ __align__(128) uint8_t sK[2 * AN * 128];
    __shared__ __align__(128) uint8_t sV[2 * AN * 128];

    const int nqb = gridDim.x;
    const int qb = nqb - 1 - static_cast<int>(blockIdx.x);   // longest (last) query blocks first
    const int h = blockIdx.y, bseq = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t ld = static_cast<size_t>(3) * d;
    const bf16* base = qkv + static_cast<size_t>(bseq) * S * ld;
    const int q0 = qb * AM;
    const int q_last = (q0 + AM < S ? q0 + AM : S) - 1;
    const int nkb = q_last / AN + 1;

    const uint32_t sq = fer::dev::smem_addr(sQ);
    const uint32_t sk0 = fer::dev::smem_addr(sK), sv0 = fer::dev::smem_addr(sV);
    constexpr uint32_t kTile = AN * 128;

    for (int i = tid; i < AM * 8; i += kAttnThreads) {
        const int r = i >> 3, c = i & 7, t = q0 + r;
        cp_async16(sq + swz(r, c), base + static_cast<size_t>(t < S ? t : 0) * ld + h * HD + c * 8, t < S);
    }
    auto load_kv = [&](int kb, int bi) {
        for (int i = tid; i < AN * 8; i += kAttnThreads) {
            const int r = i >> 3, c = i & 7, t = kb * AN + r;
            const bf16* src = base + static_cast<size_t>(t < S ? t : 0) * ld + h * HD + c * 8;
            cp_async16(sk0 + bi * kTile + swz(r, c), src + d, t < S);
            cp_async16(sv0 + bi * kTile + swz(r, c), src + 2 * d, t < S);
        }
    };
    load_kv(0, 0);
    cp_async_commit();

    uint32_t qf[4][4];
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float m_i[2] = {-INFINITY, -INFINITY}, l_i[2] = {0.0f, 0.0f};
    const int row0 = q0 + warp * 16 + (lane >> 2);   // rows of c0/c1; c2/c3 are row0 + 8

    for (int kb = 0; kb < nkb; ++kb) {
        const int bi = kb & 1;
        if (kb + 1 < nkb) {
            load_kv(kb + 1, bi ^ 1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (kb == 0) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
                ldsm_x4(qf[kk], sq + swz(warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1), 2 * kk + (lane >> 4)));
        }
        // S = Q K^T for this warp's 16 queries x 64 keys
        float s[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {
                uint32_t kf[4];
                ldsm_x4(kf, sk0 + bi * kTile + swz(16 * jp + (lane & 7) + 8 * (lane >> 4), 2 * kk + ((lane >> 3) & 1)));
                mma16816(s[2 * jp], qf[kk], kf[0], kf[1]);
                mma16816(s[2 * jp + 1], qf[kk], kf[2], kf[3]);
            }
        // scale (log2 domain) and causal mask
        const int key0 = kb * AN + 2 * (lane & 3);
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = key0 + 8 * j + (e & 1);
                const int row = row0 + 8 * (e >> 1);
                const float v = s[j][e] * scale_log2;
                s[j][e] = (key > row || key >= S) ? -INFINITY : v;
            }
        float mx[2] = {m_i[0], m_i[1]};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            mx[0] = fmaxf(mx[0], fmaxf(s[j][0], s[j][1]));
            mx[1] = fmaxf(mx[1], fmaxf(s[j][2], s[j][3]));
        }
        float alpha[2], rs[2] = {0.0f, 0.0f};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
            alpha[r] = (mx[r] == -INFINITY) ? 1.0f : exp2f(m_i[r] - mx[r]);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float m = mx[e >> 1];
                const float p = (m == -INFINITY) ? 0.0f : exp2f(s[j][e] - m);
                s[j][e] = p;
                rs[e >> 1] += p;
            }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
            rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
            l_i[r] = l_i[r] * alpha[r] + rs[r];
            m_i[r] = mx[r];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            o[j][0] *= alpha[0];
            o[j][1] *= alpha[0];
            o[j][2] *= alpha[1];
            o[j][3] *= alpha[1];
        }
        // O += P V
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint32_t pa[4] = {pack_bf16(s[2 * kk][0], s[2 * kk][1]), pack_bf16(s[2 * kk][2], s[2 * kk][3]),
                                    pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]),
                                    pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
            for (int jp = 0; jp < 4; ++jp) {
                uint32_t vf[4];
                ldsm_x4_t(vf, sv0 + bi * kTile + swz(16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1), 2 * jp + (lane >> 4)));
                mma16816(o[2 * jp], pa, vf[0], vf[1]);
                mma16816(o[2 * jp + 1], pa, vf[2], vf[3]);
            }
        }
        __syncthreads();   // everyone is done with buffer bi before it is refilled
    }
    const float inv0 = l_i[0] > 0.0f ? 1.0f / l_i[0] : 0.0f;
    const float inv1 = l_i[1] > 0.0f ? 1.0f / l_i[1] : 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int col = h * HD + 8 * j + 2 * (lane & 3);
        if (row0 < S)
            *reinterpret_cast<uint32_t*>(out + (static_cast<size_t>(bseq) * S + row0) * d + col) =
                pack_bf16(o[j][0] * inv0, o[j][1] * inv0);
        if (row0 + 8 < S)
            *reinterpret_cast<uint32_t*>(out + (static_cast<size_t>(bseq) * S + row0 + 8) * d + col) =
                pack_bf16(o[j][2] * inv1, o[j][3] * inv1);
    }
}

unsigned grid_cap(size_t n, unsigned per) {
    size_t g = (n + per - 1) / per;
    if (g > 148u * 32u) g = 148u * 32u;
    return static_cast<unsigned>(g ? g : 1);
}

}  // namespace

extern "C" cudaError_t fer_fill_normal_bf16(void* out, size_t n, uint64_t seed, float stddev, cudaStream_t s) {
    fill_normal_bf16<<<grid_cap(n, 256), 256, 0, s>>>(static_cast<bf16*>(out), n, seed, stddev);
    return cudaGetLastError();
}

extern "C" cudaError_t fer_fill_f32(float* out, size_t n, float v, cudaStream_t s) {
    fill_f32<<<grid_cap(n, 256), 256, 0, s>>>(out, n, v);
    return cudaGetLastError();
}

extern "C" cudaError_t fer_embed_f32(const int* tok, const void* emb, float* x, int T, int d, int vocab, uint32_t* err,
                                     cudaStream_t s) {
    if (d % 256) return cudaErrorInvalidValue;
    const int warps_per_block = 8;
    const cudaError_t e = fer::host::launch_pdl(embed_f32, dim3((T + warps_per_block - 1) / warps_per_block),
                                                dim3(32 * warps_per_block), 0, s, tok, static_cast<const bf16*>(emb),
                                                x, T, d, vocab, err);
    return e != cudaSuccess ? e : cudaGetLastError();
}

extern "C" cudaError_t fer_ln_bf16(const float* x, const float* g, const float* b, void* out, int T, int d, float eps,
                                   cudaStream_t s) {
    const int wpb = 8;
    const dim3 grid((T + wpb - 1) / wpb), block(32 * wpb);
    bf16* o = static_cast<bf16*>(out);
    cudaError_t e = cudaSuccess;
    switch (d / 128) {
        case 1: if (d == 128) { e = fer::host::launch_pdl(ln_bf16<1>, grid, block, 0, s, x, g, b, o, T, d, eps); break; } return cudaErrorInvalidValue;
        case 2: if (d == 256) { e = fer::host::launch_pdl(ln_bf16<2>, grid, block, 0, s, x, g, b, o, T, d, eps); break; } return cudaErrorInvalidValue;
        case 4: if (d == 512) { e = fer::host::launch_pdl(ln_bf16<4>, grid, block, 0, s, x, g, b, o, T, d, eps); break; } return cudaErrorInvalidValue;
        case 8: if (d == 1024) { e = fer::host::launch_pdl(ln_bf16<8>, grid, block, 0, s, x, g, b, o, T, d, eps); break; } return cudaErrorInvalidValue;
        case 16: if (d == 2048) { e = fer::host::launch_pdl(ln_bf16<16>, grid, block, 0, s, x, g, b, o, T, d, eps); break; } return cudaErrorInvalidValue;
        case 32: if (d == 4096) { e = fer::host::launch_pdl(ln_bf16<32>, grid, block, 0, s, x, g, b, o, T, d, eps); break; } return cudaErrorInvalidValue;
        default: return cudaErrorInvalidValue;
    }
    return e != cudaSuccess ? e : cudaGetLastError();
}

extern "C" cudaError_t fer_embed_ln_bf16(const int* tok, const void* emb, float* x, const float* g, const float* b,
                                         void* out, int T, int d, int vocab, float eps, uint32_t* err,
                                         cudaStream_t s) {
    const int wpb = 8;
    const dim3 grid((T + wpb - 1) / wpb), block(32 * wpb);
    const bf16* em = static_cast<const bf16*>(emb);
    bf16* o = static_cast<bf16*>(out);
    cudaError_t e = cudaSuccess;
    switch (d) {
        case 256: e = fer::host::launch_pdl(embed_ln_bf16<2>, grid, block, 0, s, tok, em, x, g, b, o, T, d, vocab, eps, err); break;
        case 512: e = fer::host::launch_pdl(embed_ln_bf16<4>, grid, block, 0, s, tok, em, x, g, b, o, T, d, vocab, eps, err); break;
        case 1024: e = fer::host::launch_pdl(embed_ln_bf16<8>, grid, block, 0, s, tok, em, x, g, b, o, T, d, vocab, eps, err); break;
        case 2048: e = fer::host::launch_pdl(embed_ln_bf16<16>, grid, block, 0, s, tok, em, x, g, b, o, T, d, vocab, eps, err); break;
        case 4096: e = fer::host::launch_pdl(embed_ln_bf16<32>, grid, block, 0, s, tok, em, x, g, b, o, T, d, vocab, eps, err); break;
        default: return cudaErrorInvalidValue;
    }
    return e != cudaSuccess ? e : cudaGetLastError();
}

// Causal attention for head_dim 64; B sequences of S tokens; qkv [B*S, 3d].
extern "C" cudaError_t fer_attn_causal_tc(const void* qkv, void* out, int B, int S, int d, int heads, uint32_t* err,
                                          cudaStream_t stream);

// flags bit 0: use the mma.sync kernel even where the tcgen05 kernel
// (attn_tc.cu: S a multiple of 128) applies. err: device error word for the
// tcgen05 kernel's bounded waits (may be null).
extern "C" cudaError_t fer_attn_causal_ex(const void* qkv, void* out, int B, int S, int d, int heads, int flags,
                                          uint32_t* err, cudaStream_t s) {
    if (d != heads * HD || B <= 0 || S <= 0) return cudaErrorInvalidValue;
    if (!(flags & 1)) {
        const cudaError_t e = fer_attn_causal_tc(qkv, out, B, S, d, heads, err, s);
        if (e != cudaErrorNotSupported) return e;
    }
    const float scale_log2 = 1.4426950408889634f / sqrtf(static_cast<float>(HD));
    const dim3 grid((S + AM - 1) / AM, heads, B);
    attn_causal<<<grid, kAttnThreads, 0, s>>>(static_cast<const bf16*>(qkv), static_cast<bf16*>(out), S, d, scale_log2);
    return cudaGetLastError();
}

extern "C" cudaError_t fer_attn_causal(const void* qkv, void* out, int B, int S, int d, int heads, cudaStream_t s) {
    return fer_attn_causal_ex(qkv, out, B, S, d, heads, 0, nullptr, s);
}
