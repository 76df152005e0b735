/*
 * ORACLE — test infrastructure only (see oracle.h). CPU restatement of the
 * reference algorithms; built with -O2 -ffp-contract=off -fno-fast-math.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ threads */

typedef void (*orc_range_fn)(void* ctx, size_t lo, size_t hi);
typedef struct { orc_range_fn fn; void* ctx; size_t lo, hi; } orc_job;

static void* orc_job_main(void* p) {
    orc_job* j = (orc_job*)p;
    j->fn(j->ctx, j->lo, j->hi);
    return NULL;
}

/* Splits [0, n) into `threads` contiguous ranges and runs fn on each. */
static void orc_parallel(orc_range_fn fn, void* ctx, size_t n, int threads) {
    if (threads <= 1 || n < 2) { fn(ctx, 0, n); return; }
    if ((size_t)threads > n) threads = (int)n;
    pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
    orc_job* jobs = (orc_job*)malloc(sizeof(orc_job) * (size_t)threads);
    for (int t = 0; t < threads; ++t) {
        jobs[t].fn = fn;
        jobs[t].ctx = ctx;
        jobs[t].lo = n * (size_t)t / (size_t)threads;
        jobs[t].hi = n * (size_t)(t + 1) / (size_t)threads;
        pthread_create(&tid[t], NULL, orc_job_main, &jobs[t]);
    }
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
    free(tid);
    free(jobs);
}

/* ------------------------------------------------------ fused elementwise */

typedef struct { const float* x; float* y; float a, b; } chain_ctx;

/* Reference chain for y = relu(a*x+b) * sigmoid(x), one rounding per kernel:
 *   k_affine_f32  native/core/kernels/modules/tensor_kernels_ops_core.inl:375-381  t = x*a + b
 *   k_relu_f32    tensor_kernels_ops_core.inl:257-262                              r = fmaxf(0, t)
 *   k_sigmoid_f32 tensor_kernels_ops_core.inl:308-313                              s = 1/(1+expf(-x))
 *   k_mul_f32     tensor_kernels_ops_core.inl:21-27                                y = r*s
 * (the reference builds these with -fmad=false, CMakeLists.txt:57-62). */
static void chain_range(void* p, size_t lo, size_t hi) {
    const chain_ctx* c = (const chain_ctx*)p;
    for (size_t i = lo; i < hi; ++i) {
        const float x = c->x[i];
        float t = x * c->a;
        t = t + c->b;
        const float r = fmaxf(0.0f, t);
        const float s = 1.0f / (1.0f + expf(-x));
        c->y[i] = r * s;
    }
}

void orc_chain_f32(const float* x, float* y, size_t n, float a, float b, int threads) {
    chain_ctx c = {x, y, a, b};
    orc_parallel(chain_range, &c, n, threads);
}

/* JIT affine intent kernel, native/core/jit/intent/intent_runtime.cpp:58-68:
 * `alpha * in[i] + beta`, compiled by the reference's NVRTC call
 * (native/core/jit/jit_manager.cu:379-391) with FMA contraction left on, so
 * one fused multiply-add; relu as `v < 0 ? 0 : v`. */
void orc_affine_intent_f32(const float* x, float* y, size_t n, float alpha, float beta, int relu) {
    for (size_t i = 0; i < n; ++i) {
        float v = fmaf(alpha, x[i], beta);
        if (relu && v < 0.0f) v = 0.0f;
        y[i] = v;
    }
}

/* ------------------------------------------------------------ row softmax */

#define ORC_BLOCK 256
#define ORC_WARP 32

typedef float (*orc_op)(float, float);
static float op_max(float a, float b) { return fmaxf(a, b); }
static float op_add(float a, float b) { return a + b; }

/* __shfl_down_sync tree over one warp as in warp_reduce_{sum,max}_f32,
 * tensor_kernels_ops_core.inl:486-498: at each offset, lane l combines its
 * value with lane l+off (lanes past the warp read their own value). Returns
 * lane 0's result. */
static float warp_tree(const float* lanes, orc_op op) {
    float v[ORC_WARP], nv[ORC_WARP];
    memcpy(v, lanes, sizeof(v));
    for (int off = ORC_WARP / 2; off > 0; off /= 2) {
        for (int l = 0; l < ORC_WARP; ++l) nv[l] = op(v[l], (l + off < ORC_WARP) ? v[l + off] : v[l]);
        memcpy(v, nv, sizeof(v));
    }
    return v[0];
}

/* Block reduction of k_softmax_f32 (tensor_kernels_ops_core.inl:746-770 for
 * max, :781-803 for sum): warp trees, lane 0 of each warp stores its result,
 * then warp 0 runs the tree again over the 8 warp results padded with `pad`. */
static float block_reduce_256(const float* per_thread, orc_op op, float pad) {
    float warp_res[ORC_WARP];
    const int nwarps = ORC_BLOCK / ORC_WARP;
    for (int w = 0; w < ORC_WARP; ++w) warp_res[w] = pad;
    for (int w = 0; w < nwarps; ++w) warp_res[w] = warp_tree(per_thread + w * ORC_WARP, op);
    return warp_tree(warp_res, op);
}

/* k_softmax_f32, tensor_kernels_ops_core.inl:733-808, launched with 256
 * threads per row (ptx_tensor_softmax_f32, tensor_kernels_indexing_scan.inl:391-394). */
static void softmax_row(const float* in, float* out, size_t dim) {
    float part[ORC_BLOCK];
    for (int t = 0; t < ORC_BLOCK; ++t) {
        float m = -INFINITY;
        for (size_t i = (size_t)t; i < dim; i += ORC_BLOCK) m = fmaxf(m, in[i]);
        part[t] = m;
    }
    const float mx = block_reduce_256(part, op_max, -INFINITY);
    for (int t = 0; t < ORC_BLOCK; ++t) {
        float s = 0.0f;
        for (size_t i = (size_t)t; i < dim; i += ORC_BLOCK) {
            const float e = expf(in[i] - mx);
            out[i] = e;
            s += e;
        }
        part[t] = s;
    }
    const float sum = block_reduce_256(part, op_add, 0.0f);
    const float inv = 1.0f / sum;
    for (size_t i = 0; i < dim; ++i) out[i] *= inv;
}

/* k_layer_norm_f32, src/runtime/ops_bridge.cu:33-59, launched by
 * fer::ops::layer_norm (ops_bridge.cu:100-104) with T = min(n, 256) threads:
 * strided per-thread sums, then the shared-memory halving tree
 * `for (s = T/2; s > 0; s >>= 1) sdata[t] += sdata[t+s]` (which, as in the
 * reference, only covers all T partials when T is a power of two). */
static float halving_tree(float* sdata, int T) {
    for (int s = T / 2; s > 0; s >>= 1)
        for (int t = 0; t < s; ++t) sdata[t] = sdata[t] + sdata[t + s];
    return sdata[0];
}

void orc_layer_norm_f32(const float* x, float* y, size_t n, float eps) {
    const int T = n < ORC_BLOCK ? (int)n : ORC_BLOCK;
    float sdata[ORC_BLOCK];
    for (int t = 0; t < T; ++t) {
        float s = 0.0f;
        for (size_t i = (size_t)t; i < n; i += (size_t)T) s += x[i];
        sdata[t] = s;
    }
    const float mean = halving_tree(sdata, T) / (float)n;
    for (int t = 0; t < T; ++t) {
        float s = 0.0f;
        for (size_t i = (size_t)t; i < n; i += (size_t)T) {
            const float d = x[i] - mean;
            const float sq = d * d;
            s = s + sq;
        }
        sdata[t] = s;
    }
    const float var = halving_tree(sdata, T) / (float)n;
    /* rsqrtf: CUDA's approximate reciprocal square root; the oracle uses the
     * correctly rounded value, so inv_std may differ by an ULP or two. */
    const float inv_std = (float)(1.0 / sqrt((double)(var + eps)));
    for (size_t i = 0; i < n; ++i) y[i] = (x[i] - mean) * inv_std;
}

typedef struct { const float* x; float* y; size_t cols; float eps; int ln; } rows_ctx;

static void rows_range(void* p, size_t lo, size_t hi) {
    const rows_ctx* c = (const rows_ctx*)p;
    float* tmp = c->ln ? (float*)malloc(sizeof(float) * c->cols) : NULL;
    for (size_t r = lo; r < hi; ++r) {
        const float* in = c->x + r * c->cols;
        float* out = c->y + r * c->cols;
        if (c->ln) {
            softmax_row(in, tmp, c->cols);
            orc_layer_norm_f32(tmp, out, c->cols, c->eps);
        } else {
            softmax_row(in, out, c->cols);
        }
    }
    free(tmp);
}

void orc_softmax_rows_f32(const float* x, float* y, size_t rows, size_t cols, int threads) {
    rows_ctx c = {x, y, cols, 0.0f, 0};
    orc_parallel(rows_range, &c, rows, threads);
}

void orc_softmax_layernorm_rows_f32(const float* x, float* y, size_t rows, size_t cols, float eps, int threads) {
    rows_ctx c = {x, y, cols, eps, 1};
    orc_parallel(rows_range, &c, rows, threads);
}

/* ------------------------------------------------------------------- GEMM */

typedef struct { const float* A; const float* B; float* C; int M, K, N, r0; } mm_ctx;

/* k_matmul_f32, src/runtime/ops_bridge.cu:13-31: per output one __fmaf_rn
 * chain over k = 0..K-1 in order, continued over the zero padding up to the
 * next multiple of 16 (fmaf(0,0,acc)). */
static void mm_range(void* p, size_t lo, size_t hi) {
    const mm_ctx* c = (const mm_ctx*)p;
    const int kpad = (c->K + 15) / 16 * 16;
    for (size_t rr = lo; rr < hi; ++rr) {
        const int r = c->r0 + (int)rr;
        for (int j = 0; j < c->N; ++j) {
            float acc = 0.0f;
            for (int k = 0; k < c->K; ++k) acc = fmaf(c->A[(size_t)r * c->K + k], c->B[(size_t)k * c->N + j], acc);
            for (int k = c->K; k < kpad; ++k) acc = fmaf(0.0f, 0.0f, acc);
            c->C[(size_t)r * c->N + j] = acc;
        }
    }
}

void orc_matmul_f32(const float* A, const float* B, float* C, int M, int K, int N, int r0, int r1, int threads) {
    if (r0 < 0) r0 = 0;
    if (r1 > M) r1 = M;
    if (r1 <= r0) return;
    mm_ctx c = {A, B, C, M, K, N, r0};
    orc_parallel(mm_range, &c, (size_t)(r1 - r0), threads);
}

static float bf16_to_f32(uint16_t h) {
    uint32_t u = (uint32_t)h << 16;
    float f;
    memcpy(&f, &u, sizeof(f));
    return f;
}

/* The reference's bf16 matmul path casts both operands to f32 (k_cast_to_f32,
 * src/runtime/exec_planner.cu:36-63) and runs k_matmul_f32 on them. */
void orc_matmul_bf16_tile(const uint16_t* A, const uint16_t* B, float* C, int M, int K, int N,
                          int r0, int r1, int c0, int c1) {
    (void)M;
    const int kpad = (K + 15) / 16 * 16;
    const int ld = c1 - c0;
    for (int r = r0; r < r1; ++r)
        for (int j = c0; j < c1; ++j) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k)
                acc = fmaf(bf16_to_f32(A[(size_t)r * K + k]), bf16_to_f32(B[(size_t)k * N + j]), acc);
            for (int k = K; k < kpad; ++k) acc = fmaf(0.0f, 0.0f, acc);
            C[(size_t)(r - r0) * ld + (j - c0)] = acc;
        }
}

/* ------------------------------------------------------------------- TLSF */

/* Restatement of native/core/memory/modules/tlsf_allocator_internals.inl and
 * tlsf_allocator_api.inl (alloc :111-198, free :200-296). Blocks are nodes
 * in index-linked lists; allocated offsets are found through an open-address
 * table with tombstones (the reference hashes into 4096 chained buckets;
 * the lookup structure does not affect any decision). */

#define T_FL 34
#define T_SL 16
#define T_NIL 0xFFFFFFFFu

typedef struct {
    uint64_t off, size;
    uint32_t prev_phys, next_phys, prev_free, next_free;
    int is_free;
} t_block;

struct orc_tlsf {
    uint64_t pool_size;
    t_block* b;
    uint32_t nb, cap;
    uint32_t* spare;
    uint32_t nspare, cap_spare;
    uint32_t heads[T_FL][T_SL];
    uint64_t* keys;     /* 0 empty, 1 tombstone, else off+2 */
    uint32_t* vals;
    uint64_t tcap, tused;
    uint64_t allocated;
    uint32_t blocks;
};

static void t_mapping(uint64_t size, int* fl, int* sl) {   /* internals.inl:71-91 */
    if (size < 64) { *fl = 0; *sl = 0; return; }
    int f = 63 - __builtin_clzll(size);
    if (f >= T_FL) f = T_FL - 1;
    *fl = f;
    *sl = f >= 4 ? (int)((size >> (f - 4)) & (T_SL - 1)) : 0;
}

static uint32_t t_new(orc_tlsf* t) {
    if (t->nspare) return t->spare[--t->nspare];
    if (t->nb == t->cap) {
        t->cap = t->cap ? t->cap * 2 : 1024;
        t->b = (t_block*)realloc(t->b, sizeof(t_block) * t->cap);
    }
    return t->nb++;
}

static void t_drop(orc_tlsf* t, uint32_t i) {
    if (t->nspare == t->cap_spare) {
        t->cap_spare = t->cap_spare ? t->cap_spare * 2 : 1024;
        t->spare = (uint32_t*)realloc(t->spare, sizeof(uint32_t) * t->cap_spare);
    }
    t->spare[t->nspare++] = i;
}

static uint64_t t_slot(const orc_tlsf* t, uint64_t off) {
    return ((off + 2) * 0x9E3779B97F4A7C15ull) & (t->tcap - 1);
}

static void t_put(orc_tlsf* t, uint64_t off, uint32_t v);

static void t_grow(orc_tlsf* t) {
    uint64_t oc = t->tcap;
    uint64_t* ok = t->keys;
    uint32_t* ov = t->vals;
    t->tcap = oc ? oc * 2 : 4096;
    t->keys = (uint64_t*)calloc(t->tcap, sizeof(uint64_t));
    t->vals = (uint32_t*)calloc(t->tcap, sizeof(uint32_t));
    t->tused = 0;
    for (uint64_t i = 0; i < oc; ++i)
        if (ok[i] > 1) t_put(t, ok[i] - 2, ov[i]);
    free(ok);
    free(ov);
}

static void t_put(orc_tlsf* t, uint64_t off, uint32_t v) {
    if ((t->tused + 1) * 2 > t->tcap) t_grow(t);
    uint64_t i = t_slot(t, off);
    while (t->keys[i] > 1) i = (i + 1) & (t->tcap - 1);
    if (t->keys[i] == 0) ++t->tused;
    t->keys[i] = off + 2;
    t->vals[i] = v;
}

static uint32_t t_take(orc_tlsf* t, uint64_t off) {
    uint64_t i = t_slot(t, off);
    while (t->keys[i] != 0) {
        if (t->keys[i] == off + 2) { t->keys[i] = 1; return t->vals[i]; }
        i = (i + 1) & (t->tcap - 1);
    }
    return T_NIL;
}

static void t_insert_free(orc_tlsf* t, uint32_t i) {   /* internals.inl:164-189 */
    int fl, sl;
    t_mapping(t->b[i].size, &fl, &sl);
    t->b[i].next_free = t->heads[fl][sl];
    t->b[i].prev_free = T_NIL;
    if (t->heads[fl][sl] != T_NIL) t->b[t->heads[fl][sl]].prev_free = i;
    t->heads[fl][sl] = i;
    t->b[i].is_free = 1;
}

static void t_remove_free(orc_tlsf* t, uint32_t i) {   /* internals.inl:191-206 */
    int fl, sl;
    t_mapping(t->b[i].size, &fl, &sl);
    if (t->b[i].prev_free != T_NIL) t->b[t->b[i].prev_free].next_free = t->b[i].next_free;
    else t->heads[fl][sl] = t->b[i].next_free;
    if (t->b[i].next_free != T_NIL) t->b[t->b[i].next_free].prev_free = t->b[i].prev_free;
    t->b[i].is_free = 0;
}

static uint32_t t_find(const orc_tlsf* t, uint64_t size) {   /* internals.inl:208-231 */
    int fl, sl;
    t_mapping(size, &fl, &sl);
    for (int s = sl; s < T_SL; ++s) {
        uint32_t h = t->heads[fl][s];
        if (h != T_NIL && t->b[h].size >= size) return h;
    }
    for (int f = fl + 1; f < T_FL; ++f)
        for (int s = 0; s < T_SL; ++s)
            if (t->heads[f][s] != T_NIL) return t->heads[f][s];
    return T_NIL;
}

orc_tlsf* orc_tlsf_create(uint64_t pool_size) {   /* api.inl:9-58 */
    orc_tlsf* t = (orc_tlsf*)calloc(1, sizeof(orc_tlsf));
    t->pool_size = pool_size;
    for (int f = 0; f < T_FL; ++f)
        for (int s = 0; s < T_SL; ++s) t->heads[f][s] = T_NIL;
    t_grow(t);
    uint32_t i = t_new(t);
    t->b[i].off = 0;
    t->b[i].size = pool_size;
    t->b[i].prev_phys = t->b[i].next_phys = T_NIL;
    t_insert_free(t, i);
    t->blocks = 1;
    return t;
}

void orc_tlsf_destroy(orc_tlsf* t) {
    if (!t) return;
    free(t->b);
    free(t->spare);
    free(t->keys);
    free(t->vals);
    free(t);
}

uint64_t orc_tlsf_alloc(orc_tlsf* t, uint64_t size) {   /* api.inl:111-198 */
    if (size == 0) return UINT64_MAX;
    size = (size + 255) & ~(uint64_t)255;
    uint32_t i = t_find(t, size);
    if (i == T_NIL) return UINT64_MAX;
    t_remove_free(t, i);
    uint64_t rest = t->b[i].size - size;
    if (rest >= 64) {   /* split_block, internals.inl:237-271 */
        uint32_t r = t_new(t);
        t->b[r].off = t->b[i].off + size;
        t->b[r].size = rest;
        t->b[r].prev_phys = i;
        t->b[r].next_phys = t->b[i].next_phys;
        if (t->b[i].next_phys != T_NIL) t->b[t->b[i].next_phys].prev_phys = r;
        t->b[i].size = size;
        t->b[i].next_phys = r;
        t_insert_free(t, r);
        ++t->blocks;
    }
    t_put(t, t->b[i].off, i);
    t->allocated += t->b[i].size;
    return t->b[i].off;
}

int orc_tlsf_free(orc_tlsf* t, uint64_t off) {   /* api.inl:200-296, coalesce internals.inl:273-321 */
    uint32_t i = t_take(t, off);
    if (i == T_NIL) return -1;
    t->allocated -= t->b[i].size;
    uint32_t nx = t->b[i].next_phys;
    if (nx != T_NIL && t->b[nx].is_free) {
        t_remove_free(t, nx);
        t->b[i].size += t->b[nx].size;
        t->b[i].next_phys = t->b[nx].next_phys;
        if (t->b[i].next_phys != T_NIL) t->b[t->b[i].next_phys].prev_phys = i;
        t_drop(t, nx);
        --t->blocks;
    }
    uint32_t pv = t->b[i].prev_phys;
    if (pv != T_NIL && t->b[pv].is_free) {
        t_remove_free(t, pv);
        t->b[pv].size += t->b[i].size;
        t->b[pv].next_phys = t->b[i].next_phys;
        if (t->b[pv].next_phys != T_NIL) t->b[t->b[pv].next_phys].prev_phys = pv;
        t_drop(t, i);
        i = pv;
        --t->blocks;
    }
    t_insert_free(t, i);
    return 0;
}

uint64_t orc_tlsf_allocated_bytes(const orc_tlsf* t) { return t->allocated; }
uint32_t orc_tlsf_block_count(const orc_tlsf* t) { return t->blocks; }
