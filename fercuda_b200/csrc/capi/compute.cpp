// Compute submissions: fer_submit_matmul, fer_submit_layer_norm and the
// additive fer_submit_rows / fer_submit_gemm.
//
// Argument checks and error codes follow the reference
// (src/runtime/session.cu:298-372): missing ids -> NOT_FOUND, unsupported or
// mismatched dtypes and wrong ranks -> INVALID_ARGUMENT. One check is added:
// matmul operand shapes must agree ([M,K] x [K,N] -> [M,N]); the reference
// reads and writes out of bounds when they do not.
#include "session.hpp"

#include <vector>

using fer::capi::Buffer;
using fer::capi::Session;
using fer::capi::Temp;
using fer::capi::internal;
using fer::capi::invalid;
using fer::capi::not_found;
using fer::capi::ok;

namespace {

bool compute_dtype(uint32_t dt) {
    return dt == FER_DTYPE_F32 || dt == FER_DTYPE_F16 || dt == FER_DTYPE_BF16 || dt == FER_DTYPE_I8 ||
           dt == FER_DTYPE_U8;
}

fer_status_t launched(cudaError_t e) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        return internal("kernel launch failed");
    }
    return ok();
}

}  // namespace

extern "C" {

fer_status_t fer_submit_matmul(fer_session_t* session, const fer_matmul_request_t* req, uint64_t* out_job_id) {
    if (!session) return invalid("session is null");
    if (!req) return invalid("request is null");
    Session& S = session->impl;
    const Buffer* a = S.find(req->a);
    const Buffer* b = S.find(req->b);
    const Buffer* o = S.find(req->out);
    if (!a || !b || !o) return not_found("buffer id not found");
    if (!compute_dtype(a->desc.dtype) || !compute_dtype(b->desc.dtype) || !compute_dtype(o->desc.dtype))
        return invalid("matmul requires supported buffers (f32/f16/bf16/i8/u8)");
    if (a->desc.dtype != b->desc.dtype || a->desc.dtype != o->desc.dtype)
        return invalid("matmul requires matching dtypes across A/B/out");
    if (a->desc.rank != 2 || b->desc.rank != 2 || o->desc.rank != 2) return invalid("matmul requires rank-2 buffers");
    const int M = static_cast<int>(a->desc.dims[0]), K = static_cast<int>(a->desc.dims[1]);
    const int N = static_cast<int>(b->desc.dims[1]);
    if (b->desc.dims[0] != a->desc.dims[1] || o->desc.dims[0] != a->desc.dims[0] || o->desc.dims[1] != b->desc.dims[1])
        return invalid("matmul shape mismatch");
    fer_status_t st = launched(fer_matmul_ref_order(a->ptr, b->ptr, o->ptr, M, K, N, a->desc.dtype, S.stream));
    if (st.code != FER_STATUS_OK) return st;
    uint64_t job = 0;
    st = S.make_job({}, &job);
    if (st.code == FER_STATUS_OK && out_job_id) *out_job_id = job;
    return st;
}

fer_status_t fer_submit_layer_norm(fer_session_t* session, const fer_layer_norm_request_t* req, uint64_t* out_job_id) {
    if (!session) return invalid("session is null");
    if (!req) return invalid("request is null");
    Session& S = session->impl;
    const Buffer* x = S.find(req->x);
    const Buffer* o = S.find(req->out);
    if (!x || !o) return not_found("buffer id not found");
    if (!compute_dtype(x->desc.dtype) || !compute_dtype(o->desc.dtype))
        return invalid("layer_norm requires supported buffers (f32/f16/bf16/i8/u8)");
    if (x->desc.dtype != o->desc.dtype) return invalid("layer_norm requires matching dtypes for x/out");
    // Rank 1: one row, as in the reference. Rank 2 [rows, cols]: every row
    // normalised (additive; the reference accepts rank 1 only).
    if (x->desc.rank < 1 || x->desc.rank > 2 || o->desc.rank != x->desc.rank)
        return invalid("layer_norm requires rank-1 buffers");
    if (o->numel != x->numel || (x->desc.rank == 2 && (o->desc.dims[0] != x->desc.dims[0] ||
                                                       o->desc.dims[1] != x->desc.dims[1])))
        return invalid("layer_norm shape mismatch");
    const int rows = x->desc.rank == 2 ? static_cast<int>(x->desc.dims[0]) : 1;
    const int cols = static_cast<int>(x->desc.dims[x->desc.rank - 1]);
    // Every dtype in one launch, no f32 temporaries: the kernel widens on
    // load and rounds on store exactly as the reference's cast staging does
    // (exec_planner.cu:304-387).
    fer_status_t st = launched(fer_layer_norm_typed(x->ptr, o->ptr, rows, cols, req->eps, x->desc.dtype, S.dev_err,
                                                    S.stream));
    if (st.code != FER_STATUS_OK) return st;
    uint64_t job = 0;
    st = S.make_job({}, &job);
    if (st.code == FER_STATUS_OK && out_job_id) *out_job_id = job;
    return st;
}

fer_status_t fer_submit_rows(fer_session_t* session, const fer_rows_request_t* req, uint64_t* out_job_id) {
    if (!session) return invalid("session is null");
    if (!req) return invalid("request is null");
    Session& S = session->impl;
    const Buffer* x = S.find(req->x);
    const Buffer* o = S.find(req->out);
    if (!x || !o) return not_found("buffer id not found");
    if (x->desc.dtype != FER_DTYPE_F32 || o->desc.dtype != FER_DTYPE_F32) return invalid("rows requires f32 buffers");
    if (x->desc.rank > 2 || o->numel != x->numel) return invalid("rows requires matching rank-1/2 buffers");
    const uint32_t ops = req->ops & (FER_ROWS_SOFTMAX | FER_ROWS_LAYER_NORM);
    if (ops == 0 || (req->ops & ~(FER_ROWS_SOFTMAX | FER_ROWS_LAYER_NORM | FER_ROWS_FAST)))
        return invalid("rows ops must be SOFTMAX and/or LAYER_NORM (optionally FAST)");
    const int rows = x->desc.rank == 2 ? static_cast<int>(x->desc.dims[0]) : 1;
    const int cols = x->desc.rank == 2 ? static_cast<int>(x->desc.dims[1]) : static_cast<int>(x->desc.dims[0]);
    const float* gamma = nullptr;
    const float* beta = nullptr;
    for (int k = 0; k < 2; ++k) {
        const uint64_t id = k == 0 ? req->gamma : req->beta;
        if (!id) continue;
        const Buffer* g = S.find(id);
        if (!g) return not_found("buffer id not found");
        if (g->desc.dtype != FER_DTYPE_F32 || g->numel != static_cast<size_t>(cols))
            return invalid("gamma/beta must be f32 with cols elements");
        (k == 0 ? gamma : beta) = static_cast<const float*>(g->ptr);
    }
    // programmatic launch; how much may run before the kernel waits for the
    // one before it follows from their footprints (Session::pdl_early)
    const size_t row_bytes = static_cast<size_t>(cols) * sizeof(float);
    uintptr_t in_lo[3] = {reinterpret_cast<uintptr_t>(x->ptr), 0, 0}, in_hi[3] = {in_lo[0] + x->bytes, 0, 0};
    uint32_t n_in = 1;
    for (const float* g : {gamma, beta})
        if (g) {
            in_lo[n_in] = reinterpret_cast<uintptr_t>(g);
            in_hi[n_in] = in_lo[n_in] + row_bytes;
            ++n_in;
        }
    const uintptr_t out_lo = reinterpret_cast<uintptr_t>(o->ptr), out_hi = out_lo + o->bytes;
    const uint32_t early = S.pdl_early(in_lo, in_hi, n_in, out_lo, out_hi);
    cudaError_t e = cudaErrorNotSupported;
    if (req->ops & FER_ROWS_FAST)
        e = fer_rows_fast_f32_pdl(static_cast<const float*>(x->ptr), static_cast<float*>(o->ptr), gamma, beta, rows,
                                  cols, req->eps, ops, early, S.dev_err, S.stream);
    if (e == cudaErrorNotSupported)
        e = fer_rows_f32_pdl(static_cast<const float*>(x->ptr), static_cast<float*>(o->ptr), gamma, beta, rows, cols,
                             req->eps, ops, early, S.dev_err, S.stream);
    if (e == cudaSuccess) S.pdl_record(in_lo, in_hi, n_in, out_lo, out_hi);
    fer_status_t st = launched(e);
    if (st.code != FER_STATUS_OK) return st;
    uint64_t job = 0;
    st = S.make_job({}, &job);
    if (st.code == FER_STATUS_OK && out_job_id) *out_job_id = job;
    return st;
}

fer_status_t fer_submit_gemm(fer_session_t* session, const fer_gemm_request_t* req, uint64_t* out_job_id) {
    if (!session) return invalid("session is null");
    if (!req) return invalid("request is null");
    Session& S = session->impl;
    const Buffer* a = S.find(req->a);
    const Buffer* b = S.find(req->b);
    const Buffer* o = S.find(req->out);
    if (!a || !b || !o) return not_found("buffer id not found");
    if (a->desc.dtype != FER_DTYPE_BF16 || b->desc.dtype != FER_DTYPE_BF16)
        return invalid("gemm requires bf16 operands");
    if (o->desc.dtype != FER_DTYPE_F32 && o->desc.dtype != FER_DTYPE_BF16) return invalid("gemm output must be f32 or bf16");
    if (a->desc.rank != 2 || b->desc.rank != 2 || o->desc.rank != 2) return invalid("gemm requires rank-2 buffers");
    if (b->desc.dims[0] != a->desc.dims[1] || o->desc.dims[0] != a->desc.dims[0] || o->desc.dims[1] != b->desc.dims[1])
        return invalid("gemm shape mismatch");
    if (req->flags != 0) return invalid("gemm flags must be 0");
    const int M = static_cast<int>(a->desc.dims[0]), K = static_cast<int>(a->desc.dims[1]);
    const int N = static_cast<int>(b->desc.dims[1]);
    cudaError_t e;
    if (K % 8 == 0 && N % 8 == 0) {
        e = fer_gemm_bf16_tc(a->ptr, b->ptr, o->ptr, M, N, K, o->desc.dtype, S.dev_err, S.stream);
    } else if (o->desc.dtype == FER_DTYPE_BF16) {
        e = fer_matmul_ref_order(a->ptr, b->ptr, o->ptr, M, K, N, FER_DTYPE_BF16, S.stream);
    } else {
        e = fer_matmul_bf16_f32_ref_order(a->ptr, b->ptr, static_cast<float*>(o->ptr), M, K, N, S.stream);
    }
    fer_status_t st = launched(e);
    if (st.code != FER_STATUS_OK) return st;
    uint64_t job = 0;
    st = S.make_job({}, &job);
    if (st.code == FER_STATUS_OK && out_job_id) *out_job_id = job;
    return st;
}

}  // extern "C"
