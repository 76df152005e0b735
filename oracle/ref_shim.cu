// ORACLE — test infrastructure only. Exposes the reference's own fer::ops
// GEMM and layer-norm launchers (src/runtime/ops_bridge.cu:87-104, compiled
// from the reference sources by oracle/Makefile) under plain C names so the
// GPU parity tests can run them on the same device buffers as the product.
#include "fercuda/compute/ops.cuh"

#include <cuda_runtime.h>

extern "C" void refshim_matmul_f32(const float* A, const float* B, float* C, int M, int K, int N, cudaStream_t s) {
    fer::FTensor2D a(reinterpret_cast<fer::F32*>(const_cast<float*>(A)), fer::Shape<2>(M, K));
    fer::FTensor2D b(reinterpret_cast<fer::F32*>(const_cast<float*>(B)), fer::Shape<2>(K, N));
    fer::FTensor2D c(reinterpret_cast<fer::F32*>(C), fer::Shape<2>(M, N));
    fer::ops::matmul(a, b, c, s);
}

extern "C" void refshim_layer_norm_f32(const float* x, float* y, int n, float eps, cudaStream_t s) {
    fer::FTensor1D xi(reinterpret_cast<fer::F32*>(const_cast<float*>(x)), fer::Shape<1>(n));
    fer::FTensor1D yo(reinterpret_cast<fer::F32*>(y), fer::Shape<1>(n));
    fer::ops::layer_norm(xi, yo, eps, s);
}
