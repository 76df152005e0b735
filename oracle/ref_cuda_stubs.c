/* ORACLE — test infrastructure only. Host-only stand-ins for the CUDA driver
 * and runtime calls that the reference TLSF source references
 * (native/core/include/memory/ptx_cuda_driver.h). The parity tests only use
 * ptx_tlsf_create_from_pool over a fake address range, which never reaches
 * these; every stub reports failure. */
#include <stddef.h>

typedef int CUresult;
typedef unsigned long long CUdeviceptr;
typedef int CUdevice;
typedef void* CUcontext;

CUresult cuInit(unsigned int f) { (void)f; return 3; }
CUresult cuGetErrorString(CUresult e, const char** s) { (void)e; if (s) *s = "stub"; return 0; }
CUresult cuCtxGetCurrent(CUcontext* c) { if (c) *c = 0; return 3; }
CUresult cuDeviceGet(CUdevice* d, int o) { (void)d; (void)o; return 3; }
CUresult cuDevicePrimaryCtxRetain(CUcontext* c, CUdevice d) { (void)c; (void)d; return 3; }
CUresult cuCtxSetCurrent(CUcontext c) { (void)c; return 3; }
CUresult cuMemAlloc_v2(CUdeviceptr* p, size_t n) { (void)p; (void)n; return 2; }
CUresult cuMemFree_v2(CUdeviceptr p) { (void)p; return 0; }
int cudaGetDevice(int* d) { if (d) *d = 0; return 100; }
int cudaMemcpy(void* d, const void* s, size_t n, int kind) { (void)d; (void)s; (void)n; (void)kind; return 1; }
