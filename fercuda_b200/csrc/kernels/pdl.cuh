// Programmatic dependent launch (PDL).
//
// A kernel launched with the programmatic-serialization attribute may be
// scheduled while the kernel before it on the stream is still running, so
// its launch and prologue overlap that kernel's tail. Such a kernel calls
// pdl_begin() before its first global-memory access: griddepcontrol.wait
// returns once the preceding kernel has completed and its writes are
// visible; launch_dependents then lets the next kernel be scheduled. Without
// a programmatic predecessor both are no-ops, so the kernels stay correct
// under plain launches. FERCUDA_PDL=0 launches without the attribute.
//
// Since every kernel of a chain triggers only after its own wait, a kernel
// that starts running finds the kernel two places back (and all before it)
// complete. Data that the immediately preceding kernel does not write
// (weights, cache rows of earlier steps) may therefore be read before
// pdl_wait(); everything else after it.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <utility>

namespace fer::dev {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

__device__ __forceinline__ void pdl_begin() {
    pdl_wait();
    pdl_trigger();
}

}  // namespace fer::dev

// Process-wide count of programmatic launches (kernels/pdl.cu).
extern "C" uint64_t fer_pdl_launch_count();
extern "C" void fer_pdl_note_launch();

namespace fer::host {

inline bool pdl_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("FERCUDA_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Launches a kernel that begins with pdl_begin(), with the PDL attribute.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    // counted even without the attribute: the kernel still triggers its
    // dependents, so a programmatic launch after it may start early
    fer_pdl_note_launch();
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace fer::host
