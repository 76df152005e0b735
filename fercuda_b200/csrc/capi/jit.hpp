// JIT manager: NVRTC compile of CUDA source to a sm_100a cubin, memory and
// disk caches keyed by FNV-1a of (lowered source, options, device arch,
// NVRTC version), contract-checked launches, and the code generator for
// fused elementwise chains.
//
// Replaces the reference JitManager (native/core/jit/jit_manager.cu:273-672)
// and LoweringPipeline (native/core/jit/lowering/pipeline/lowering_pipeline.cpp:10-43).
#pragma once

#include "session.hpp"

#include <cuda_runtime_api.h>

#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

namespace fer::capi {

struct Module {
    cudaLibrary_t lib = nullptr;
    std::string key;
    bool strict = false;
    ~Module();
};

struct ChainKernels {
    cudaKernel_t v4 = nullptr;   // 16-byte aligned streams, float4 per step
    cudaKernel_t s1 = nullptr;   // scalar tail / unaligned streams
    // the same kernels as driver functions of this session's context,
    // resolved once (null: launched through the runtime)
    void* fv4 = nullptr;
    void* fs1 = nullptr;
    std::shared_ptr<Module> mod;
};

class JitManager {
public:
    explicit JitManager(Session* s) : session_(s) {}

    fer_status_t compile(const fer_jit_source_t* src, const fer_jit_options_t* opt, fer_jit_program_t* out,
                         fer_jit_compile_result_t* res);
    fer_status_t release_program(fer_jit_program_t p);
    fer_status_t get_kernel(fer_jit_program_t p, const char* name, const fer_jit_kernel_sig_t* sig,
                            fer_jit_kernel_t* out);
    fer_status_t release_kernel(fer_jit_kernel_t k);
    fer_status_t launch(fer_jit_kernel_t k, const fer_jit_launch_cfg_t* cfg, const fer_jit_arg_pack_t* args,
                        uint64_t* out_job);
    fer_status_t cache_clear();
    fer_status_t stats(fer_jit_stats_t* out);

    // Compiles (once) and returns the kernels for a chain program.
    fer_status_t chain_kernels(const fer_chain_op_t* ops, uint32_t n_ops, uint32_t n_inputs, const ChainKernels** out);
    // Compiles (once) an internal module from generated source.
    fer_status_t internal_module(const std::string& source, std::shared_ptr<Module>* out, std::string* log);

    int sm() const;   // device compute capability * 10

private:
    fer_status_t build(const std::string& source, uint32_t kind, const std::vector<std::string>& opts,
                       const char* cache_dir, bool strict, std::shared_ptr<Module>* out, bool* hit,
                       std::string* log);

    Session* session_;
    std::mutex mu_;
    std::unordered_map<std::string, std::shared_ptr<Module>> cache_;
    std::unordered_map<std::string, ChainKernels> chains_;
    fer_jit_stats_t stats_{};
    std::string last_log_;
    int sm_ = 0;
};

}  // namespace fer::capi

struct fer_jit_program {
    std::shared_ptr<fer::capi::Module> mod;
};

struct fer_jit_kernel {
    std::shared_ptr<fer::capi::Module> mod;
    cudaKernel_t fn = nullptr;
    std::vector<fer_jit_arg_desc_t> sig;
};
