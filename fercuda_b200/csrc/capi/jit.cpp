// JIT: lowering, NVRTC compile, caches, contract-checked launch, intents and
// fused elementwise chains.
//
// Lowering keeps the reference's pragma language
// (native/core/jit/lowering/transforms/pragma_parse_pass.cpp:26-91,
//  capabilities/capability_lowering_pass.cpp, fusion/fusion_pass.cpp:41-175):
//   // fercuda:require_sm>=N            rejected with INVALID_ARGUMENT below sm N
//   // fercuda:require=tensor_cores     -DFERCUDA_ENABLE_TENSOR_CORES=1
//   // fercuda:require=cooperative_groups
//   // fercuda:fuse=elementwise_chain   fuse the declared ir_node chain
//   // fercuda:ir_node=elementwise_{add,mul,relu,sigmoid,tanh,exp}
//   // fercuda:nvrtc_opt=<option>
// Where the reference generates a fused kernel string and never compiles it,
// this lowering appends the generated `fer_fused_elementwise(in, out, n)`
// (vectorised, grid-stride) to the module so fer_jit_get_kernel can return it.
//
// Compilation targets the device's own arch-specific SASS (sm_100a on B200)
// and loads it with cudaLibraryLoadData; launches go through cudaLaunchKernel,
// so the library needs no direct link to the driver library.
#include "jit.hpp"

#include <cuda.h>
#include <nvrtc.h>

#include <cerrno>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <sstream>
#include <sys/stat.h>
#include <unistd.h>

using fer::capi::Buffer;
using fer::capi::ChainKernels;
using fer::capi::JitManager;
using fer::capi::Module;
using fer::capi::Session;
using fer::capi::Temp;
using fer::capi::internal;
using fer::capi::invalid;
using fer::capi::not_found;
using fer::capi::ok;

extern "C" {
cudaError_t fer_reduce_f32(const float* in, float* out, float* scratch, unsigned int n, int is_max, cudaStream_t s);
size_t fer_reduce_scratch_floats(unsigned int n);
cudaError_t fer_conv2d_f32(const float* input, const float* weights, const float* bias, float* output, unsigned int H,
                           unsigned int W, unsigned int C, unsigned int KH, unsigned int KW, unsigned int F,
                           unsigned int pad_h, unsigned int pad_w, unsigned int sh, unsigned int sw, int relu,
                           cudaStream_t s);
}

namespace fer::capi {

Module::~Module() {
    if (lib) cudaLibraryUnload(lib);
}

namespace {

const char* const kBackend = "nvrtc";

uint64_t fnv1a(const void* data, size_t n, uint64_t h = 1469598103934665603ull) {
    const unsigned char* p = static_cast<const unsigned char*>(data);
    for (size_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}

std::vector<std::string> split_ws(const char* s) {
    std::vector<std::string> out;
    if (!s) return out;
    std::istringstream is(s);
    std::string tok;
    while (is >> tok) out.push_back(tok);
    return out;
}

std::string hex64(uint64_t v) {
    char b[17];
    std::snprintf(b, sizeof b, "%016llx", static_cast<unsigned long long>(v));
    return b;
}

bool read_file(const std::string& path, std::string* out) {
    std::ifstream f(path, std::ios::binary);
    if (!f) return false;
    std::ostringstream ss;
    ss << f.rdbuf();
    *out = ss.str();
    return !out->empty();
}

void write_file(const std::string& path, const std::string& data) {
    const std::string tmp = path + ".tmp" + std::to_string(::getpid());
    {
        std::ofstream f(tmp, std::ios::binary);
        if (!f) return;
        f.write(data.data(), static_cast<std::streamsize>(data.size()));
    }
    std::rename(tmp.c_str(), path.c_str());
}

bool ensure_dir(const char* dir) {
    if (!dir || !*dir) return false;
    return ::mkdir(dir, 0755) == 0 || errno == EEXIST;
}

// ------------------------------------------------------------------ lowering

struct Lowered {
    std::string source;
    std::vector<std::string> opts;
    std::vector<std::string> notes;
    int min_sm = 0;
    bool tensor_cores = false;
    bool coop = false;
    bool fuse = false;
    std::vector<std::string> ir_ops;
};

const char* elementwise_expr(const std::string& op) {
    if (op == "elementwise_relu") return "(a < 0.0f ? 0.0f : a)";
    if (op == "elementwise_sigmoid") return "(1.0f / (1.0f + expf(-a)))";
    if (op == "elementwise_tanh") return "tanhf(a)";
    if (op == "elementwise_exp") return "expf(a)";
    return nullptr;   // add / mul are binary
}

bool is_elementwise(const std::string& op) {
    return op == "elementwise_add" || op == "elementwise_mul" || elementwise_expr(op) != nullptr;
}

fer_status_t lower(const std::string& in, int sm, Lowered* L) {
    L->source = in;
    if (L->source.empty()) return invalid("source code is empty");
    if (L->source.back() != '\n') L->source.push_back('\n');
    L->notes.emplace_back("canonicalized source formatting");
    // pragma parse
    size_t pos = 0;
    while (pos < L->source.size()) {
        size_t end = L->source.find('\n', pos);
        if (end == std::string::npos) end = L->source.size();
        const std::string line = L->source.substr(pos, end - pos);
        const size_t tag = line.find("fercuda:");
        if (tag != std::string::npos) {
            const std::string cmd = line.substr(tag + 8);
            if (cmd.find("require=tensor_cores") != std::string::npos) {
                L->tensor_cores = true;
            } else if (cmd.find("require=cooperative_groups") != std::string::npos) {
                L->coop = true;
            } else if (cmd.find("fuse=elementwise_chain") != std::string::npos) {
                L->fuse = true;
            } else if (cmd.rfind("ir_node=", 0) == 0) {
                std::string op = cmd.substr(8);
                while (!op.empty() && (op.back() == '\r' || op.back() == ' ')) op.pop_back();
                if (is_elementwise(op) || op == "reduce_sum" || op == "reduce_max") {
                    L->ir_ops.push_back(op);
                    L->notes.emplace_back("ir node parsed: " + op);
                }
            } else if (cmd.rfind("nvrtc_opt=", 0) == 0) {
                L->opts.push_back(cmd.substr(10));
            } else if (cmd.rfind("require_sm>=", 0) == 0) {
                L->min_sm = std::atoi(cmd.c_str() + 12);
            }
        }
        pos = end == L->source.size() ? end : end + 1;
    }
    L->notes.emplace_back("pragmas parsed");
    // capability contracts
    if (L->min_sm > 0 && sm < L->min_sm) return invalid("required SM not available");
    L->opts.push_back("-DFERCUDA_TARGET_SM=" + std::to_string(sm));
    if (L->tensor_cores) L->opts.push_back("-DFERCUDA_ENABLE_TENSOR_CORES=1");
    if (L->coop) L->opts.push_back("-DFERCUDA_ENABLE_COOP_GROUPS=1");
    L->notes.emplace_back("capability contracts validated");
    if (L->source.find("fercuda:fuse") != std::string::npos) {
        L->notes.emplace_back("fusion hint detected");
        L->notes.emplace_back("tensor-core capable target");
    }
    // elementwise fusion
    if (L->fuse) {
        std::vector<std::string> chain;
        for (const auto& op : L->ir_ops)
            if (is_elementwise(op)) chain.push_back(op);
        if (chain.size() >= 2) {
            L->notes.emplace_back("elementwise IR chain fused (" + std::to_string(chain.size()) + " ops)");
            bool unary = true;
            for (const auto& op : chain)
                if (!elementwise_expr(op)) unary = false;
            if (unary && L->source.find("fer_fused_elementwise") == std::string::npos) {
                std::ostringstream k;
                k << "\n// fused elementwise chain generated by fercuda lowering\n"
                     "static __device__ __forceinline__ float fer_fused_apply(float a) {\n";
                for (const auto& op : chain) k << "  a = " << elementwise_expr(op) << ";\n";
                k << "  return a;\n}\n"
                     "extern \"C\" __global__ void __launch_bounds__(256) fer_fused_elementwise(\n"
                     "    const float* __restrict__ in, float* __restrict__ out, unsigned int n) {\n"
                     "  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;\n"
                     "  unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x;\n"
                     "  const bool vec = ((((unsigned long long)in) | ((unsigned long long)out)) & 15ull) == 0ull;\n"
                     "  if (vec) {\n"
                     "    const unsigned long long n4 = n / 4;\n"
                     "    for (unsigned long long j = i; j < n4; j += stride) {\n"
                     "      float4 v = reinterpret_cast<const float4*>(in)[j];\n"
                     "      v.x = fer_fused_apply(v.x); v.y = fer_fused_apply(v.y);\n"
                     "      v.z = fer_fused_apply(v.z); v.w = fer_fused_apply(v.w);\n"
                     "      reinterpret_cast<float4*>(out)[j] = v;\n"
                     "    }\n"
                     "    for (unsigned long long j = n4 * 4 + i; j < n; j += stride) out[j] = fer_fused_apply(in[j]);\n"
                     "  } else {\n"
                     "    for (unsigned long long j = i; j < n; j += stride) out[j] = fer_fused_apply(in[j]);\n"
                     "  }\n}\n";
                L->source += k.str();
                L->notes.emplace_back("fused unary elementwise kernel generated");
            }
            if (L->source.find("#define FERCUDA_FUSED_ELEMENTWISE 1") == std::string::npos) {
                L->source = "#define FERCUDA_FUSED_ELEMENTWISE 1\n" + L->source;
                L->notes.emplace_back("elementwise fusion rewrite materialized");
            }
        }
    }
    // elementwise -> reduce marker
    for (size_t i = 1; i < L->ir_ops.size(); ++i)
        if ((L->ir_ops[i] == "reduce_sum" || L->ir_ops[i] == "reduce_max") && is_elementwise(L->ir_ops[i - 1])) {
            L->notes.emplace_back("elementwise+reduce fused");
            if (L->source.find("#define FERCUDA_FUSED_REDUCE 1") == std::string::npos)
                L->source = "#define FERCUDA_FUSED_REDUCE 1\n" + L->source;
            break;
        }
    return ok();
}

std::string join(const std::vector<std::string>& v, const char* sep) {
    std::string s;
    for (size_t i = 0; i < v.size(); ++i) {
        if (i) s += sep;
        s += v[i];
    }
    return s;
}

// -------------------------------------------------------------- chain codegen

// Expression emitted for each unary opcode (operand `x`, parameters p0/p1).
const char* unary_expr(uint32_t op) {
    switch (op) {
        case FER_CHAIN_AFFINE: return "$X * $P0 + $P1";
        case FER_CHAIN_ADD_SCALAR: return "$X + $P0";
        case FER_CHAIN_MUL_SCALAR: return "$X * $P0";
        case FER_CHAIN_RELU: return "fmaxf(0.0f, $X)";
        case FER_CHAIN_SIGMOID: return "1.0f / (1.0f + expf(-$X))";
        case FER_CHAIN_EXP: return "expf($X)";
        case FER_CHAIN_TANH: return "tanhf($X)";
        case FER_CHAIN_GELU_TANH: return "fer_gelu_tanh($X)";
        case FER_CHAIN_SILU: return "$X / (1.0f + expf(-$X))";
        case FER_CHAIN_NEG: return "-$X";
        case FER_CHAIN_ABS: return "fabsf($X)";
        case FER_CHAIN_CLAMP: return "fminf($P1, fmaxf($P0, $X))";
        case FER_CHAIN_RELU_LT: return "($X < 0.0f ? 0.0f : $X)";
        case FER_CHAIN_FMA: return "fmaf($X, $P0, $P1)";
        default: return nullptr;
    }
}

const char* binary_expr(uint32_t op) {
    switch (op) {
        case FER_CHAIN_ADD: return "$A + $B";
        case FER_CHAIN_SUB: return "$A - $B";
        case FER_CHAIN_MUL: return "$A * $B";
        case FER_CHAIN_DIV: return "$A / $B";
        case FER_CHAIN_MAX: return "fmaxf($A, $B)";
        case FER_CHAIN_MIN: return "fminf($A, $B)";
        default: return nullptr;
    }
}

std::string replace_all(std::string s, const std::string& from, const std::string& to) {
    size_t p = 0;
    while ((p = s.find(from, p)) != std::string::npos) {
        s.replace(p, from.size(), to);
        p += to.size();
    }
    return s;
}

// Validates the stack program; writes the generated CUDA source.
fer_status_t chain_source(const fer_chain_op_t* ops, uint32_t n, uint32_t n_inputs, std::string* out) {
    if (!ops || n == 0) return invalid("chain is empty");
    if (n > FER_CHAIN_MAX_OPS) return invalid("chain has too many ops");
    std::ostringstream body;
    int depth = 0, max_depth = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const uint32_t op = ops[i].opcode;
        const std::string p0 = "p.v[" + std::to_string(2 * i) + "]";
        const std::string p1 = "p.v[" + std::to_string(2 * i + 1) + "]";
        if (op == FER_CHAIN_LOAD) {
            if (ops[i].arg >= n_inputs) return invalid("chain loads an input that was not bound");
            body << "  float s" << depth << " = i" << ops[i].arg << ";\n";
            ++depth;
            if (depth > max_depth) max_depth = depth;
        } else if (const char* u = unary_expr(op)) {
            if (depth < 1) return invalid("chain op needs an operand");
            const std::string e =
                replace_all(replace_all(replace_all(u, "$P0", p0), "$P1", p1), "$X", "s" + std::to_string(depth - 1));
            body << "  s" << depth - 1 << " = " << e << ";\n";
        } else if (const char* b = binary_expr(op)) {
            if (depth < 2) return invalid("chain op needs two operands");
            const std::string e =
                replace_all(replace_all(b, "$A", "s" + std::to_string(depth - 2)), "$B", "s" + std::to_string(depth - 1));
            body << "  s" << depth - 2 << " = " << e << ";\n";
            --depth;
        } else {
            return invalid("unknown chain opcode");
        }
    }
    if (depth != 1) return invalid("chain must leave exactly one value");
    if (max_depth > 8) return invalid("chain stack deeper than 8");
    std::ostringstream src;
    src << "// fused elementwise chain generated by fercuda\n"
           "struct FerChainParams { float v[" << 2 * FER_CHAIN_MAX_OPS << "]; };\n"
           "static __device__ __forceinline__ float fer_gelu_tanh(float x) {\n"
           "  const float x3 = x * x * x;\n"
           "  const float inner = 0.7978845608028654f * (x + 0.044715f * x3);\n"
           "  return 0.5f * x * (1.0f + tanhf(inner));\n}\n"
           "static __device__ __forceinline__ float fer_chain_eval(float i0, float i1, float i2, float i3,\n"
           "                                                      const FerChainParams& p) {\n"
           "  (void)i0; (void)i1; (void)i2; (void)i3;\n"
        << body.str() << "  return s0;\n}\n"
        << "static __device__ __forceinline__ float4 fer_chain_eval4(float4 x0, float4 x1, float4 x2, float4 x3,\n"
           "                                                       const FerChainParams& p) {\n"
           "  float4 r;\n"
           "  r.x = fer_chain_eval(x0.x, x1.x, x2.x, x3.x, p);\n"
           "  r.y = fer_chain_eval(x0.y, x1.y, x2.y, x3.y, p);\n"
           "  r.z = fer_chain_eval(x0.z, x1.z, x2.z, x3.z, p);\n"
           "  r.w = fer_chain_eval(x0.w, x1.w, x2.w, x3.w, p);\n"
           "  return r;\n}\n"
           "// early 1: the host found that the kernel just before this one on the\n"
           "// stream writes none of the inputs, so each thread's first two groups are\n"
           "// loaded and evaluated before the dependency wait; their stores wait.\n"
           "// early 2: that kernel also neither reads nor writes the output, so the\n"
           "// two groups are stored before the wait too. Every thread still waits\n"
           "// before it exits, so this kernel completes after that one.\n"
           "extern \"C\" __global__ void __launch_bounds__(256) fer_chain_v4(\n"
           "    const float4* __restrict__ a0, const float4* __restrict__ a1, const float4* __restrict__ a2,\n"
           "    const float4* __restrict__ a3, float4* __restrict__ out, unsigned long long n4, FerChainParams p,\n"
           "    unsigned early) {\n"
           "  const unsigned long long stride = (unsigned long long)gridDim.x * 256ull;\n"
           "  unsigned long long i = (unsigned long long)blockIdx.x * 256ull + threadIdx.x;\n"
           "  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);\n"
           "  float4 r0 = z, r1 = z;\n"
           "  if (early) {\n"
           "    if (i < n4)\n"
           "      r0 = fer_chain_eval4(a0 ? __ldcs(a0 + i) : z, a1 ? __ldcs(a1 + i) : z, a2 ? __ldcs(a2 + i) : z,\n"
           "                           a3 ? __ldcs(a3 + i) : z, p);\n"
           "    const unsigned long long k = i + stride;\n"
           "    if (k < n4)\n"
           "      r1 = fer_chain_eval4(a0 ? __ldcs(a0 + k) : z, a1 ? __ldcs(a1 + k) : z, a2 ? __ldcs(a2 + k) : z,\n"
           "                           a3 ? __ldcs(a3 + k) : z, p);\n"
           "  }\n"
           "  if (early == 2u) {\n"
           "    if (i < n4) __stcs(out + i, r0);\n"
           "    if (i + stride < n4) __stcs(out + i + stride, r1);\n"
           "  }\n"
           "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n"
           "  asm volatile(\"griddepcontrol.launch_dependents;\");\n"
           "  if (early) {\n"
           "    if (early == 1u) {\n"
           "      if (i < n4) __stcs(out + i, r0);\n"
           "      if (i + stride < n4) __stcs(out + i + stride, r1);\n"
           "    }\n"
           "    i += 2ull * stride;\n"
           "  }\n"
           "  for (; i + 3ull * stride < n4; i += 4ull * stride) {\n"
           "    float4 x0[4], x1[4], x2[4], x3[4];\n"
           "#pragma unroll\n"
           "    for (int u = 0; u < 4; ++u) {\n"
           "      const unsigned long long j = i + u * stride;\n"
           "      x0[u] = a0 ? __ldcs(a0 + j) : z; x1[u] = a1 ? __ldcs(a1 + j) : z;\n"
           "      x2[u] = a2 ? __ldcs(a2 + j) : z; x3[u] = a3 ? __ldcs(a3 + j) : z;\n"
           "    }\n"
           "#pragma unroll\n"
           "    for (int u = 0; u < 4; ++u) {\n"
           "      float4 r;\n"
           "      r.x = fer_chain_eval(x0[u].x, x1[u].x, x2[u].x, x3[u].x, p);\n"
           "      r.y = fer_chain_eval(x0[u].y, x1[u].y, x2[u].y, x3[u].y, p);\n"
           "      r.z = fer_chain_eval(x0[u].z, x1[u].z, x2[u].z, x3[u].z, p);\n"
           "      r.w = fer_chain_eval(x0[u].w, x1[u].w, x2[u].w, x3[u].w, p);\n"
           "      __stcs(out + i + u * stride, r);\n"
           "    }\n"
           "  }\n"
           "  for (; i < n4; i += stride) {\n"
           "    const float4 x0 = a0 ? __ldcs(a0 + i) : z, x1 = a1 ? __ldcs(a1 + i) : z;\n"
           "    const float4 x2 = a2 ? __ldcs(a2 + i) : z, x3 = a3 ? __ldcs(a3 + i) : z;\n"
           "    float4 r;\n"
           "    r.x = fer_chain_eval(x0.x, x1.x, x2.x, x3.x, p);\n"
           "    r.y = fer_chain_eval(x0.y, x1.y, x2.y, x3.y, p);\n"
           "    r.z = fer_chain_eval(x0.z, x1.z, x2.z, x3.z, p);\n"
           "    r.w = fer_chain_eval(x0.w, x1.w, x2.w, x3.w, p);\n"
           "    __stcs(out + i, r);\n"
           "  }\n}\n"
           "extern \"C\" __global__ void __launch_bounds__(256) fer_chain_s1(\n"
           "    const float* a0, const float* a1, const float* a2, const float* a3, float* out,\n"
           "    unsigned long long lo, unsigned long long n, FerChainParams p) {\n"
           "  asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n"
           "  asm volatile(\"griddepcontrol.launch_dependents;\");\n"
           "  const unsigned long long stride = (unsigned long long)gridDim.x * 256ull;\n"
           "  for (unsigned long long i = lo + (unsigned long long)blockIdx.x * 256ull + threadIdx.x; i < n; i += stride)\n"
           "    out[i] = fer_chain_eval(a0 ? a0[i] : 0.f, a1 ? a1[i] : 0.f, a2 ? a2[i] : 0.f, a3 ? a3[i] : 0.f, p);\n"
           "}\n";
    *out = src.str();
    return ok();
}

struct ChainParams {
    float v[2 * FER_CHAIN_MAX_OPS];
};

// Driver entry points for launching the chain kernels by CUfunction: a
// library kernel launched through the runtime is looked up for the current
// context on every launch; the function resolved once skips that.
// FERCUDA_CHAIN_DRIVER_LAUNCH=0 keeps the runtime launch.
struct DriverLaunch {
    CUresult (*get)(CUfunction*, CUkernel) = nullptr;
    CUresult (*launch)(const CUlaunchConfig*, CUfunction, void**, void**) = nullptr;
    bool ok = false;
};

const DriverLaunch& driver_launch() {
    static const DriverLaunch d = [] {
        DriverLaunch r;
        const char* e = std::getenv("FERCUDA_CHAIN_DRIVER_LAUNCH");
        if (e && e[0] == '0') return r;
        void* f0 = nullptr;
        void* f1 = nullptr;
        cudaDriverEntryPointQueryResult q0{}, q1{};
        if (cudaGetDriverEntryPointByVersion("cuKernelGetFunction", &f0, 12000, cudaEnableDefault, &q0) ==
                cudaSuccess &&
            cudaGetDriverEntryPointByVersion("cuLaunchKernelEx", &f1, 12000, cudaEnableDefault, &q1) == cudaSuccess &&
            q0 == cudaDriverEntryPointSuccess && q1 == cudaDriverEntryPointSuccess && f0 && f1) {
            r.get = reinterpret_cast<CUresult (*)(CUfunction*, CUkernel)>(f0);
            r.launch = reinterpret_cast<CUresult (*)(const CUlaunchConfig*, CUfunction, void**, void**)>(f1);
            r.ok = true;
        } else {
            cudaGetLastError();
        }
        return r;
    }();
    return d;
}

// The driver function of a library kernel in the current context (null if
// the driver path is off or the lookup fails).
void* driver_function(cudaKernel_t k) {
    const DriverLaunch& d = driver_launch();
    if (!d.ok || !k) return nullptr;
    CUfunction f = nullptr;
    return d.get(&f, reinterpret_cast<CUkernel>(k)) == CUDA_SUCCESS ? reinterpret_cast<void*>(f) : nullptr;
}

}  // namespace

int JitManager::sm() const {
    if (sm_ == 0) {
        int dev = 0, maj = 0, min = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&maj, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&min, cudaDevAttrComputeCapabilityMinor, dev);
        const_cast<JitManager*>(this)->sm_ = maj * 10 + min;
    }
    return sm_;
}

fer_status_t JitManager::build(const std::string& source, uint32_t kind, const std::vector<std::string>& opts,
                               const char* cache_dir, bool strict, std::shared_ptr<Module>* out, bool* hit,
                               std::string* log) {
    int nv_major = 0, nv_minor = 0;
    nvrtcVersion(&nv_major, &nv_minor);
    std::string keytext = source;
    keytext += '\0';
    keytext += join(opts, " ");
    keytext += ":k" + std::to_string(kind) + ":sm" + std::to_string(sm()) + ":nvrtc" + std::to_string(nv_major) + "." +
               std::to_string(nv_minor);
    const std::string key = hex64(fnv1a(keytext.data(), keytext.size()));
    *hit = false;
    {
        std::lock_guard<std::mutex> lk(mu_);
        auto it = cache_.find(key);
        if (it != cache_.end()) {
            *out = it->second;
            *hit = true;
            stats_.cache_hit_count++;
            return ok();
        }
    }
    const auto t0 = std::chrono::steady_clock::now();
    std::string image;
    const std::string disk = (cache_dir && ensure_dir(cache_dir)) ? std::string(cache_dir) + "/" + key + ".bin" : "";
    bool from_disk = !disk.empty() && read_file(disk, &image);
    if (!from_disk) {
        if (kind == FER_JIT_SOURCE_PTX) {
            image = source;
        } else {
            nvrtcProgram prog = nullptr;
            if (nvrtcCreateProgram(&prog, source.c_str(), "fer_jit.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
                return internal("nvrtcCreateProgram failed");
            std::vector<const char*> o;
            for (const auto& s : opts) o.push_back(s.c_str());
            const nvrtcResult r = nvrtcCompileProgram(prog, static_cast<int>(o.size()), o.data());
            size_t lsz = 0;
            nvrtcGetProgramLogSize(prog, &lsz);
            std::string l(lsz, '\0');
            if (lsz) nvrtcGetProgramLog(prog, &l[0]);
            while (!l.empty() && (l.back() == '\0' || l.back() == '\n')) l.pop_back();
            *log = l;
            if (r != NVRTC_SUCCESS) {
                nvrtcDestroyProgram(&prog);
                return internal("NVRTC compile failed");
            }
            bool real_arch = false;
            for (const auto& s : opts)
                if (s.rfind("--gpu-architecture=sm_", 0) == 0) real_arch = true;
            size_t sz = 0;
            if (real_arch) {
                nvrtcGetCUBINSize(prog, &sz);
                image.assign(sz, '\0');
                nvrtcGetCUBIN(prog, &image[0]);
            } else {
                nvrtcGetPTXSize(prog, &sz);
                image.assign(sz, '\0');
                nvrtcGetPTX(prog, &image[0]);
            }
            nvrtcDestroyProgram(&prog);
        }
    }
    auto mod = std::make_shared<Module>();
    mod->key = key;
    mod->strict = strict;
    if (cudaLibraryLoadData(&mod->lib, image.data(), nullptr, nullptr, 0, nullptr, nullptr, 0) != cudaSuccess) {
        cudaGetLastError();
        mod->lib = nullptr;
        return internal(kind == FER_JIT_SOURCE_PTX ? "PTX module load failed" : "module load failed");
    }
    if (!disk.empty() && !from_disk) write_file(disk, image);
    const uint64_t us = static_cast<uint64_t>(
        std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count());
    std::lock_guard<std::mutex> lk(mu_);
    cache_[key] = mod;
    if (from_disk) {
        stats_.cache_hit_count++;
        *hit = true;
    } else {
        stats_.compile_count++;
        stats_.compile_time_us += us;
    }
    *out = mod;
    return ok();
}

fer_status_t JitManager::compile(const fer_jit_source_t* src, const fer_jit_options_t* opt, fer_jit_program_t* out,
                                 fer_jit_compile_result_t* res) {
    if (!src) return invalid("source is null");
    if (!src->code || src->code_len == 0) return invalid("source code is empty");
    if (!out) return invalid("out_program is null");
    *out = nullptr;
    if (src->kind != FER_JIT_SOURCE_CUDA && src->kind != FER_JIT_SOURCE_PTX) return invalid("unknown source kind");
    if (opt && opt->backend != FER_JIT_BACKEND_NVRTC && opt->backend != FER_JIT_BACKEND_AUTO)
        return invalid("unsupported JIT backend");
    const std::string text(src->code, src->code_len);
    Lowered L;
    std::vector<std::string> opts;
    std::string notes;
    if (src->kind == FER_JIT_SOURCE_CUDA) {
        fer_status_t st = lower(text, sm(), &L);
        if (st.code != FER_STATUS_OK) return st;
        opts.emplace_back("--std=c++17");
        if (opt && opt->arch && opt->arch[0]) {
            opts.push_back(std::string("--gpu-architecture=") + opt->arch);
        } else {
            const int s = sm();
            const bool has_a = s == 90 || s == 100 || s == 101 || s == 103 || s == 120 || s == 121;
            opts.push_back("--gpu-architecture=sm_" + std::to_string(s) + (has_a ? "a" : ""));
        }
        for (auto& o : L.opts) opts.push_back(o);
        for (auto& o : split_ws(opt ? opt->extra_nvrtc_opts : nullptr)) opts.push_back(o);
        notes = "[lowering] " + join(L.notes, "; ");
    } else {
        L.source = text;
        if (L.source.back() != '\0') L.source.push_back('\0');
    }
    const char* cache_dir = (opt && opt->enable_disk_cache && opt->cache_dir) ? opt->cache_dir : nullptr;
    std::shared_ptr<Module> mod;
    bool hit = false;
    std::string log;
    fer_status_t st = build(L.source, src->kind, opts, cache_dir, opt && opt->mode == FER_JIT_MODE_STRICT, &mod, &hit, &log);
    {
        std::lock_guard<std::mutex> lk(mu_);
        last_log_ = hit ? std::string() : (log.empty() ? notes : notes + "\n" + log);
    }
    if (res) {
        res->cache_hit = hit ? 1 : 0;
        res->backend_name = kBackend;
        res->log = last_log_.c_str();
    }
    if (st.code != FER_STATUS_OK) return st;
    auto* p = new fer_jit_program();
    p->mod = mod;
    *out = p;
    return ok();
}

fer_status_t JitManager::release_program(fer_jit_program_t p) {
    delete p;
    return ok();
}

fer_status_t JitManager::get_kernel(fer_jit_program_t p, const char* name, const fer_jit_kernel_sig_t* sig,
                                    fer_jit_kernel_t* out) {
    if (!p || !p->mod) return invalid("program is null");
    if (!name || !*name) return invalid("kernel_name is empty");
    if (!out) return invalid("out_kernel is null");
    if (p->mod->strict && (!sig || !sig->args || sig->arg_count == 0))
        return invalid("strict mode requires kernel signature");
    *out = nullptr;
    cudaKernel_t fn = nullptr;
    if (cudaLibraryGetKernel(&fn, p->mod->lib, name) != cudaSuccess) {
        cudaGetLastError();
        return not_found("kernel symbol not found");
    }
    auto* k = new fer_jit_kernel();
    k->mod = p->mod;
    k->fn = fn;
    if (sig && sig->args && sig->arg_count) k->sig.assign(sig->args, sig->args + sig->arg_count);
    *out = k;
    return ok();
}

fer_status_t JitManager::release_kernel(fer_jit_kernel_t k) {
    delete k;
    return ok();
}

fer_status_t JitManager::launch(fer_jit_kernel_t k, const fer_jit_launch_cfg_t* cfg, const fer_jit_arg_pack_t* args,
                                uint64_t* out_job) {
    if (!k) return invalid("kernel is null");
    if (!cfg) return invalid("cfg is null");
    if (!args) return invalid("args is null");
    if (!out_job) return invalid("out_job_id is null");
    if (args->arg_count > 0 && !args->args) return invalid("args array is null");
    if (cfg->grid_x == 0 || cfg->block_x == 0) return invalid("invalid launch dimensions");
    if (cfg->block_y == 0 || cfg->block_z == 0) return invalid("invalid block dimensions");
    const uint64_t threads = static_cast<uint64_t>(cfg->block_x) * cfg->block_y * cfg->block_z;
    if (threads > 1024) return invalid("threads per block out of range");
    if (!k->sig.empty() && k->sig.size() != args->arg_count) return invalid("arg_count mismatch");
    const auto t0 = std::chrono::steady_clock::now();
    Session& S = *session_;
    std::vector<uint64_t> store(args->arg_count, 0);
    std::vector<void*> params(args->arg_count, nullptr);
    for (size_t i = 0; i < args->arg_count; ++i) {
        const fer_jit_arg_value_t& av = args->args[i];
        const fer_jit_arg_desc_t* d = i < k->sig.size() ? &k->sig[i] : nullptr;
        if (d && d->kind != av.kind) return invalid("arg kind mismatch");
        switch (av.kind) {
            case FER_JIT_ARG_BUFFER: {
                const Buffer* b = S.find(av.as.buffer_id);
                if (!b) return not_found("buffer id not found");
                if (d) {
                    if ((d->access == FER_JIT_ACCESS_WRITE || d->access == FER_JIT_ACCESS_READ_WRITE) && b->desc.immutable)
                        return invalid("immutable buffer cannot be used for write access");
                    if (d->expected_dtype != FER_JIT_WILDCARD_U32 && b->desc.dtype != d->expected_dtype)
                        return invalid("buffer dtype contract mismatch");
                    if (d->expected_rank != FER_JIT_WILDCARD_U32) {
                        if (b->desc.rank != d->expected_rank) return invalid("buffer rank contract mismatch");
                        for (uint32_t r = 0; r < b->desc.rank && r < 4; ++r)
                            if (d->expected_dims[r] != FER_JIT_WILDCARD_U32 && b->desc.dims[r] != d->expected_dims[r])
                                return invalid("buffer shape contract mismatch");
                    }
                    if (d->expected_bytes != FER_JIT_WILDCARD_U64 && b->bytes != d->expected_bytes)
                        return invalid("buffer byte-size contract mismatch");
                }
                if (cfg->memory_regime != FER_MEMORY_AUTO && b->regime != cfg->memory_regime)
                    return invalid("buffer regime does not match launch regime");
                store[i] = static_cast<uint64_t>(reinterpret_cast<uintptr_t>(b->ptr));
                break;
            }
            case FER_JIT_ARG_SCALAR_I32: std::memcpy(&store[i], &av.as.i32, 4); break;
            case FER_JIT_ARG_SCALAR_U32: std::memcpy(&store[i], &av.as.u32, 4); break;
            case FER_JIT_ARG_SCALAR_I64: std::memcpy(&store[i], &av.as.i64, 8); break;
            case FER_JIT_ARG_SCALAR_U64: std::memcpy(&store[i], &av.as.u64, 8); break;
            case FER_JIT_ARG_SCALAR_F32: std::memcpy(&store[i], &av.as.f32, 4); break;
            case FER_JIT_ARG_SCALAR_F64: std::memcpy(&store[i], &av.as.f64, 8); break;
            default: return invalid("unsupported arg kind");
        }
        params[i] = &store[i];
    }
    const cudaError_t e = cudaLaunchKernel(reinterpret_cast<const void*>(k->fn), dim3(cfg->grid_x, cfg->grid_y, cfg->grid_z),
                                           dim3(cfg->block_x, cfg->block_y, cfg->block_z),
                                           params.empty() ? nullptr : params.data(), cfg->shared_mem_bytes, S.stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return internal("kernel launch failed");
    }
    fer_status_t st = S.make_job({}, out_job);
    const uint64_t us = static_cast<uint64_t>(
        std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now() - t0).count());
    std::lock_guard<std::mutex> lk(mu_);
    stats_.launch_count++;
    stats_.launch_time_us += us;
    return st;
}

fer_status_t JitManager::cache_clear() {
    std::lock_guard<std::mutex> lk(mu_);
    cache_.clear();
    chains_.clear();
    return ok();
}

fer_status_t JitManager::stats(fer_jit_stats_t* out) {
    if (!out) return invalid("out_stats is null");
    std::lock_guard<std::mutex> lk(mu_);
    *out = stats_;
    out->memory_cache_entries = cache_.size();
    return ok();
}

fer_status_t JitManager::internal_module(const std::string& source, std::shared_ptr<Module>* out, std::string* log) {
    const int s = sm();
    const bool has_a = s == 90 || s == 100 || s == 101 || s == 103 || s == 120 || s == 121;
    std::vector<std::string> opts = {"--std=c++17", "--gpu-architecture=sm_" + std::to_string(s) + (has_a ? "a" : ""),
                                     "--fmad=false", "-default-device"};
    bool hit = false;
    return build(source, FER_JIT_SOURCE_CUDA, opts, std::getenv("FERCUDA_JIT_CACHE_DIR"), false, out, &hit, log);
}

fer_status_t JitManager::chain_kernels(const fer_chain_op_t* ops, uint32_t n_ops, uint32_t n_inputs,
                                       const ChainKernels** out) {
    // key: one byte per opcode (and the input index of a load), then the
    // input count; short chains stay within std::string's inline buffer
    std::string sig;
    for (uint32_t i = 0; i < n_ops; ++i) {
        if (ops[i].opcode > 126) return invalid("unknown chain opcode");
        if (ops[i].opcode == FER_CHAIN_LOAD && ops[i].arg >= n_inputs)
            return invalid("chain loads an input that was not bound");
        sig += static_cast<char>(ops[i].opcode + 1);
        if (ops[i].opcode == FER_CHAIN_LOAD) sig += static_cast<char>(ops[i].arg + 1);
    }
    sig += static_cast<char>(0x7f);
    sig += static_cast<char>(n_inputs);
    {
        std::lock_guard<std::mutex> lk(mu_);
        auto it = chains_.find(sig);
        if (it != chains_.end()) {
            *out = &it->second;
            return ok();
        }
    }
    std::string src, log;
    fer_status_t st = chain_source(ops, n_ops, n_inputs, &src);
    if (st.code != FER_STATUS_OK) return st;
    std::shared_ptr<Module> mod;
    st = internal_module(src, &mod, &log);
    if (st.code != FER_STATUS_OK) {
        std::lock_guard<std::mutex> lk(mu_);
        last_log_ = log;
        return st;
    }
    ChainKernels ck;
    ck.mod = mod;
    if (cudaLibraryGetKernel(&ck.v4, mod->lib, "fer_chain_v4") != cudaSuccess ||
        cudaLibraryGetKernel(&ck.s1, mod->lib, "fer_chain_s1") != cudaSuccess) {
        cudaGetLastError();
        return internal("generated chain kernel missing");
    }
    ck.fv4 = driver_function(ck.v4);
    ck.fs1 = driver_function(ck.s1);
    std::lock_guard<std::mutex> lk(mu_);
    auto res = chains_.emplace(sig, ck);
    *out = &res.first->second;
    return ok();
}

}  // namespace fer::capi

// ============================================================ C entry points

namespace {

int sm_count() {
    static const int n = [] {
        int dev = 0, v = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        return v > 0 ? v : 148;
    }();
    return n;
}

// Programmatic dependent launch: the kernel may be scheduled while the
// previous kernel on the stream drains. The chain kernels wait
// (griddepcontrol.wait) for that kernel to complete and its writes to be
// visible before any memory access the host has not cleared (launch_chain's
// `early`), and every thread waits before it exits.
bool chain_pdl_enabled() {
    static const bool pdl = [] {
        const char* e = std::getenv("FERCUDA_CHAIN_PDL");   // 0: plain launches
        return !(e && e[0] == '0');
    }();
    return pdl;
}

// FERCUDA_CHAIN_EARLY=0: the chain kernel never reads before its wait.
bool chain_early_enabled() {
    static const bool on = [] {
        const char* e = std::getenv("FERCUDA_CHAIN_EARLY");
        return !(e && e[0] == '0');
    }();
    return on;
}

cudaError_t launch_pdl(const void* fn, unsigned grid, void** args, cudaStream_t stream, void* drv = nullptr) {
    fer_pdl_note_launch();   // the chain kernels trigger their dependents however they are launched
    if (drv) {
        CUlaunchConfig cfg{};
        cfg.gridDimX = grid;
        cfg.gridDimY = 1;
        cfg.gridDimZ = 1;
        cfg.blockDimX = 256;
        cfg.blockDimY = 1;
        cfg.blockDimZ = 1;
        cfg.sharedMemBytes = 0;
        cfg.hStream = reinterpret_cast<CUstream>(stream);
        CUlaunchAttribute attr[1];
        attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
        attr[0].value.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = chain_pdl_enabled() ? 1 : 0;
        const CUresult r = fer::capi::driver_launch().launch(&cfg, reinterpret_cast<CUfunction>(drv), args, nullptr);
        return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorLaunchFailure;
    }
    if (!chain_pdl_enabled()) return cudaLaunchKernel(fn, dim3(grid), dim3(256), args, 0, stream);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// Launches a compiled chain over n elements of device streams.
fer_status_t launch_chain(Session& S, const ChainKernels& ck, const fer_chain_op_t* ops, uint32_t n_ops,
                          const float* const* in, uint32_t n_inputs, float* out, uint64_t n) {
    fer::capi::ChainParams p{};
    for (uint32_t i = 0; i < n_ops; ++i) {
        p.v[2 * i] = ops[i].p0;
        p.v[2 * i + 1] = ops[i].p1;
    }
    const void* a[4] = {nullptr, nullptr, nullptr, nullptr};
    bool aligned = (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
    for (uint32_t i = 0; i < n_inputs; ++i) {
        a[i] = in[i];
        if (reinterpret_cast<uintptr_t>(in[i]) & 15u) aligned = false;
    }
    const uint64_t cap = static_cast<uint64_t>(sm_count()) * 8;
    // Work before the dependency wait: see Session::pdl_early.
    uintptr_t in_lo[4] = {0, 0, 0, 0}, in_hi[4] = {0, 0, 0, 0};
    for (uint32_t i = 0; i < n_inputs; ++i) {
        in_lo[i] = reinterpret_cast<uintptr_t>(in[i]);
        in_hi[i] = in_lo[i] + n * sizeof(float);
    }
    const uintptr_t out_lo = reinterpret_cast<uintptr_t>(out), out_hi = out_lo + n * sizeof(float);
    unsigned early = (chain_pdl_enabled() && chain_early_enabled())
                         ? S.pdl_early(in_lo, in_hi, n_inputs, out_lo, out_hi)
                         : 0u;
    S.last_pdl.valid = false;
    uint64_t done = 0;
    if (aligned && n >= 4) {
        unsigned long long n4 = n / 4;
        uint64_t g = (n4 + 511) / 512;   // two groups per thread before the wait
        if (g > cap) g = cap;
        void* args[] = {&a[0], &a[1], &a[2], &a[3], &out, &n4, &p, &early};
        if (launch_pdl(reinterpret_cast<const void*>(ck.v4), static_cast<unsigned>(g), args, S.stream, ck.fv4) !=
            cudaSuccess) {
            cudaGetLastError();
            return internal("kernel launch failed");
        }
        done = n4 * 4;
    }
    if (done < n) {
        unsigned long long lo = done, hi = n;
        uint64_t g = (n - done + 255) / 256;
        if (g > cap) g = cap;
        void* args[] = {&a[0], &a[1], &a[2], &a[3], &out, &lo, &hi, &p};
        if (launch_pdl(reinterpret_cast<const void*>(ck.s1), static_cast<unsigned>(g), args, S.stream, ck.fs1) !=
            cudaSuccess) {
            cudaGetLastError();
            return internal("kernel launch failed");
        }
    }
    S.pdl_record(in_lo, in_hi, n_inputs, out_lo, out_hi);
    return ok();
}

// Contract check of one intent buffer, as the reference's launch would do it
// (jit_manager.cu:548-587), with the launch regime the intent runtime sets
// (AUTO -> CUSTOM_POOL, intent_runtime.cpp:311-313).
fer_status_t check_intent_buffer(const Session& S, uint64_t id, uint32_t access, uint32_t dtype, uint32_t rank,
                                 uint64_t bytes, const uint32_t* dims, uint32_t launch_regime, const Buffer** out) {
    const Buffer* b = S.find(id);
    if (!b) return not_found("buffer id not found");
    if ((access == FER_JIT_ACCESS_WRITE || access == FER_JIT_ACCESS_READ_WRITE) && b->desc.immutable)
        return invalid("immutable buffer cannot be used for write access");
    if (dtype != FER_JIT_WILDCARD_U32 && b->desc.dtype != dtype) return invalid("buffer dtype contract mismatch");
    if (rank != FER_JIT_WILDCARD_U32) {
        if (b->desc.rank != rank) return invalid("buffer rank contract mismatch");
        if (dims)
            for (uint32_t r = 0; r < rank && r < 4; ++r)
                if (dims[r] != FER_JIT_WILDCARD_U32 && b->desc.dims[r] != dims[r])
                    return invalid("buffer shape contract mismatch");
    }
    if (bytes != FER_JIT_WILDCARD_U64 && b->bytes != bytes) return invalid("buffer byte-size contract mismatch");
    if (launch_regime != FER_MEMORY_AUTO && b->regime != launch_regime)
        return invalid("buffer regime does not match launch regime");
    *out = b;
    return ok();
}

uint32_t intent_regime(const fer_jit_intent_t* it) {
    return it->memory_regime == FER_MEMORY_AUTO ? FER_MEMORY_CUSTOM_POOL : it->memory_regime;
}

fer_status_t count_launch(Session& S, fer_status_t st) {
    (void)S;
    return st;
}

fer_status_t run_affine(Session& S, const fer_jit_intent_t* it, const fer_jit_intent_bindings_t* bd, uint64_t* job) {
    if (it->n == 0) return invalid("intent n must be > 0");
    const uint32_t reg = intent_regime(it);
    const uint32_t dims[1] = {it->n};
    const Buffer *in = nullptr, *out = nullptr;
    fer_status_t st = check_intent_buffer(S, bd->input, FER_JIT_ACCESS_READ, FER_DTYPE_F32, 1,
                                          static_cast<uint64_t>(it->n) * 4, dims, reg, &in);
    if (st.code != FER_STATUS_OK) return st;
    st = check_intent_buffer(S, bd->output, FER_JIT_ACCESS_WRITE, FER_DTYPE_F32, 1, static_cast<uint64_t>(it->n) * 4,
                             dims, reg, &out);
    if (st.code != FER_STATUS_OK) return st;
    if (it->fusion_mask & ~(FER_JIT_INTENT_FUSION_RELU | FER_JIT_INTENT_FUSION_MUL_SIGMOID_INPUT))
        return invalid("unsupported fusion bits");
    fer_chain_op_t ops[6];
    uint32_t n = 0;
    ops[n++] = fer_chain_op_t{FER_CHAIN_LOAD, 0, 0.f, 0.f};
    if (it->fusion_mask & FER_JIT_INTENT_FUSION_MUL_SIGMOID_INPUT) {
        // relu(a*x + b) * sigmoid(x) with the native kernels' rounding:
        // k_affine_f32 (mul, add), k_relu_f32 (fmaxf), k_sigmoid_f32, k_mul_f32.
        ops[n++] = fer_chain_op_t{FER_CHAIN_AFFINE, 0, it->alpha, it->beta};
        if (it->fusion_mask & FER_JIT_INTENT_FUSION_RELU) ops[n++] = fer_chain_op_t{FER_CHAIN_RELU, 0, 0.f, 0.f};
        ops[n++] = fer_chain_op_t{FER_CHAIN_LOAD, 0, 0.f, 0.f};
        ops[n++] = fer_chain_op_t{FER_CHAIN_SIGMOID, 0, 0.f, 0.f};
        ops[n++] = fer_chain_op_t{FER_CHAIN_MUL, 0, 0.f, 0.f};
    } else {
        // The reference's affine intent kernel `alpha * in + beta`, built by
        // NVRTC with FMA contraction on (intent_runtime.cpp:58-68,
        // jit_manager.cu:379-391): one fused multiply-add; relu as `v < 0 ? 0 : v`.
        ops[n++] = fer_chain_op_t{FER_CHAIN_FMA, 0, it->alpha, it->beta};
        if (it->fusion_mask & FER_JIT_INTENT_FUSION_RELU) ops[n++] = fer_chain_op_t{FER_CHAIN_RELU_LT, 0, 0.f, 0.f};
    }
    const ChainKernels* ck = nullptr;
    st = S.jit->chain_kernels(ops, n, 1, &ck);
    if (st.code != FER_STATUS_OK) return st;
    const float* ins[1] = {static_cast<const float*>(in->ptr)};
    st = launch_chain(S, *ck, ops, n, ins, 1, static_cast<float*>(out->ptr), it->n);
    if (st.code != FER_STATUS_OK) return st;
    return S.make_job({}, job);
}

fer_status_t run_softmax(Session& S, const fer_jit_intent_t* it, const fer_jit_intent_bindings_t* bd, uint64_t* job) {
    if (it->n == 0) return invalid("intent n (cols) must be > 0");
    const uint32_t rows = it->height ? it->height : 1;
    const uint64_t bytes = static_cast<uint64_t>(rows) * it->n * 4;
    const uint32_t reg = intent_regime(it);
    const Buffer *in = nullptr, *out = nullptr;
    fer_status_t st = check_intent_buffer(S, bd->input, FER_JIT_ACCESS_READ, FER_DTYPE_F32, FER_JIT_WILDCARD_U32,
                                          bytes, nullptr, reg, &in);
    if (st.code != FER_STATUS_OK) return st;
    st = check_intent_buffer(S, bd->output, FER_JIT_ACCESS_WRITE, FER_DTYPE_F32, FER_JIT_WILDCARD_U32, bytes, nullptr,
                             reg, &out);
    if (st.code != FER_STATUS_OK) return st;
    // 1 = softmax, 4 = the intent kernel's reduction order.
    if (fer_rows_f32(static_cast<const float*>(in->ptr), static_cast<float*>(out->ptr), nullptr, nullptr,
                     static_cast<int>(rows), static_cast<int>(it->n), 0.0f, 1u | 4u, S.dev_err, S.stream) != cudaSuccess) {
        cudaGetLastError();
        return internal("kernel launch failed");
    }
    return S.make_job({}, job);
}

fer_status_t run_reduce(Session& S, const fer_jit_intent_t* it, const fer_jit_intent_bindings_t* bd, uint64_t* job,
                        bool is_max) {
    if (it->n == 0) return invalid("intent n must be > 0");
    const uint32_t reg = intent_regime(it);
    const Buffer *in = nullptr, *out = nullptr;
    fer_status_t st = check_intent_buffer(S, bd->input, FER_JIT_ACCESS_READ, FER_DTYPE_F32, 1,
                                          static_cast<uint64_t>(it->n) * 4, nullptr, reg, &in);
    if (st.code != FER_STATUS_OK) return st;
    st = check_intent_buffer(S, bd->output, FER_JIT_ACCESS_READ_WRITE, FER_DTYPE_F32, 1, 4, nullptr, reg, &out);
    if (st.code != FER_STATUS_OK) return st;
    Temp scratch{};
    st = S.alloc_temp(fer_reduce_scratch_floats(it->n) * 4, it->memory_regime, &scratch);
    if (st.code != FER_STATUS_OK) return st;
    if (fer_reduce_f32(static_cast<const float*>(in->ptr), static_cast<float*>(out->ptr),
                       static_cast<float*>(scratch.ptr), it->n, is_max ? 1 : 0, S.stream) != cudaSuccess) {
        cudaGetLastError();
        S.free_bytes(scratch.ptr, scratch.regime, scratch.tier, scratch.bytes);
        return internal("kernel launch failed");
    }
    return S.make_job({scratch}, job);
}

fer_status_t run_conv2d(Session& S, const fer_jit_intent_t* it, const fer_jit_intent_bindings_t* bd, uint64_t* job) {
    if (it->height == 0 || it->width == 0 || it->channels == 0)
        return invalid("conv2d requires height, width, channels > 0");
    if (it->kernel_h == 0 || it->kernel_w == 0 || it->num_filters == 0)
        return invalid("conv2d requires kernel_h, kernel_w, num_filters > 0");
    const uint32_t H = it->height, W = it->width, C = it->channels, KH = it->kernel_h, KW = it->kernel_w,
                   F = it->num_filters;
    const uint32_t sh = it->stride_h ? it->stride_h : 1, sw = it->stride_w ? it->stride_w : 1;
    if (H + 2 * it->pad_h < KH || W + 2 * it->pad_w < KW) return invalid("conv2d kernel larger than padded input");
    const uint32_t oh = (H + 2 * it->pad_h - KH) / sh + 1, ow = (W + 2 * it->pad_w - KW) / sw + 1;
    const uint32_t reg = intent_regime(it);
    const Buffer *in = nullptr, *w = nullptr, *b = nullptr, *out = nullptr;
    fer_status_t st = check_intent_buffer(S, bd->input, FER_JIT_ACCESS_READ, FER_DTYPE_F32, FER_JIT_WILDCARD_U32,
                                          static_cast<uint64_t>(H) * W * C * 4, nullptr, reg, &in);
    if (st.code != FER_STATUS_OK) return st;
    st = check_intent_buffer(S, bd->weights, FER_JIT_ACCESS_READ, FER_DTYPE_F32, FER_JIT_WILDCARD_U32,
                             static_cast<uint64_t>(F) * C * KH * KW * 4, nullptr, reg, &w);
    if (st.code != FER_STATUS_OK) return st;
    if (bd->bias) {
        st = check_intent_buffer(S, bd->bias, FER_JIT_ACCESS_READ, FER_DTYPE_F32, FER_JIT_WILDCARD_U32,
                                 static_cast<uint64_t>(F) * 4, nullptr, reg, &b);
        if (st.code != FER_STATUS_OK) return st;
    }
    st = check_intent_buffer(S, bd->output, FER_JIT_ACCESS_WRITE, FER_DTYPE_F32, FER_JIT_WILDCARD_U32,
                             static_cast<uint64_t>(oh) * ow * F * 4, nullptr, reg, &out);
    if (st.code != FER_STATUS_OK) return st;
    if (fer_conv2d_f32(static_cast<const float*>(in->ptr), static_cast<const float*>(w->ptr),
                       b ? static_cast<const float*>(b->ptr) : nullptr, static_cast<float*>(out->ptr), H, W, C, KH, KW,
                       F, it->pad_h, it->pad_w, sh, sw, (it->fusion_mask & FER_JIT_INTENT_FUSION_RELU) ? 1 : 0,
                       S.stream) != cudaSuccess) {
        cudaGetLastError();
        return internal("kernel launch failed");
    }
    return S.make_job({}, job);
}

}  // namespace

#define FER_JIT_SESSION(s)                                        \
    if (!(s) || !(s)->impl.jit) return invalid("session is null"); \
    Session& S = (s)->impl

extern "C" {

fer_status_t fer_jit_compile(fer_session_t* session, const fer_jit_source_t* source, const fer_jit_options_t* options,
                             fer_jit_program_t* out_program, fer_jit_compile_result_t* out_result) {
    FER_JIT_SESSION(session);
    return S.jit->compile(source, options, out_program, out_result);
}

fer_status_t fer_jit_release_program(fer_session_t* session, fer_jit_program_t program) {
    FER_JIT_SESSION(session);
    return S.jit->release_program(program);
}

fer_status_t fer_jit_get_kernel(fer_session_t* session, fer_jit_program_t program, const char* kernel_name,
                                const fer_jit_kernel_sig_t* signature, fer_jit_kernel_t* out_kernel) {
    FER_JIT_SESSION(session);
    return S.jit->get_kernel(program, kernel_name, signature, out_kernel);
}

fer_status_t fer_jit_release_kernel(fer_session_t* session, fer_jit_kernel_t kernel) {
    FER_JIT_SESSION(session);
    return S.jit->release_kernel(kernel);
}

fer_status_t fer_jit_launch(fer_session_t* session, fer_jit_kernel_t kernel, const fer_jit_launch_cfg_t* cfg,
                            const fer_jit_arg_pack_t* args, uint64_t* out_job_id) {
    FER_JIT_SESSION(session);
    return S.jit->launch(kernel, cfg, args, out_job_id);
}

fer_status_t fer_jit_cache_clear(fer_session_t* session) {
    FER_JIT_SESSION(session);
    return S.jit->cache_clear();
}

fer_status_t fer_jit_get_stats(fer_session_t* session, fer_jit_stats_t* out_stats) {
    FER_JIT_SESSION(session);
    return S.jit->stats(out_stats);
}

fer_status_t fer_jit_run_intent(fer_session_t* session, const fer_jit_intent_t* intent,
                                const fer_jit_intent_bindings_t* bindings, uint64_t* out_job_id) {
    if (!session) return invalid("session is null");
    if (!intent) return invalid("intent is null");
    if (!bindings) return invalid("bindings are null");
    if (!out_job_id) return invalid("out_job_id is null");
    if (intent->abi_version != FER_JIT_INTENT_ABI_VERSION) return invalid("intent ABI mismatch");
    Session& S = session->impl;
    if (intent->caps_mask & ~(FER_JIT_INTENT_CAPS_REQUIRE_TENSOR_CORES | FER_JIT_INTENT_CAPS_REQUIRE_COOP_GROUPS))
        return invalid("unsupported capability bits");
    switch (intent->op) {
        case FER_JIT_INTENT_OP_AFFINE_F32: return count_launch(S, run_affine(S, intent, bindings, out_job_id));
        case FER_JIT_INTENT_OP_SOFTMAX_F32: return count_launch(S, run_softmax(S, intent, bindings, out_job_id));
        case FER_JIT_INTENT_OP_REDUCE_SUM_F32: return count_launch(S, run_reduce(S, intent, bindings, out_job_id, false));
        case FER_JIT_INTENT_OP_REDUCE_MAX_F32: return count_launch(S, run_reduce(S, intent, bindings, out_job_id, true));
        case FER_JIT_INTENT_OP_CONV2D_F32: return count_launch(S, run_conv2d(S, intent, bindings, out_job_id));
        default: return invalid("unsupported intent op");
    }
}

fer_status_t fer_tensor_run_affine_f32(fer_session_t* session, fer_tensor_handle_t input, fer_tensor_handle_t output,
                                       uint32_t n, float alpha, float beta, uint32_t fusion_mask, uint32_t caps_mask,
                                       uint32_t memory_regime, uint64_t* out_job_id) {
    fer_jit_intent_t it{};
    it.abi_version = FER_JIT_INTENT_ABI_VERSION;
    it.op = FER_JIT_INTENT_OP_AFFINE_F32;
    it.fusion_mask = fusion_mask;
    it.caps_mask = caps_mask;
    it.memory_regime = memory_regime;
    it.n = n;
    it.alpha = alpha;
    it.beta = beta;
    fer_jit_intent_bindings_t b{};
    b.input = input.id;
    b.output = output.id;
    return fer_jit_run_intent(session, &it, &b, out_job_id);
}

fer_status_t fer_jit_run_chain_f32(fer_session_t* session, const fer_chain_op_t* ops, uint32_t n_ops,
                                   const uint64_t* inputs, uint32_t n_inputs, uint64_t output, uint64_t* out_job_id) {
    FER_JIT_SESSION(session);
    if (!ops || n_ops == 0) return invalid("chain is empty");
    if (n_inputs == 0 || n_inputs > FER_CHAIN_MAX_INPUTS || !inputs) return invalid("chain needs 1..4 inputs");
    const Buffer* o = S.find(output);
    if (!o) return not_found("buffer id not found");
    if (o->desc.dtype != FER_DTYPE_F32) return invalid("chain buffers must be f32");
    if (o->desc.immutable) return invalid("immutable buffer cannot be used for write access");
    const float* ins[FER_CHAIN_MAX_INPUTS] = {nullptr, nullptr, nullptr, nullptr};
    for (uint32_t i = 0; i < n_inputs; ++i) {
        const Buffer* b = S.find(inputs[i]);
        if (!b) return not_found("buffer id not found");
        if (b->desc.dtype != FER_DTYPE_F32) return invalid("chain buffers must be f32");
        if (b->numel != o->numel) return invalid("chain buffers must have the same element count");
        ins[i] = static_cast<const float*>(b->ptr);
    }
    const ChainKernels* ck = nullptr;
    fer_status_t st = S.jit->chain_kernels(ops, n_ops, n_inputs, &ck);
    if (st.code != FER_STATUS_OK) return st;
    st = launch_chain(S, *ck, ops, n_ops, ins, n_inputs, static_cast<float*>(o->ptr), o->numel);
    if (st.code != FER_STATUS_OK) return st;
    return S.make_job({}, out_job_id);
}

}  // extern "C"
