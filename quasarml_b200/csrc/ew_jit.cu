// Runtime-compiled fused elementwise kernels.
//
// Reference: the reference generates a GLSL compute shader per op at run time
// (Ops/ShaderGen.cpp:40-66) and compiles it with shaderc
// (Backend/Vulkan/VulkanBackend.cpp:44-80), caching pipelines per shader.
// Here the generated code is CUDA for a whole fused expression: NVRTC
// compiles it for sm_100a on first use and the cubin is loaded through the
// driver API; kernels are cached per device and expression signature.
//
// The generated kernel is straight-line code: each thread loads 16 elements
// of every input (16-byte vectors for inputs contiguous along the inner dim,
// one value per row for inputs broadcast along it), evaluates the DAG node by
// node in registers, and stores one vector per 16 bytes of output.  The node
// bodies are the operator functors of ew_ops.cuh, embedded verbatim as source
// text, each result rounded to the storage dtype, so results are
// bit-identical to the per-op kernels and to the interpreter.
//
// NVRTC is opened with dlopen and the driver entry points are fetched from
// the runtime; if either is missing the caller falls back to the precompiled
// interpreter kernel.
#include "ew_jit.cuh"

#include <cuda.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <cinttypes>
#include <sstream>
#include <unordered_map>
#include <vector>

namespace qsml {
namespace {

const char kOpsSource[] =
#include "ew_ops_src.inc"
    ;

constexpr int kJitThreads = 256;
constexpr int kJitElems = 16;  // elements per thread

// ---------------------------------------------------------------------------
// NVRTC and driver entry points
// ---------------------------------------------------------------------------
struct Rtc {
    bool ok = false;
    nvrtcResult (*create)(nvrtcProgram*, const char*, const char*, int, const char* const*, const char* const*);
    nvrtcResult (*compile)(nvrtcProgram, int, const char* const*);
    nvrtcResult (*log_size)(nvrtcProgram, size_t*);
    nvrtcResult (*log)(nvrtcProgram, char*);
    nvrtcResult (*cubin_size)(nvrtcProgram, size_t*);
    nvrtcResult (*cubin)(nvrtcProgram, char*);
    nvrtcResult (*destroy)(nvrtcProgram*);
    CUresult (*load)(CUmodule*, const void*);
    CUresult (*get_function)(CUfunction*, CUmodule, const char*);
    CUresult (*launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, CUstream,
                       void**, void**);
    // cuLaunchKernelEx, for programmatic dependent launch; null if absent
    CUresult (*launch_ex)(const CUlaunchConfig*, CUfunction, void**, void**) = nullptr;
    std::string why;  // reason when !ok
};

template <typename F> bool sym(void* lib, const char* name, F* out) {
    *out = reinterpret_cast<F>(dlsym(lib, name));
    return *out != nullptr;
}

template <typename F> bool drv(const char* name, F* out) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess) {
        cudaGetLastError();
        return false;
    }
    *out = reinterpret_cast<F>(p);
    return true;
}

const Rtc& rtc() {
    static Rtc r = [] {
        Rtc t;
        void* lib = dlopen("libnvrtc.so.12", RTLD_NOW | RTLD_LOCAL);
        if (!lib) lib = dlopen("libnvrtc.so", RTLD_NOW | RTLD_LOCAL);
        if (!lib) {
            t.why = "libnvrtc not found";
            return t;
        }
        bool ok = sym(lib, "nvrtcCreateProgram", &t.create) && sym(lib, "nvrtcCompileProgram", &t.compile) &&
                  sym(lib, "nvrtcGetProgramLogSize", &t.log_size) && sym(lib, "nvrtcGetProgramLog", &t.log) &&
                  sym(lib, "nvrtcGetCUBINSize", &t.cubin_size) && sym(lib, "nvrtcGetCUBIN", &t.cubin) &&
                  sym(lib, "nvrtcDestroyProgram", &t.destroy);
        ok = ok && drv("cuModuleLoadData", &t.load) && drv("cuModuleGetFunction", &t.get_function) &&
             drv("cuLaunchKernel", &t.launch);
        if (!drv("cuLaunchKernelEx", &t.launch_ex)) t.launch_ex = nullptr;
        t.ok = ok;
        if (!ok) t.why = "NVRTC or driver entry points missing";
        return t;
    }();
    return r;
}

// ---------------------------------------------------------------------------
// Source generation
// ---------------------------------------------------------------------------
std::string prologue() {
    std::ostringstream s;
    s << "typedef int int32_t;\ntypedef unsigned int uint32_t;\n#define INT32_MIN (-2147483647 - 1)\n";
    s << "#define QSML_OP_ADD " << QSML_OP_ADD << "\n#define QSML_OP_SUB " << QSML_OP_SUB << "\n#define QSML_OP_MUL "
      << QSML_OP_MUL << "\n#define QSML_OP_DIV " << QSML_OP_DIV << "\n#define QSML_OP_POW " << QSML_OP_POW << "\n";
    const std::pair<const char*, int> un[] = {
        {"RELU", QSML_UN_RELU}, {"NEG", QSML_UN_NEG},   {"ABS", QSML_UN_ABS},   {"SQRT", QSML_UN_SQRT},
        {"EXP", QSML_UN_EXP},   {"LOG", QSML_UN_LOG},   {"SIN", QSML_UN_SIN},   {"COS", QSML_UN_COS},
        {"TANH", QSML_UN_TANH}, {"SIGMOID", QSML_UN_SIGMOID}, {"GELU", QSML_UN_GELU}};
    for (const auto& u : un) s << "#define QSML_UN_" << u.first << " " << u.second << "\n";
    return s.str();
}

// binary16 <-> binary32 with the conversions cuda_fp16's __half2float /
// __float2half_rn use.
const char kHalfHelpers[] = R"(
__device__ __forceinline__ float qsml_h2f(unsigned short h) { float f; asm("cvt.f32.f16 %0, %1;" : "=f"(f) : "h"(h)); return f; }
__device__ __forceinline__ unsigned short qsml_f2h(float f) { unsigned short h; asm("cvt.rn.f16.f32 %0, %1;" : "=h"(h) : "f"(f)); return h; }
__device__ __forceinline__ float qsml_rh(float f) { return qsml_h2f(qsml_f2h(f)); }
)";

// Compact signature of what the generated code depends on.
std::string signature(const qsml_fuse_node* nodes, int n, const JitInput* ins, int nin, bool half) {
    std::ostringstream k;
    k << (half ? 'h' : 'f') << nin << ':';
    for (int j = 0; j < nin; ++j) k << (ins[j].vec ? 'v' : 'b');
    for (int i = 0; i < n; ++i) {
        uint32_t bits;
        std::memcpy(&bits, &nodes[i].value, 4);
        k << ';' << nodes[i].kind << ',' << nodes[i].code << ',' << nodes[i].a << ',' << nodes[i].b;
        if (nodes[i].kind == QSML_FUSE_CONST) k << ',' << bits;
    }
    return k.str();
}

std::string generate(const qsml_fuse_node* nodes, int n, const JitInput* ins, int nin, bool half) {
    const int V = half ? 8 : 4;
    const int U = kJitElems / V;
    const char* T = half ? "unsigned short" : "float";
    std::ostringstream s;
    s << prologue() << kOpsSource << "\nusing namespace qsml::ew;\n";
    if (half) s << kHalfHelpers;
    s << "extern \"C\" __global__ void __launch_bounds__(" << kJitThreads << ") qsml_fused_kernel(";
    for (int j = 0; j < nin; ++j) s << "const " << T << "* __restrict__ p" << j << ", long long r" << j << ", ";
    s << T << "* __restrict__ out, unsigned items, unsigned cpr, unsigned magic, unsigned sh1, unsigned sh2, "
         "int defer) {\n";
    // programmatic dependent launch: wait for the previous kernel on the
    // stream before touching memory (at the end instead when the launch
    // overlaps it, see plan_launch), then let the next one launch
    s << "  if (!defer) asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n";
    s << "  asm volatile(\"griddepcontrol.launch_dependents;\" ::: \"memory\");\n";
    s << "  const int V = " << V << ", U = " << U << ";\n";
    s << "  const unsigned base = blockIdx.x * (" << kJitThreads << "u * U) + threadIdx.x;\n";
    for (int j = 0; j < nin; ++j) s << "  float x" << j << "[U * V];\n";
    s << "  bool ok[U];\n  unsigned its[U];\n";
    s << "#pragma unroll\n  for (int u = 0; u < U; ++u) {\n";
    s << "    const unsigned it = base + u * " << kJitThreads << "u;\n";
    s << "    ok[u] = it < items;\n    its[u] = it;\n";
    // row = it / cpr by multiply-high (Granlund-Montgomery, exact for 32-bit it)
    s << "    const unsigned t1 = __umulhi(magic, it);\n";
    s << "    const unsigned row = ok[u] ? (t1 + ((it - t1) >> sh1)) >> sh2 : 0u;\n    const unsigned cv = it - row * cpr;\n";
    for (int j = 0; j < nin; ++j) {
        if (ins[j].vec) {
            s << "    { const uint4 w = ok[u] ? *reinterpret_cast<const uint4*>(p" << j << " + (long long)row * r" << j
              << " + (long long)cv * V) : make_uint4(0u, 0u, 0u, 0u);\n";
            if (half) {
                const char* c[4] = {"w.x", "w.y", "w.z", "w.w"};
                for (int q = 0; q < 4; ++q)
                    s << "      x" << j << "[u * V + " << 2 * q << "] = qsml_h2f((unsigned short)(" << c[q]
                      << " & 0xffffu)); x" << j << "[u * V + " << 2 * q + 1 << "] = qsml_h2f((unsigned short)("
                      << c[q] << " >> 16));\n";
            } else {
                s << "      x" << j << "[u * V + 0] = __uint_as_float(w.x); x" << j
                  << "[u * V + 1] = __uint_as_float(w.y); x" << j << "[u * V + 2] = __uint_as_float(w.z); x" << j
                  << "[u * V + 3] = __uint_as_float(w.w);\n";
            }
            s << "    }\n";
        } else {
            s << "    { const float v = ok[u] ? " << (half ? "qsml_h2f(" : "(") << "p" << j << "[(long long)row * r" << j
              << "]) : 0.0f;\n#pragma unroll\n      for (int e = 0; e < V; ++e) x" << j << "[u * V + e] = v; }\n";
        }
    }
    s << "  }\n  float y[U * V];\n#pragma unroll\n  for (int e = 0; e < U * V; ++e) {\n";
    const char* R = half ? "qsml_rh" : "";
    for (int i = 0; i < n; ++i) {
        const qsml_fuse_node& d = nodes[i];
        s << "    const float n" << i << " = ";
        switch (d.kind) {
            case QSML_FUSE_INPUT: s << "x" << d.code << "[e];\n"; break;
            case QSML_FUSE_CONST: {
                uint32_t bits;
                std::memcpy(&bits, &d.value, 4);
                s << "__uint_as_float(0x" << std::hex << bits << std::dec << "u);\n";
                break;
            }
            case QSML_FUSE_BINARY:
                s << R << "(BinOp<" << d.code << ">()(n" << d.a << ", n" << d.b << "));\n";
                break;
            default: s << R << "(UnOp<" << d.code << ">()(n" << d.a << "));\n"; break;
        }
    }
    s << "    y[e] = n" << n - 1 << ";\n  }\n";
    s << "#pragma unroll\n  for (int u = 0; u < U; ++u) {\n    if (!ok[u]) continue;\n";
    if (half) {
        s << "    uint4 w;\n";
        const char* c[4] = {"w.x", "w.y", "w.z", "w.w"};
        for (int q = 0; q < 4; ++q)
            s << "    " << c[q] << " = (unsigned)qsml_f2h(y[u * V + " << 2 * q << "]) | ((unsigned)qsml_f2h(y[u * V + "
              << 2 * q + 1 << "]) << 16);\n";
    } else {
        s << "    uint4 w = make_uint4(__float_as_uint(y[u * V + 0]), __float_as_uint(y[u * V + 1]), "
             "__float_as_uint(y[u * V + 2]), __float_as_uint(y[u * V + 3]));\n";
    }
    s << "    *reinterpret_cast<uint4*>(out + (long long)its[u] * V) = w;\n  }\n";
    s << "  if (defer) asm volatile(\"griddepcontrol.wait;\" ::: \"memory\");\n}\n";
    return s.str();
}

// ---------------------------------------------------------------------------
// Cache
// ---------------------------------------------------------------------------
std::mutex g_mu;
std::unordered_map<std::string, CUfunction> g_kernels;  // "<device>|<signature>" -> kernel
std::unordered_map<std::string, bool> g_failed;         // signatures that did not compile
uint64_t g_compiled = 0;

bool compile(const Rtc& r, const std::string& src, CUfunction* fn, std::string* err) {
    nvrtcProgram prog;
    if (r.create(&prog, src.c_str(), "qsml_fused.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS) {
        *err = "nvrtcCreateProgram failed";
        return false;
    }
    const char* opts[] = {"--gpu-architecture=sm_100a", "-std=c++17", "--fmad=false"};
    const nvrtcResult cr = r.compile(prog, 3, opts);
    if (cr != NVRTC_SUCCESS) {
        size_t n = 0;
        r.log_size(prog, &n);
        std::string log(n, '\0');
        if (n) r.log(prog, &log[0]);
        *err = "NVRTC: " + log.substr(0, 2000);
        r.destroy(&prog);
        return false;
    }
    size_t n = 0;
    r.cubin_size(prog, &n);
    std::vector<char> cubin(n);
    r.cubin(prog, cubin.data());
    r.destroy(&prog);
    CUmodule mod;
    if (r.load(&mod, cubin.data()) != CUDA_SUCCESS) {
        *err = "cuModuleLoadData failed";
        return false;
    }
    if (r.get_function(fn, mod, "qsml_fused_kernel") != CUDA_SUCCESS) {
        *err = "cuModuleGetFunction failed";
        return false;
    }
    return true;
}

}  // namespace

uint64_t fused_jit_kernels() {
    std::lock_guard<std::mutex> lk(g_mu);
    return g_compiled;
}

qsml_status_t fused_jit(Context* ctx, const qsml_fuse_node* nodes, int n_nodes, const JitInput* ins, int nin,
                        bool half, void* out, int64_t items, int64_t cpr, bool* ran) {
    *ran = false;
    const Rtc& r = rtc();
    if (!r.ok || nin < 1 || items <= 0 || items >= (int64_t(1) << 31)) return QSML_OK;
    const std::string sig = signature(nodes, n_nodes, ins, nin, half);
    const std::string key = std::to_string(ctx->device) + "|" + sig;
    CUfunction fn = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_kernels.find(key);
        if (it != g_kernels.end()) fn = it->second;
        else if (g_failed.count(key)) return QSML_OK;
    }
    if (!fn) {
        std::string err;
        CUfunction f = nullptr;
        const bool good = compile(r, generate(nodes, n_nodes, ins, nin, half), &f, &err);
        std::lock_guard<std::mutex> lk(g_mu);
        if (!good) {
            g_failed[key] = true;
            return QSML_OK;  // the interpreter runs this expression
        }
        auto ins_it = g_kernels.emplace(key, f);
        if (ins_it.second) ++g_compiled;
        fn = ins_it.first->second;
    }
    std::vector<void*> args;
    std::vector<const void*> ptrs(nin);
    std::vector<long long> strides(nin);
    unsigned items32 = static_cast<unsigned>(items), cpr32 = static_cast<unsigned>(cpr);
    // Division by cpr as (t1 + ((n - t1) >> sh1)) >> sh2, t1 = mulhi(magic, n)
    // (Granlund & Montgomery 1994, unsigned division by invariant integers):
    // l = ceil(log2 cpr), magic = floor(2^32 (2^l - cpr) / cpr) + 1.
    unsigned l = 0;
    while ((uint64_t(1) << l) < cpr32) ++l;
    unsigned magic = static_cast<unsigned>(((uint64_t(1) << 32) * ((uint64_t(1) << l) - cpr32)) / cpr32 + 1);
    unsigned sh1 = l < 1 ? l : 1, sh2 = l > 1 ? l - 1 : 0;
    void* outp = out;
    for (int j = 0; j < nin; ++j) {
        ptrs[j] = ins[j].ptr;
        strides[j] = static_cast<long long>(ins[j].row_stride);
    }
    for (int j = 0; j < nin; ++j) {
        args.push_back(&ptrs[j]);
        args.push_back(&strides[j]);
    }
    args.push_back(&outp);
    args.push_back(&items32);
    args.push_back(&cpr32);
    args.push_back(&magic);
    args.push_back(&sh1);
    args.push_back(&sh2);
    const int per_block = kJitThreads * (kJitElems / (half ? 8 : 4));
    const int64_t blocks = (items + per_block - 1) / per_block;
    // what the launch reads and writes, for overlap with the kernels before it
    const size_t es = half ? 2 : 4;
    const int64_t rows = items / cpr;
    Footprint fp;
    for (int j = 0; j < nin; ++j)
        fp.read(span_of(ins[j].ptr, static_cast<size_t>((rows - 1) * ins[j].row_stride +
                                                        (ins[j].vec ? cpr * (half ? 8 : 4) : 1)) * es));
    fp.write(span_of(out, static_cast<size_t>(items) * (half ? 8 : 4) * es));
    int defer = r.launch_ex ? plan_launch(ctx, fp) : 0;
    args.push_back(&defer);
    CUresult lr;
    if (r.launch_ex) {
        CUlaunchAttribute attr[1];
        std::memset(attr, 0, sizeof(attr));
        attr[0].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
        attr[0].value.programmaticStreamSerializationAllowed = 1;
        CUlaunchConfig cfg;
        std::memset(&cfg, 0, sizeof(cfg));
        cfg.gridDimX = static_cast<unsigned>(blocks);
        cfg.gridDimY = cfg.gridDimZ = 1;
        cfg.blockDimX = kJitThreads;
        cfg.blockDimY = cfg.blockDimZ = 1;
        cfg.sharedMemBytes = 0;
        cfg.hStream = reinterpret_cast<CUstream>(ctx->stream);
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        lr = r.launch_ex(&cfg, fn, args.data(), nullptr);
    } else {
        lr = r.launch(fn, static_cast<unsigned>(blocks), 1, 1, kJitThreads, 1, 1, 0,
                      reinterpret_cast<CUstream>(ctx->stream), args.data(), nullptr);
    }
    if (lr != CUDA_SUCCESS) {
        ctx->planned_for = 0;
        end_window(ctx->stream);
        return set_error(ctx, QSML_E_CUDA, "launch of the fused kernel failed (CUresult " + std::to_string(lr) + ")");
    }
    *ran = true;
    return after_launch(ctx, "qsml_fused_kernel");
}

}  // namespace qsml
