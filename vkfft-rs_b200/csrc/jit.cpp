// Run-time specialised pass kernels.  The op-program interpreter (kernels.cu) reads every
// size, stride and radix of a pass from its parameters; here each generic pass gets its own
// kernel in which all of them are compile-time constants, so index arithmetic folds,
// loops have constant trip counts and only the stages the pass uses are instantiated.
// The kernel calls the same op functions (pass_device.cuh) as the interpreter.  Sources
// are compiled once per process with NVRTC for sm_100a and loaded with the runtime's
// library API (context independent); any failure leaves the pass on the interpreter.
//
// B200FFT_JIT=0 disables it, B200FFT_JIT=require turns a compile failure into an error.
#include <cuda_runtime.h>
#include <nvrtc.h>

#include <cinttypes>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include "program.hpp"

namespace b200fft {

extern const int kJitHeaderCount;
extern const char *const kJitHeaderNames[];
extern const char *const kJitHeaderSources[];

namespace {

std::string side_literal(const Side &s) {
    char b[256];
    std::snprintf(b, sizeof b, "Side{%" PRId64 "LL, %" PRId64 "LL, %" PRId64 "LL, %" PRId64 "LL, %d, %d, %d, %d, %d, 0}",
                  (int64_t)s.os, (int64_t)s.is, (int64_t)s.cs, (int64_t)s.es, s.real, s.count, s.cm, s.em, s.herm);
    return b;
}

std::string fastdiv_literal(const FastDiv &f) {
    char b[96];
    std::snprintf(b, sizeof b, "FastDiv{%uu, %uu, %uu, 0u}", f.d, f.m, f.s);
    return b;
}

bool stage_radix_supported(int r) { return (r >= 2 && r <= 13) || r == 16; }

}  // namespace

// CUDA C++ source of the specialised kernel of one pass, or "" when a pass uses
// something the generator does not specialise.
std::string jit_pass_source(const PassPlan &pp, int scalar_kind) {
    const PassParams &p = pp.p;
    std::ostringstream o;
    o << "#define B200FFT_NT " << pp.threads << "\n#include \"pass_device.cuh\"\nusing namespace b200fft;\n"
      << "extern \"C\" __global__ void __launch_bounds__(" << pp.threads
      << ") b200fft_pass(const __grid_constant__ PassParams p) {\n"
      << "  typedef " << (scalar_kind == 2 ? "b200fft::dd" : scalar_kind == 1 ? "double" : "float") << " T;\n"
      << "  extern __shared__ __align__(16) unsigned char smem_raw[];\n"
      << "  cplx<T> *sm = reinterpret_cast<cplx<T> *>(smem_raw);\n"
      << "  PassShape sh = p;\n"
      << "  sh.nlines = " << p.nlines << "LL; sh.ni = " << p.ni << "LL; sh.nc = " << p.nc << "LL;\n"
      << "  sh.G = " << p.G << "; sh.nops = " << p.nops << "; sh.line_len = " << p.line_len
      << "; sh.line_stride = " << p.line_stride << "; sh.meta_off = " << p.meta_off << ";\n"
      << "  sh.div_g = " << fastdiv_literal(p.div_g) << ";\n"
      << "  sh.in = " << side_literal(p.in) << ";\n"
      << "  sh.out = " << side_literal(p.out) << ";\n";
    if (!pp.peer_scatter) o << "  sh.peer.n = 0;\n";
    o << "  const LineMeta lm = pass_prologue<T>(sh, smem_raw);\n  __syncthreads();\n";
    char num[64];
    for (int k = 0; k < p.nops; k++) {
        const Op &op = p.ops[k];
        o << "  {\n    Op op = p.ops[" << k << "];\n"
          << "    op.type = " << op.type << "; op.flags = " << op.flags << "; op.radix = " << op.radix
          << "; op.P = " << op.P << "; op.len = " << op.len << "; op.nsub = " << op.nsub << ";\n"
          << "    op.src_base = " << op.src_base << "; op.dst_base = " << op.dst_base
          << "; op.sub_stride = " << op.sub_stride << "; op.mul = " << op.mul << "; op.cm = " << op.cm
          << "; op.em = " << op.em << ";\n"
          << "    op.w_base = " << op.w_base << "; op.w_stride = " << op.w_stride << "; op.x0_base = " << op.x0_base
          << "; op.nfull = " << op.nfull << "; op.pad_shift = " << op.pad_shift << ";\n"
          << "    op.div_a = " << fastdiv_literal(op.div_a) << "; op.div_b = " << fastdiv_literal(op.div_b)
          << "; op.div_c = " << fastdiv_literal(op.div_c) << ";\n";
        std::snprintf(num, sizeof num, "%a", op.scale);
        o << "    op.scale = " << num << ";";
        std::snprintf(num, sizeof num, "%a", op.scale_lo);
        o << " op.scale_lo = " << num << "; op.om = " << (int64_t)op.om << "LL; op.lut_off = " << (int64_t)op.lut_off
          << "LL;\n    ";
        switch (op.type) {
            case OP_LOAD: o << "op_load<T>(sh, op, sm, lm);"; break;
            case OP_STORE: o << "op_store<T>(sh, op, sm, lm);"; break;
            case OP_STAGE:
                if (!stage_radix_supported(op.radix)) return "";
                o << "op_stage<T, " << op.radix << ">(op, sm);";
                break;
            case OP_MUL: o << "op_mul<T>(op, sm, lm);"; break;
            case OP_R2C_POST: o << "op_r2c_post<T>(sh, op, sm);"; break;
            case OP_C2R_PRE: o << "op_c2r_pre<T>(sh, op, sm);"; break;
            case OP_RADER_GATHER: o << "op_rader_gather<T>(op, sm);"; break;
            case OP_RADER_SCATTER: o << "op_rader_scatter<T>(op, sm);"; break;
            case OP_HERM_EXPAND: o << "op_herm_expand<T>(sh, op, sm);"; break;
            case OP_PERMUTE_GATHER: o << "op_permute_gather<T>(op, sm);"; break;
            case OP_PERMUTE_SCATTER: o << "op_permute_scatter<T>(op, sm);"; break;
            case OP_SAVE_DC: o << "op_save_dc<T>(op, sm);"; break;
            default: return "";
        }
        o << "\n  }\n  __syncthreads();\n";
    }
    o << "}\n";
    return o.str();
}

namespace {

struct JitEntry {
    bool done = false;
    const void *fn = nullptr;  // cudaKernel_t, or null when compilation failed
    std::string log;
    unsigned long long smem_set_mask = 0;  // devices whose shared-memory limit is raised
};

std::mutex g_mu;
std::map<std::string, JitEntry> g_cache;

int jit_mode() {  // 0 off, 1 on (fall back on failure), 2 required
    static int mode = [] {
        const char *e = std::getenv("B200FFT_JIT");
        if (!e) return 1;
        if (!std::strcmp(e, "0")) return 0;
        if (!std::strcmp(e, "require")) return 2;
        return 1;
    }();
    return mode;
}

const void *compile(const std::string &src, std::string &log) {
    nvrtcProgram prog;
    if (nvrtcCreateProgram(&prog, src.c_str(), "b200fft_pass.cu", kJitHeaderCount, kJitHeaderSources,
                           kJitHeaderNames) != NVRTC_SUCCESS) {
        log = "nvrtcCreateProgram failed";
        return nullptr;
    }
    const char *opts[] = {"--gpu-architecture=sm_100a", "-std=c++17", "-DB200FFT_JIT=1"};
    const nvrtcResult r = nvrtcCompileProgram(prog, 3, opts);
    size_t n = 0;
    nvrtcGetProgramLogSize(prog, &n);
    if (n > 1) {
        log.resize(n);
        nvrtcGetProgramLog(prog, &log[0]);
    }
    if (r != NVRTC_SUCCESS) {
        nvrtcDestroyProgram(&prog);
        return nullptr;
    }
    size_t cn = 0;
    nvrtcGetCUBINSize(prog, &cn);
    std::vector<char> cubin(cn);
    nvrtcGetCUBIN(prog, cubin.data());
    nvrtcDestroyProgram(&prog);
    cudaLibrary_t lib;
    if (cudaLibraryLoadData(&lib, cubin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0) != cudaSuccess) {
        cudaGetLastError();
        log += "\ncudaLibraryLoadData failed";
        return nullptr;
    }
    cudaKernel_t k;
    if (cudaLibraryGetKernel(&k, lib, "b200fft_pass") != cudaSuccess) {
        cudaGetLastError();
        log += "\ncudaLibraryGetKernel failed";
        return nullptr;
    }
    return reinterpret_cast<const void *>(k);
}

}  // namespace

bool jit_enabled() { return jit_mode() != 0; }

// Compiles (without loading) the specialised kernel of every generic pass of a program;
// returns how many compiled, or -1 with the first NVRTC log.  Needs no GPU.
int jit_compile_check(const Program &prog, std::string &log) {
    int n = 0;
    for (const PassPlan &pp : prog.passes) {
        if (pp.kernel != KERNEL_PASS) continue;
        const std::string src = jit_pass_source(pp, prog.scalar_kind());
        if (src.empty()) continue;
        nvrtcProgram np;
        if (nvrtcCreateProgram(&np, src.c_str(), "b200fft_pass.cu", kJitHeaderCount, kJitHeaderSources,
                               kJitHeaderNames) != NVRTC_SUCCESS) {
            log = "nvrtcCreateProgram failed";
            return -1;
        }
        const char *opts[] = {"--gpu-architecture=sm_100a", "-std=c++17", "-DB200FFT_JIT=1"};
        const nvrtcResult r = nvrtcCompileProgram(np, 3, opts);
        if (r != NVRTC_SUCCESS) {
            size_t m = 0;
            nvrtcGetProgramLogSize(np, &m);
            log.resize(m);
            if (m) nvrtcGetProgramLog(np, &log[0]);
            log = src.substr(0, 4000) + "\n----\n" + log;
            nvrtcDestroyProgram(&np);
            return -1;
        }
        nvrtcDestroyProgram(&np);
        n++;
    }
    return n;
}

// Specialised kernels for every generic pass of a program (null entries stay on the
// interpreter).  Compiles the missing ones, in parallel.
std::vector<const void *> jit_kernels_for(const Program &prog, int device) {
    std::vector<const void *> out(prog.passes.size(), nullptr);
    if (!jit_enabled()) return out;
    std::vector<std::string> srcs(prog.passes.size());
    std::vector<size_t> todo;
    for (size_t i = 0; i < prog.passes.size(); i++) {
        if (prog.passes[i].kernel != KERNEL_PASS) continue;
        srcs[i] = jit_pass_source(prog.passes[i], prog.scalar_kind());
        if (srcs[i].empty()) continue;
        std::lock_guard<std::mutex> g(g_mu);
        if (!g_cache[srcs[i]].done) todo.push_back(i);
    }
    if (!todo.empty()) {
        std::vector<std::thread> workers;
        std::vector<std::string> logs(todo.size());
        std::vector<const void *> fns(todo.size(), nullptr);
        for (size_t t = 0; t < todo.size(); t++)
            workers.emplace_back([&, t] { fns[t] = compile(srcs[todo[t]], logs[t]); });
        for (auto &w : workers) w.join();
        std::lock_guard<std::mutex> g(g_mu);
        for (size_t t = 0; t < todo.size(); t++) {
            JitEntry &e = g_cache[srcs[todo[t]]];
            if (e.done) continue;
            e.done = true;
            e.fn = fns[t];
            e.log = logs[t];
        }
    }
    std::lock_guard<std::mutex> g(g_mu);
    for (size_t i = 0; i < prog.passes.size(); i++) {
        if (srcs[i].empty()) continue;
        JitEntry &e = g_cache[srcs[i]];
        if (!e.fn) {
            if (jit_mode() == 2) fail_runtime("pass kernel specialisation failed: " + e.log.substr(0, 2000));
            continue;
        }
        if (device >= 0 && device < 64 && !(e.smem_set_mask & (1ull << device))) {
            if (cudaFuncSetAttribute(e.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448) != cudaSuccess) {
                cudaGetLastError();
                if (jit_mode() == 2) fail_runtime("specialised pass kernel: cudaFuncSetAttribute failed");
                e.fn = nullptr;
                continue;
            }
            e.smem_set_mask |= 1ull << device;
        }
        out[i] = e.fn;
    }
    return out;
}

}  // namespace b200fft
