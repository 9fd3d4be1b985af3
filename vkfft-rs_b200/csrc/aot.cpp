// Structure keys, kernel sources and the registry of the ahead-of-time specialised pass
// kernels (aot.hpp).  The key and the source come from one list of (field, value)
// assignments, so a kernel is registered under exactly the fields it has as constants.
#include "aot.hpp"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <sstream>
#include <unordered_map>

namespace b200fft {

namespace {

struct Assign {
    std::string lhs, rhs;
};

std::string fastdiv(const FastDiv &f) {
    char b[96];
    std::snprintf(b, sizeof b, "FastDiv{%uu, %uu, %uu, 0u}", f.d, f.m, f.s);
    return b;
}

void side_fields(std::vector<Assign> &a, const char *name, const Side &s) {
    const std::string n = std::string("sh.") + name + ".";
    a.push_back({n + "real", std::to_string(s.real)});
    a.push_back({n + "count", std::to_string(s.count)});
    a.push_back({n + "cm", std::to_string(s.cm)});
    a.push_back({n + "em", std::to_string(s.em)});
    a.push_back({n + "herm", std::to_string(s.herm)});
    // unit element stride (contiguous lines) is a constant: the element-fast addressing
    // branch folds; other element strides are read from the parameters
    if (s.es == 1) a.push_back({n + "es", "1LL"});
}

bool stage_radix_supported(int r) { return (r >= 2 && r <= 13) || r == 16; }

const char *op_call(const Op &op) {
    switch (op.type) {
        case OP_LOAD: return "op_load<T>(sh, op, sm, lm);";
        case OP_STORE: return "op_store<T>(sh, op, sm, lm);";
        case OP_MUL: return "op_mul<T>(op, sm, lm);";
        case OP_R2C_POST: return "op_r2c_post<T>(sh, op, sm);";
        case OP_C2R_PRE: return "op_c2r_pre<T>(sh, op, sm);";
        case OP_RADER_GATHER: return "op_rader_gather<T>(op, sm);";
        case OP_RADER_SCATTER: return "op_rader_scatter<T>(op, sm);";
        case OP_HERM_EXPAND: return "op_herm_expand<T>(sh, op, sm);";
        case OP_PERMUTE_GATHER: return "op_permute_gather<T>(op, sm);";
        case OP_PERMUTE_SCATTER: return "op_permute_scatter<T>(op, sm);";
        case OP_SAVE_DC: return "op_save_dc<T>(op, sm);";
        default: return nullptr;
    }
}

// The compile-time fields of a pass: shape fields, then per op its fields and call.
// Returns false for a pass the specialisation does not cover.
bool pass_fields(const PassPlan &pp, std::vector<Assign> &shape, std::vector<std::vector<Assign>> &ops,
                 std::vector<std::string> &calls) {
    const PassParams &p = pp.p;
    if (pp.kernel != KERNEL_PASS || p.nops <= 0 || p.nops > kMaxOps) return false;
    shape.push_back({"sh.G", std::to_string(p.G)});
    shape.push_back({"sh.nops", std::to_string(p.nops)});
    shape.push_back({"sh.line_len", std::to_string(p.line_len)});
    shape.push_back({"sh.line_stride", std::to_string(p.line_stride)});
    shape.push_back({"sh.meta_off", std::to_string(p.meta_off)});
    shape.push_back({"sh.div_g", fastdiv(p.div_g)});
    side_fields(shape, "in", p.in);
    side_fields(shape, "out", p.out);
    if (!pp.peer_scatter) shape.push_back({"sh.peer.n", "0"});
    ops.assign(p.nops, {});
    calls.assign(p.nops, "");
    for (int k = 0; k < p.nops; k++) {
        const Op &op = p.ops[k];
        std::vector<Assign> &a = ops[k];
        a.push_back({"op.type", std::to_string(op.type)});
        a.push_back({"op.flags", std::to_string(op.flags)});
        a.push_back({"op.radix", std::to_string(op.radix)});
        a.push_back({"op.P", std::to_string(op.P)});
        a.push_back({"op.len", std::to_string(op.len)});
        a.push_back({"op.nsub", std::to_string(op.nsub)});
        a.push_back({"op.src_base", std::to_string(op.src_base)});
        a.push_back({"op.dst_base", std::to_string(op.dst_base)});
        a.push_back({"op.sub_stride", std::to_string(op.sub_stride)});
        a.push_back({"op.mul", std::to_string(op.mul)});
        a.push_back({"op.cm", std::to_string(op.cm)});
        a.push_back({"op.em", std::to_string(op.em)});
        a.push_back({"op.w_base", std::to_string(op.w_base)});
        a.push_back({"op.w_stride", std::to_string(op.w_stride)});
        a.push_back({"op.x0_base", std::to_string(op.x0_base)});
        a.push_back({"op.nfull", std::to_string(op.nfull)});
        a.push_back({"op.pad_shift", std::to_string(op.pad_shift)});
        a.push_back({"op.div_a", fastdiv(op.div_a)});
        a.push_back({"op.div_b", fastdiv(op.div_b)});
        a.push_back({"op.div_c", fastdiv(op.div_c)});
        if (op.type == OP_STAGE) {
            if (!stage_radix_supported(op.radix)) return false;
            calls[k] = "op_stage<T, " + std::to_string(op.radix) + ">(op, sm);";
        } else {
            const char *c = op_call(op);
            if (!c) return false;
            calls[k] = c;
        }
    }
    return true;
}

const char *scalar_type(int scalar_kind) {
    return scalar_kind == 2 ? "b200fft::dd" : scalar_kind == 1 ? "double" : "float";
}

struct Registry {
    std::mutex mu;
    std::unordered_map<std::string, const void *> kernels;
    std::unordered_map<const void *, unsigned long long> smem_set;  // devices opted in, per kernel
};

Registry &registry() {
    static Registry r;
    return r;
}

bool interpreter_forced() {
    static const bool forced = [] {
        const char *e = std::getenv("B200FFT_INTERPRET");
        return e && std::strcmp(e, "0") != 0;
    }();
    return forced;
}

}  // namespace

std::string aot_pass_key(const PassPlan &pp, int scalar_kind) {
    std::vector<Assign> shape;
    std::vector<std::vector<Assign>> ops;
    std::vector<std::string> calls;
    if (!pass_fields(pp, shape, ops, calls)) return "";
    std::ostringstream o;
    o << "k" << scalar_kind << ";nt" << pp.threads;
    for (const Assign &a : shape) o << ";" << a.rhs;
    for (size_t k = 0; k < ops.size(); k++) {
        o << "|";
        for (const Assign &a : ops[k]) o << a.rhs << ",";
    }
    return o.str();
}

std::string aot_pass_source(const PassPlan &pp, int scalar_kind, const std::string &name) {
    std::vector<Assign> shape;
    std::vector<std::vector<Assign>> ops;
    std::vector<std::string> calls;
    if (!pass_fields(pp, shape, ops, calls)) return "";
    std::ostringstream o;
    o << "extern \"C\" __global__ void __launch_bounds__(" << pp.threads << ") " << name
      << "(const __grid_constant__ PassParams p) {\n"
      << "  typedef " << scalar_type(scalar_kind) << " T;\n"
      << "  extern __shared__ __align__(16) unsigned char smem_raw[];\n"
      << "  cplx<T> *sm = reinterpret_cast<cplx<T> *>(smem_raw);\n"
      << "  PassShape sh = p;\n";
    for (const Assign &a : shape) o << "  " << a.lhs << " = " << a.rhs << ";\n";
    o << "  const LineMeta lm = pass_prologue<T>(sh, smem_raw);\n  __syncthreads();\n";
    for (size_t k = 0; k < ops.size(); k++) {
        o << "  {\n    Op op = p.ops[" << k << "];\n   ";
        for (const Assign &a : ops[k]) o << " " << a.lhs << " = " << a.rhs << ";";
        o << "\n    " << calls[k] << "\n  }\n  __syncthreads();\n";
    }
    o << "}\n";
    return o.str();
}

void aot_register(const char *key, const void *fn) {
    Registry &r = registry();
    std::lock_guard<std::mutex> g(r.mu);
    r.kernels.emplace(key, fn);
}

std::vector<const void *> aot_kernels_for(const Program &prog, int device) {
    std::vector<const void *> out(prog.passes.size(), nullptr);
    if (interpreter_forced()) return out;
    Registry &r = registry();
    std::lock_guard<std::mutex> g(r.mu);
    for (size_t i = 0; i < prog.passes.size(); i++) {
        if (prog.passes[i].kernel != KERNEL_PASS) continue;
        auto it = r.kernels.find(aot_pass_key(prog.passes[i], prog.scalar_kind()));
        if (it == r.kernels.end()) continue;
        const void *fn = it->second;
        unsigned long long &mask = r.smem_set[fn];
        if (device >= 0 && device < 64 && !(mask & (1ull << device))) {
            const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
            if (e != cudaSuccess)
                fail_runtime(std::string("specialised pass kernel: cudaFuncSetAttribute failed: ") +
                             cudaGetErrorString(e));
            mask |= 1ull << device;
        }
        out[i] = fn;
    }
    return out;
}

int aot_coverage(const Program &prog, int *generic_passes) {
    int total = 0, covered = 0;
    Registry &r = registry();
    std::lock_guard<std::mutex> g(r.mu);
    for (const PassPlan &pp : prog.passes) {
        if (pp.kernel != KERNEL_PASS) continue;
        total++;
        if (r.kernels.count(aot_pass_key(pp, prog.scalar_kind()))) covered++;
    }
    if (generic_passes) *generic_passes = total;
    return covered;
}

}  // namespace b200fft
