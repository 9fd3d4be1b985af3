// Execution out of a fixed, library-owned device region: the engine of
// b200fft_execute_static_workspace.  No device memory is allocated or freed here.
//
// The region is one file-scope __device__ array.  Its address is looked up once per
// device with cudaGetSymbolAddress (with that device current) and cached.  A call lays
// the region out as [packed tables | scratch buffers], copies the transform's tables in
// from the packed host image the transform keeps (built on its first call here), and
// launches the same passes as execute_program.  Every call uploads its own tables, so a
// call's result never depends on which transform used the region before it.  Nothing
// in the region has to start at zero: every pass writes each scratch element before a
// later pass reads it, and the tables are copied in before the first launch that reads
// them.  The kernels' error word is the context's.
#include <cstring>
#include <mutex>

#include "runtime.hpp"

namespace b200fft {

int kernel_variant_for(int scalar_kind);
cudaError_t launch_pass(int variant, const PassParams &p, int64_t grid, int threads, size_t smem, cudaStream_t stream);
cudaError_t launch_reg(int variant, const RegParams &rp, cudaStream_t stream);
cudaError_t launch_boundary_copy(const BoundaryCopy &b, cudaStream_t stream);
cudaError_t launch_conv_multiply(const ConvMultiply &m, int kind, cudaStream_t stream);
cudaError_t launch_r2r(const R2rPass &r, int kind, cudaStream_t stream);

constexpr size_t kStaticWorkspaceBytes = size_t(16) << 20;  // B200FFT_STATIC_WORKSPACE_BYTES
constexpr int kMaxStaticDevices = 64;
constexpr size_t kMaxStaticTables = 512;

static __device__ __align__(256) unsigned char g_static_workspace[kStaticWorkspaceBytes];

namespace {
std::mutex g_static_mu;
unsigned char *g_static_base[kMaxStaticDevices];  // device address of g_static_workspace per device
}  // namespace

static void check(cudaError_t e, const char *what) {
    if (e != cudaSuccess) fail_runtime(std::string(what) + " failed: " + cudaGetErrorString(e));
}

static size_t round256(size_t v) { return (v + 255) & ~size_t(255); }

void execute_program_static(Context *ctx, uint64_t /*id*/, const Program &prog, const void *in, void *out,
                            cudaStream_t stream) {
    if (ctx->device < 0 || ctx->device >= kMaxStaticDevices)
        throw FftError(B200FFT_RESOURCE_LIMIT_EXCEEDED, "static workspace supports CUDA device ordinals below " +
                                                            std::to_string(kMaxStaticDevices));
    if (prog.tables.size() > kMaxStaticTables)
        throw FftError(B200FFT_RESOURCE_LIMIT_EXCEEDED, "static workspace execution supports at most " +
                                                            std::to_string(kMaxStaticTables) + " tables per transform");
    size_t table_bytes = 0;
    for (auto &t : prog.tables) table_bytes += round256(t.bytes(prog.cbytes()));
    const size_t scratch_bytes = prog.scratch_bytes();
    if (table_bytes + scratch_bytes > kStaticWorkspaceBytes)
        throw FftError(B200FFT_RESOURCE_LIMIT_EXCEEDED,
                       "static workspace holds " + std::to_string(kStaticWorkspaceBytes) +
                           " bytes but this transform needs " + std::to_string(table_bytes + scratch_bytes) +
                           " (tables " + std::to_string(table_bytes) + ", scratch " + std::to_string(scratch_bytes) +
                           "); execute it with b200fft_execute and a workspace instead");
    for (const PassPlan &pp : prog.passes)
        if (pp.peer_scatter)
            throw FftError(B200FFT_UNSUPPORTED_KERNEL_PATH,
                           "static workspace execution does not run slab exchange passes (they store into other "
                           "ranks' buffers); execute slab transforms with b200fft_execute_slab");
    check(cudaSetDevice(ctx->device), "cudaSetDevice");
    if (!stream) stream = ctx->stream;
    std::lock_guard<std::mutex> g(g_static_mu);
    unsigned char *&base = g_static_base[ctx->device];
    if (!base) {
        void *p = nullptr;
        check(cudaGetSymbolAddress(&p, g_static_workspace), "cudaGetSymbolAddress of the static workspace");
        base = static_cast<unsigned char *>(p);
    }
    const void *tables[kMaxStaticTables];
    size_t off = 0;
    for (size_t k = 0; k < prog.tables.size(); k++) {
        tables[k] = base + off;
        off += round256(prog.tables[k].bytes(prog.cbytes()));
    }
    if (table_bytes > 0) {
        // The packed image (pass precision, as the context's table upload packs it) is
        // built once per program and lives as long as the program; the copy is
        // stream-ordered before the passes that read the tables.
        if (!prog.static_table_image) {
            auto img = std::make_shared<std::vector<unsigned char>>(table_bytes, 0);
            off = 0;
            for (const HostTable &t : prog.tables) {
                pack_table(t, prog, img->data() + off);
                off += round256(t.bytes(prog.cbytes()));
            }
            prog.static_table_image = img;
        }
        check(cudaMemcpyAsync(base, prog.static_table_image->data(), table_bytes, cudaMemcpyHostToDevice, stream),
              "static workspace table upload");
    }
    unsigned char *scr = base + table_bytes;
    const size_t esz = (size_t)prog.cbytes();
    void *bufs[2 + kScratchBuffers] = {const_cast<void *>(in), out};
    for (int k = 0; k < kScratchBuffers; k++) bufs[2 + k] = scr + prog.scratch_offset(k);
    const int variant = kernel_variant_for(prog.scalar_kind());
    for (const PassPlan &pp : prog.passes) {
        if (pp.kernel == KERNEL_R2R) {
            R2rPass rr = pp.rr;
            rr.src = bufs[pp.src_buf];
            rr.dst = bufs[pp.dst_buf];
            rr.tb = pp.reg_table2 >= 0 ? tables[pp.reg_table2] : nullptr;
            check(launch_r2r(rr, prog.scalar_kind(), stream), "kernel launch");
            continue;
        }
        if (pp.kernel == KERNEL_CMUL) {
            ConvMultiply cm = pp.cm;
            cm.src = bufs[pp.src_buf];
            cm.dst = bufs[pp.dst_buf];
            cm.ker = tables[pp.reg_table];
            check(launch_conv_multiply(cm, prog.scalar_kind(), stream), "kernel launch");
            continue;
        }
        if (pp.kernel == KERNEL_COPY) {
            BoundaryCopy bc = pp.bc;
            bc.src = bufs[pp.src_buf];
            bc.dst = bufs[pp.dst_buf];
            check(launch_boundary_copy(bc, stream), "kernel launch");
            continue;
        }
        if (pp.kernel == KERNEL_REG) {
            RegParams rp = pp.rp;
            rp.in = static_cast<const unsigned char *>(bufs[pp.src_buf]) + pp.src_off * (pp.reg_in_real ? esz / 2 : esz);
            rp.out = static_cast<unsigned char *>(bufs[pp.dst_buf]) + pp.dst_off * (pp.reg_out_real ? esz / 2 : esz);
            rp.tw = tables[pp.reg_table];
            rp.tw2 = pp.reg_table2 >= 0 ? tables[pp.reg_table2] : nullptr;
            rp.tw3 = pp.reg_table3 >= 0 ? tables[pp.reg_table3] : nullptr;
            rp.err = ctx->d_err;
            int rv = pp.reg_variant;
            if (pp.reg_variant_plain >= 0 && (reinterpret_cast<uintptr_t>(rp.in) & 15)) rv = pp.reg_variant_plain;
            check(launch_reg(rv, rp, stream), "kernel launch");
            continue;
        }
        PassParams p = pp.p;
        for (int k = 0; k < p.nops; k++) {
            const void **slots[3] = {&p.ops[k].lut, &p.ops[k].lut2, &p.ops[k].lut3};
            for (int s = 0; s < 3; s++) *slots[s] = pp.op_tables[k][s] >= 0 ? tables[pp.op_tables[k][s]] : nullptr;
        }
        const size_t in_sz = p.in.real ? esz / 2 : esz, out_sz = p.out.real ? esz / 2 : esz;
        p.src = static_cast<const unsigned char *>(bufs[pp.src_buf]) + pp.src_off * in_sz;
        p.dst = static_cast<unsigned char *>(bufs[pp.dst_buf]) + pp.dst_off * out_sz;
        p.err = ctx->d_err;
        check(launch_pass(variant, p, pp.grid, pp.threads, pp.smem, stream), "kernel launch");
    }
}

}  // namespace b200fft
