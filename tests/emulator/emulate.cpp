// CPU emulation of the B200 pass kernel -- TEST INFRASTRUCTURE ONLY.
//
// Builds the product's planner and lowering (the same sources as libb200fft.so) and
// runs every pass of a transform's launch program on host memory: for each CTA the
// prologue and then each op are executed for every thread in turn.  This is valid
// because the kernel's threads only communicate through shared memory across the
// __syncthreads() that separates ops.  Compiled with AddressSanitizer by the tests so
// any out-of-bounds global or shared-memory index in the lowering or the kernel is a
// CPU test failure.  Shared memory is filled with NaN bytes before every CTA so reads
// of unwritten slots poison the result.  Never linked into the product library.
#define B200FFT_EMULATE 1
#include "emu_shim.hpp"

EmuDim threadIdx, blockIdx, blockDim;

#include <cstring>
#include <string>
#include <vector>

#include "../../vkfft-rs_b200/csrc/kernels.cu"
#include "../../vkfft-rs_b200/csrc/boundary_device.cuh"
#include "../../vkfft-rs_b200/csrc/slab.hpp"
#include "../../vkfft-rs_b200/csrc/transform.hpp"

using namespace b200fft;

template <typename T>
static void emu_launch(const PassParams &p, int64_t grid, int threads, size_t smem) {
    std::vector<unsigned char> buf(smem + 16);
    unsigned char *sm_raw = buf.data() + ((16 - ((uintptr_t)buf.data() & 15)) & 15);
    blockDim.x = threads;
    for (int64_t b = 0; b < grid; b++) {
        std::memset(buf.data(), 0xff, buf.size());
        blockIdx.x = (unsigned)b;
        LineMeta lm{};
        for (int t = 0; t < threads; t++) {
            threadIdx.x = t;
            lm = pass_prologue<T>(p, sm_raw);
        }
        for (int k = 0; k < p.nops; k++) {
            Op op = p.ops[k];
            for (int t = 0; t < threads; t++) {
                threadIdx.x = t;
                run_op<T>(p, op, reinterpret_cast<cplx<T> *>(sm_raw), lm);
            }
        }
    }
}

static void run_program(const Program &prog, const void *in, void *out, const PeerStore *peer = nullptr) {
    const size_t esz = (size_t)prog.cbytes();
    std::vector<std::vector<unsigned char>> tables;
    for (const HostTable &t : prog.tables) {
        std::vector<unsigned char> v(t.bytes(prog.cbytes()));
        pack_table(t, prog, v.data());
        tables.push_back(std::move(v));
    }
    std::vector<std::vector<unsigned char>> scratch(kScratchBuffers);
    for (int k = 0; k < kScratchBuffers; k++) scratch[k].assign(prog.scratch_elems[k] * esz, 0xff);
    void *bufs[2 + kScratchBuffers] = {const_cast<void *>(in), out};
    for (int k = 0; k < kScratchBuffers; k++) bufs[2 + k] = scratch[k].empty() ? nullptr : scratch[k].data();
    int err = 0;
    for (const PassPlan &pp : prog.passes) {
        if (pp.kernel == KERNEL_R2R) {
            R2rPass rr = pp.rr;
            rr.src = bufs[pp.src_buf];
            rr.dst = bufs[pp.dst_buf];
            rr.tb = pp.reg_table2 >= 0 ? tables[pp.reg_table2].data() : nullptr;
            for (int64_t t = 0; t < rr.total; t++) {
                if (prog.is_dd)
                    r2r_one<dd>(rr, t);
                else if (prog.is_double)
                    r2r_one<double>(rr, t);
                else
                    r2r_one<float>(rr, t);
            }
            continue;
        }
        if (pp.kernel == KERNEL_CMUL) {
            ConvMultiply cm = pp.cm;
            cm.src = bufs[pp.src_buf];
            cm.dst = bufs[pp.dst_buf];
            cm.ker = tables[pp.reg_table].data();
            for (int64_t L = 0; L < cm.total; L++) {
                if (prog.is_dd)
                    conv_multiply_one<dd>(cm, L);
                else if (prog.is_double)
                    conv_multiply_one<double>(cm, L);
                else
                    conv_multiply_one<float>(cm, L);
            }
            continue;
        }
        if (pp.kernel == KERNEL_COPY) {
            BoundaryCopy bc = pp.bc;
            bc.src = bufs[pp.src_buf];
            bc.dst = bufs[pp.dst_buf];
            for (int64_t L = 0; L < bc.total; L++) boundary_copy_one(bc, L);
            continue;
        }
        PassParams p = pp.p;
        for (int k = 0; k < p.nops; k++) {
            const void **slots[3] = {&p.ops[k].lut, &p.ops[k].lut2, &p.ops[k].lut3};
            for (int s = 0; s < 3; s++)
                *slots[s] = pp.op_tables[k][s] >= 0 ? tables[pp.op_tables[k][s]].data() : nullptr;
        }
        const size_t in_sz = p.in.real ? esz / 2 : esz, out_sz = p.out.real ? esz / 2 : esz;
        p.src = static_cast<const unsigned char *>(bufs[pp.src_buf]) + pp.src_off * in_sz;
        p.dst = static_cast<unsigned char *>(bufs[pp.dst_buf]) + pp.dst_off * out_sz;
        p.err = &err;
        if (pp.peer_scatter) {
            if (!peer) fail_runtime("exchange pass without peers");
            p.peer = *peer;
            p.peer.sub = peer->chunk * pp.peer_es;
        }
        if (pp.threads > 1024 || pp.smem > 232448) fail_invalid_ir("pass launch exceeds sm_100 limits");
        if (prog.is_dd)
            emu_launch<dd>(p, pp.grid, pp.threads, pp.smem);
        else if (prog.is_double)
            emu_launch<double>(p, pp.grid, pp.threads, pp.smem);
        else
            emu_launch<float>(p, pp.grid, pp.threads, pp.smem);
        if (err) fail_runtime("emulated kernel reported error word " + std::to_string(err));
    }
}

extern "C" int b200fft_emu_run(const b200fft_config *cfg, int direction, const b200fft_device_profile *dev,
                               const void *in, size_t in_bytes, void *out, size_t out_bytes, char *errbuf,
                               size_t errlen, int *launches) {
    try {
        DeviceProfile d;
        d.backend = static_cast<Backend>(dev->backend);
        d.vendor = static_cast<Vendor>(dev->vendor);
        d.shared_memory_bytes = dev->shared_memory_bytes;
        d.shared_memory_pow2_bytes = dev->shared_memory_pow2_bytes;
        d.max_threads_per_block = dev->max_threads_per_block;
        for (int i = 0; i < 3; i++) d.max_workgroup_size[i] = dev->max_workgroup_size[i];
        d.coalesced_memory_bytes = dev->coalesced_memory_bytes;
        d.supports_f64 = dev->supports_f64;
        auto t = build_transform(FftConfig::from_c(*cfg), direction, d);
        const Program &prog = t->prog;
        size_t in_need = prog.input_bytes();
        size_t out_need = prog.output_bytes();
        if (in_bytes != in_need || out_bytes != out_need) fail_input_length(in_need, in_bytes);
        // private copies so AddressSanitizer sees exact-size heap buffers
        std::vector<unsigned char> din((const unsigned char *)in, (const unsigned char *)in + in_need);
        std::vector<unsigned char> dout(out_need, 0xff);
        run_program(prog, din.data(), dout.data());
        std::memcpy(out, dout.data(), out_need);
        if (launches) *launches = (int)prog.passes.size();
        return 0;
    } catch (const FftError &e) {
        std::strncpy(errbuf, e.message.c_str(), errlen - 1);
        errbuf[errlen - 1] = 0;
        return e.code;
    }
}

extern "C" int b200fft_emu_convolution_run(const b200fft_config *cfg, const b200fft_device_profile *dev,
                                           const void *spectrum, uint64_t copies, const void *in, size_t in_bytes,
                                           void *out, size_t out_bytes, char *errbuf, size_t errlen, int *launches) {
    try {
        DeviceProfile d;
        d.backend = static_cast<Backend>(dev->backend);
        d.vendor = static_cast<Vendor>(dev->vendor);
        d.shared_memory_bytes = dev->shared_memory_bytes;
        d.shared_memory_pow2_bytes = dev->shared_memory_pow2_bytes;
        d.max_threads_per_block = dev->max_threads_per_block;
        for (int i = 0; i < 3; i++) d.max_workgroup_size[i] = dev->max_workgroup_size[i];
        d.coalesced_memory_bytes = dev->coalesced_memory_bytes;
        d.supports_f64 = dev->supports_f64;
        auto c = build_convolution(FftConfig::from_c(*cfg), d, spectrum, copies);
        const Program &prog = c->prog;
        const size_t csz = (size_t)prog.cbytes();
        const size_t isz = prog.input_real ? csz / 2 : csz, osz = prog.output_real ? csz / 2 : csz;
        if (in_bytes != prog.input_elems * isz || out_bytes != prog.output_elems * osz)
            fail_input_length(prog.input_elems, in_bytes / isz);
        std::vector<unsigned char> din((const unsigned char *)in, (const unsigned char *)in + in_bytes);
        std::vector<unsigned char> dout(out_bytes, 0xff);
        run_program(prog, din.data(), dout.data());
        std::memcpy(out, dout.data(), out_bytes);
        if (launches) *launches = (int)prog.passes.size();
        return 0;
    } catch (const FftError &e) {
        std::strncpy(errbuf, e.message.c_str(), errlen - 1);
        errbuf[errlen - 1] = 0;
        return e.code;
    }
}

// All ranks of a slab transform in one process: every rank's pre program (ending in the
// exchange pass, which scatters into the ranks' exchange buffers), then every post program.
extern "C" int b200fft_emu_slab_run(const b200fft_config *cfg, int direction, const b200fft_device_profile *dev,
                                    int nranks, const void *in, size_t in_bytes_per_rank, void *out,
                                    size_t out_bytes_per_rank, char *errbuf, size_t errlen, int *launches) {
    try {
        DeviceProfile d;
        d.backend = static_cast<Backend>(dev->backend);
        d.vendor = static_cast<Vendor>(dev->vendor);
        d.shared_memory_bytes = dev->shared_memory_bytes;
        d.shared_memory_pow2_bytes = dev->shared_memory_pow2_bytes;
        d.max_threads_per_block = dev->max_threads_per_block;
        for (int i = 0; i < 3; i++) d.max_workgroup_size[i] = dev->max_workgroup_size[i];
        d.coalesced_memory_bytes = dev->coalesced_memory_bytes;
        d.supports_f64 = dev->supports_f64;
        std::vector<std::unique_ptr<Slab>> slabs;
        for (int r = 0; r < nranks; r++) slabs.push_back(build_slab(FftConfig::from_c(*cfg), direction, nranks, r, d));
        const Slab &s0 = *slabs[0];
        const size_t esz = (size_t)s0.pre.cbytes();
        const size_t in_need = s0.input_elems * (s0.input_real ? esz / 2 : esz);
        const size_t out_need = s0.output_elems * (s0.output_real ? esz / 2 : esz);
        if (in_bytes_per_rank != in_need || out_bytes_per_rank != out_need) fail_input_length(in_need, in_bytes_per_rank);
        std::vector<std::vector<unsigned char>> ex(nranks), din(nranks), dout(nranks);
        for (int r = 0; r < nranks; r++) {
            ex[r].assign(s0.exchange_elems * esz, 0xff);
            din[r].assign((const unsigned char *)in + r * in_need, (const unsigned char *)in + (r + 1) * in_need);
            dout[r].assign(out_need, 0xff);
        }
        for (int r = 0; r < nranks; r++) {
            PeerStore ps = slabs[r]->peer;
            for (int q = 0; q < nranks; q++) ps.ptr[q] = ex[q].data();
            run_program(slabs[r]->pre, din[r].data(), dout[r].data(), &ps);
        }
        for (int r = 0; r < nranks; r++) run_program(slabs[r]->post, ex[r].data(), dout[r].data());
        for (int r = 0; r < nranks; r++) std::memcpy((unsigned char *)out + r * out_need, dout[r].data(), out_need);
        if (launches) *launches = (int)(s0.pre.passes.size() + s0.post.passes.size());
        return 0;
    } catch (const FftError &e) {
        std::strncpy(errbuf, e.message.c_str(), errlen - 1);
        errbuf[errlen - 1] = 0;
        return e.code;
    }
}

namespace b200fft {
void release_slab_device(Slab *) {}
}  // namespace b200fft

// The register-resident kernels are not emulated (their threads exchange data inside
// one op); the lowering never selects them in this build.
namespace b200fft {
int reg_variant_for(bool, size_t, int, bool) { return -1; }
}  // namespace b200fft
namespace b200fft {
int reg_variant_radices(int, int *) { return 0; }
int reg_variant_peer_twin(int) { return -1; }
int reg_variant_persistent_twin(int) { return -1; }
int reg_variant_length(int) { return 0; }
}  // namespace b200fft
