// Build-time generator of the ahead-of-time specialised pass kernels (aot.hpp).
//
//     gen_aot <output directory>
//
// Lowers a catalogue of transforms for the B200 device profile, collects the structure
// key of every generic pass, and writes one CUDA source per CTA thread count (the op
// functions take the thread count as the B200FFT_NT macro) holding one kernel per
// distinct key plus the static initialiser that registers them.  The catalogue is the
// BASELINE configurations 3-5 in both precisions and directions, the reference's own
// published and test shapes, and common lengths of every algorithm family (Rader direct
// and FFT, nested Rader, fused and three-pass Bluestein, four-step, real even-half, DCT
// reductions, double-double); batches are large enough that no pass's lines per CTA is
// clipped by the batch, so the keys are those of any larger batch of the same shape.
// Runs on the build host; needs no GPU.
#include <cstdio>
#include <algorithm>
#include <cstdlib>
#include <fstream>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "aot.hpp"
#include "slab.hpp"
#include "transform.hpp"

using namespace b200fft;

namespace {

DeviceProfile b200_profile() {
    // the attributes a B200 reports, mapped as the runtime maps them (runtime.cpp)
    return cuda_device_profile(49152, 1024, 1024, 1024, 64, true);
}

struct Entry {
    std::vector<size_t> dims;
    size_t batch;
    Precision prec;
    TransformKind kind;
    bool rec = false;   // recursive FFT-Rader tuning
    bool conv = false;  // ND real convolution, batch = coordinate features
    size_t shared = 0;  // planner device with this much shared memory, portable tuning
};

PlannerTuning rec_tuning() {
    PlannerTuning t;
    t.min_rader_direct_prime = 17;
    t.max_rader_direct_prime = 89;
    t.min_rader_fft_prime = 17;
    t.max_rader_fft_prime = 16384;
    t.allow_recursive_fft_rader = true;
    return t;
}

std::vector<Entry> catalogue() {
    const Precision F32 = Precision::F32, F64 = Precision::F64, DD = Precision::DoubleDouble;
    const TransformKind C2C = TransformKind::C2C, R2C = TransformKind::R2C, DCT2 = TransformKind::Dct2;
    std::vector<Entry> e;
    for (Precision p : {F32, F64}) {
        // BASELINE config 3 (power-of-two: register kernels), config 4, config 5
        e.push_back({{512, 512, 512}, 1, p, C2C});
        e.push_back({{1024, 1024, 1024}, 1, p, R2C});
        e.push_back({{1024, 17, 65537}, 1, p, C2C});
        e.push_back({{4099}, 16384, p, C2C});
        e.push_back({{4099}, 16384, p, C2C, true});
        e.push_back({{65537}, 2048, p, C2C});
        e.push_back({{2048, 2048}, 64, p, R2C, false, true});
        // sub-shapes the parity tests check the ND configs through
        e.push_back({{17, 65537}, 1024, p, C2C});
        e.push_back({{2, 17, 65537}, 1, p, C2C});
        e.push_back({{2, 17, 4099}, 1, p, C2C});
        // the reference's published pair-timing lengths (docs/PORTING_PLAN.md:281)
        for (size_t n : {103, 257, 5760, 4089}) e.push_back({{n}, 64, p, C2C});
        e.push_back({{4089}, 64, p, C2C, true});
        // its p29-FFT witnesses: portable tuning on 32 / 16 KiB of planner shared memory
        // (examples/native_benchmark.rs:733-757)
        e.push_back({{4089}, 64, p, C2C, false, false, 32 * 1024});
        e.push_back({{4089}, 64, p, C2C, false, false, 16 * 1024});
        // family representatives: Rader direct / FFT, Bluestein fused / three-pass,
        // mixed radix, four-step, composite Rader
        for (size_t n : {17, 47, 89, 97, 360, 1000, 1536, 2187, 2401, 3125, 2288, 6000, 10000, 4106, 8191,
                         16411, 131072, 524288, 83 * 1009, 6 * 683})
            e.push_back({{n}, 256, p, C2C});
        for (size_t n : {4099, 107, 683}) e.push_back({{n}, 256, p, C2C, true});
        // real transforms on non-power-of-two rows and ND real shapes
        for (size_t n : {30, 94, 206, 1000, 4106, 8704, 6000}) e.push_back({{n}, 256, p, R2C});
        e.push_back({{17, 34}, 64, p, R2C});
        e.push_back({{16, 32, 30}, 16, p, R2C});
        e.push_back({{1000, 1000}, 4, p, R2C});
        // 2D / 3D complex with odd axes
        e.push_back({{32, 17, 100}, 8, p, C2C});
        e.push_back({{5, 47, 12}, 8, p, C2C});
        e.push_back({{1000, 1000}, 4, p, C2C});
        // DCT / DST reductions of non-power-of-two lengths
        e.push_back({{1000}, 256, p, DCT2});
    }
    for (size_t n : {4096, 1000, 360, 4099}) e.push_back({{n}, 512, DD, C2C});
    return e;
}

void add_program(const Program &prog, std::map<int, std::map<std::string, const PassPlan *>> &by_nt,
                 std::vector<std::unique_ptr<Program>> &keep, int &passes) {
    keep.push_back(std::make_unique<Program>(prog));
    const Program &p = *keep.back();
    for (const PassPlan &pp : p.passes) {
        if (pp.kernel != KERNEL_PASS) continue;
        passes++;
        const std::string key = aot_pass_key(pp, p.scalar_kind());
        if (key.empty()) continue;
        by_nt[pp.threads].emplace(key, &pp);
    }
}

std::string c_string(const std::string &s) {
    std::string o = "\"";
    for (char c : s) {
        if (c == '"' || c == '\\') o += '\\';
        o += c;
    }
    return o + "\"";
}

}  // namespace

int main(int argc, char **argv) {
    if (argc != 2) {
        std::fprintf(stderr, "usage: gen_aot <output directory>\n");
        return 2;
    }
    const std::string outdir = argv[1];
    const DeviceProfile dev = b200_profile();
    std::map<int, std::map<std::string, const PassPlan *>> by_nt;  // threads -> key -> pass
    std::vector<std::unique_ptr<Program>> keep;
    int passes = 0;
    for (const Entry &en : catalogue()) {
        FftConfig cfg = FftConfig::make(en.dims);
        cfg.batch_count = en.batch;
        cfg.precision = en.prec;
        cfg.transform = en.kind;
        if (en.rec) cfg.with_tuning(rec_tuning());
        DeviceProfile d = dev;
        if (en.shared) {
            d.shared_memory_bytes = d.shared_memory_pow2_bytes = en.shared;
            cfg.with_tuning(PlannerTuning::portable());
        }
        try {
            if (en.conv) {
                cfg.batch_count = 1;
                cfg.perform_convolution = true;
                cfg.coordinate_features = en.batch;
                size_t half = 1;
                for (size_t k = 0; k + 1 < en.dims.size(); k++) half *= en.dims[k];
                half *= en.dims.back() / 2 + 1;
                std::vector<unsigned char> spec(half * compute_complex_bytes(en.prec), 0);
                auto conv = build_convolution(cfg, dev, spec.data(), 1);
                add_program(conv->prog, by_nt, keep, passes);
                continue;
            }
            std::vector<std::pair<int, bool>> dirs = {{0, false}, {1, true}, {1, false}};
            for (auto [dir, norm] : dirs) {
                FftConfig c = cfg;
                c.normalize_inverse = norm;
                if (dir == 1 && en.kind == TransformKind::R2C) c.transform = TransformKind::C2R;
                auto t = build_transform(c, dir, d);
                add_program(t->prog, by_nt, keep, passes);
            }
            if (en.dims.size() == 3 && en.kind == TransformKind::C2C && en.dims[0] % 8 == 0 && en.batch == 1) {
                for (int ranks : {2, 4, 8})
                    for (int dir : {0, 1}) {
                        FftConfig c = cfg;
                        c.normalize_inverse = dir == 1;
                        auto s = build_slab(c, dir, ranks, 0, dev);
                        add_program(s->pre, by_nt, keep, passes);
                        add_program(s->post, by_nt, keep, passes);
                    }
            }
        } catch (const std::exception &ex) {
            std::fprintf(stderr, "gen_aot: catalogue entry skipped: %s\n", ex.what());
        }
    }
    // one unit per thread count and shard of kShard kernels (parallel compilation)
    constexpr size_t kShard = 12;
    size_t kernels = 0, units = 0;
    for (auto &[nt, keys] : by_nt) {
        std::vector<std::pair<std::string, const PassPlan *>> list(keys.begin(), keys.end());
        for (size_t s0 = 0; s0 < list.size(); s0 += kShard, units++) {
            const std::string tag = std::to_string(nt) + "_" + std::to_string(s0 / kShard);
            std::ofstream f(outdir + "/aot_nt" + tag + ".cu");
            f << "// Generated by gen_aot: specialised pass kernels with " << nt << " threads per CTA.\n"
              << "#define B200FFT_NT " << nt << "\n#include \"pass_device.cuh\"\n#include \"aot.hpp\"\n"
              << "using namespace b200fft;\n\n";
            std::vector<std::pair<std::string, std::string>> regs;
            for (size_t k = s0; k < std::min(list.size(), s0 + kShard); k++) {
                const std::string &key = list[k].first;
                const std::string name = "b200fft_aot_nt" + tag + "_" + std::to_string(k - s0);
                f << aot_pass_source(*list[k].second, key[1] - '0', name) << "\n";
                regs.push_back({key, name});
            }
            f << "namespace {\nconst bool registered = [] {\n";
            for (auto &[key, name] : regs)
                f << "    aot_register(" << c_string(key) << ", reinterpret_cast<const void *>(" << name << "));\n";
            f << "    return true;\n}();\n}  // namespace\n";
            kernels += regs.size();
        }
    }
    std::printf("gen_aot: %d generic passes in the catalogue, %zu distinct specialised kernels in %zu units\n",
                passes, kernels, units);
    return 0;
}
