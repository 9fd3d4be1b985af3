// Stress test of the host copy pool (vkfft-rs_b200/csrc/host_staging.cpp) on the CPU:
// every item of every job runs exactly once, jobs started with start() finish before
// finish() returns, an item's exception reaches the caller and leaves the pool usable.
// Workers only call cudaSetDevice, whose failure without a GPU is ignored.
#include <atomic>
#include <cstdio>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "host_staging.hpp"

namespace b200fft {
[[noreturn]] void fail_runtime(const std::string &message) { throw std::runtime_error(message); }
}  // namespace b200fft

using b200fft::CopyPool;

static int failures = 0;
#define EXPECT(cond, ...)                                   \
    do {                                                    \
        if (!(cond)) {                                      \
            std::fprintf(stderr, "FAILED: " __VA_ARGS__);   \
            std::fprintf(stderr, " (%s)\n", #cond);         \
            failures++;                                     \
        }                                                   \
    } while (0)

int main() {
    for (int workers : {0, 1, 3, 7}) {
        for (int spin : {0, 200}) {
            CopyPool pool(0, workers, spin);
            // many back-to-back jobs of varying size: each item exactly once
            for (int job = 0; job < 3000; job++) {
                const size_t n = 1 + (size_t)(job * 7919) % 61;
                std::vector<std::atomic<int>> hits(n);
                for (auto &h : hits) h.store(0);
                pool.run(n, [&](size_t k) { hits[k].fetch_add(1); });
                for (size_t k = 0; k < n; k++)
                    EXPECT(hits[k].load() == 1, "run: workers %d spin %d job %d item %zu ran %d times", workers, spin,
                           job, k, hits[k].load());
            }
            if (workers > 0) {
                // start / finish: the caller sees every item complete, in any order
                for (int job = 0; job < 500; job++) {
                    const size_t n = 1 + (size_t)job % 32;
                    std::unique_ptr<std::atomic<int>[]> done(new std::atomic<int>[n]);
                    for (size_t k = 0; k < n; k++) done[k].store(0);
                    const std::function<void(size_t)> fn = [&](size_t k) { done[k].store(1, std::memory_order_release); };
                    pool.start(n, fn);
                    for (size_t k = 0; k < n; k++)
                        while (!done[k].load(std::memory_order_acquire)) {
                        }
                    pool.finish();
                }
            }
            // an item's exception reaches the caller; the pool keeps working
            bool thrown = false;
            try {
                pool.run(16, [&](size_t k) {
                    if (k == 5) throw std::runtime_error("item 5");
                });
            } catch (const std::runtime_error &e) {
                thrown = std::string(e.what()) == "item 5";
            }
            EXPECT(thrown, "exception: workers %d spin %d", workers, spin);
            std::atomic<int> total{0};
            pool.run(100, [&](size_t) { total.fetch_add(1); });
            EXPECT(total.load() == 100, "after exception: workers %d spin %d ran %d", workers, spin, total.load());
        }
    }
    if (failures) return 1;
    std::printf("ok\n");
    return 0;
}
