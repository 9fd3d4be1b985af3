// Staged host copies: a copy pool and pinned rings (host_staging.hpp).
#include "host_staging.hpp"

#include <algorithm>
#include <chrono>
#include <cstring>
#include <string>

#include "core.hpp"

namespace b200fft {

static void check_cuda(cudaError_t e, const char *what) {
    if (e != cudaSuccess) fail_runtime(std::string(what) + " failed: " + cudaGetErrorString(e));
}

bool host_is_pageable(const void *p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();  // older drivers report unregistered memory as an error
        return true;
    }
    return a.type == cudaMemoryTypeUnregistered;
}

static inline void cpu_relax() {
#if defined(__x86_64__) || defined(__i386__)
    __builtin_ia32_pause();
#endif
}

// ---- copy pool ---------------------------------------------------------------------

CopyPool::CopyPool(int device, int workers, int spin_us) : device_(device), spin_us_(spin_us) {
    for (int i = 0; i < workers; i++) workers_.emplace_back([this] { worker_main(); });
}

CopyPool::~CopyPool() {
    {
        std::lock_guard<std::mutex> l(mu_);
        stop_ = true;
    }
    cv_.notify_all();
    for (auto &t : workers_) t.join();
}

void CopyPool::claim_items(uint64_t gen) {
    for (;;) {
        uint64_t v = next_.load(std::memory_order_acquire);
        if ((v >> kGenShift) != gen) return;
        const size_t k = (size_t)(v & kField);
        if (k >= (size_t)((v >> kCountShift) & kField)) return;  // the job's own count
        if (!next_.compare_exchange_weak(v, v + 1, std::memory_order_acq_rel)) continue;
        // item k of job `gen` is ours: the job (and fn_) stays in place until it is done
        try {
            (*fn_)(k);
        } catch (...) {
            std::lock_guard<std::mutex> l(err_mu_);
            if (!err_) err_ = std::current_exception();
        }
        done_.fetch_add(1, std::memory_order_acq_rel);
    }
}

void CopyPool::worker_main() {
    cudaSetDevice(device_);
    uint64_t seen = 0;
    for (;;) {
        uint64_t gen = next_.load(std::memory_order_acquire) >> kGenShift;
        if (gen == seen) {
            // poll for a short while, then sleep until the next job or shutdown
            const auto t0 = std::chrono::steady_clock::now();
            while ((gen = next_.load(std::memory_order_acquire) >> kGenShift) == seen &&
                   std::chrono::steady_clock::now() - t0 < std::chrono::microseconds(spin_us_))
                cpu_relax();
            if (gen == seen) {
                std::unique_lock<std::mutex> l(mu_);
                cv_.wait(l, [&] { return stop_ || (next_.load(std::memory_order_acquire) >> kGenShift) != seen; });
                if (stop_) return;
                gen = next_.load(std::memory_order_acquire) >> kGenShift;
            }
        }
        {
            std::lock_guard<std::mutex> l(mu_);
            if (stop_) return;
        }
        seen = gen;
        claim_items(gen);
    }
}

void CopyPool::start(size_t n, const std::function<void(size_t)> &fn) {
    if (n > kField) fail_runtime("host copy pool: a job of more than 2^20 - 1 items");
    fn_ = &fn;
    err_ = nullptr;
    job_n_ = n;
    done_.store(0, std::memory_order_relaxed);
    const uint64_t gen = ++gen_ & ((1ull << (64 - kGenShift)) - 1);
    next_.store((gen << kGenShift) | ((uint64_t)n << kCountShift), std::memory_order_release);
    if (!workers_.empty()) {
        { std::lock_guard<std::mutex> l(mu_); }  // a worker between its check and its wait sees the job
        cv_.notify_all();
    }
}

void CopyPool::finish() {
    while (done_.load(std::memory_order_acquire) < job_n_) cpu_relax();
    if (err_) std::rethrow_exception(err_);
}

void CopyPool::run(size_t n, const std::function<void(size_t)> &fn) {
    if (n == 0) return;
    start(n, fn);
    claim_items(gen_ & ((1ull << (64 - kGenShift)) - 1));
    finish();
}

// ---- pinned rings --------------------------------------------------------------------

HostStaging::HostStaging(int device, const StagingTuning &tuning)
    : device_(device), tuning_(tuning), pool_(device, std::max(0, tuning.workers), tuning.spin_us) {
    for (auto &r : ready_) r.store(0, std::memory_order_relaxed);
    check_cuda(cudaHostAlloc(reinterpret_cast<void **>(&word_), sizeof(int), cudaHostAllocDefault),
               "pinned error word allocation");
}

HostStaging::~HostStaging() {
    cudaSetDevice(device_);
    for (Ring *r : {&up_, &down_}) {
        for (cudaEvent_t e : r->ev) {
            if (!e) continue;
            cudaEventSynchronize(e);
            cudaEventDestroy(e);
        }
        if (r->buf) cudaFreeHost(r->buf);
    }
    if (word_) cudaFreeHost(word_);
}

// A window is a few chunks per copying thread: every thread has a chunk to copy while the
// first DMAs run, and each chunk is large enough that its copy call costs little against
// its transfer.
void HostStaging::plan(size_t bytes, bool caller_copies, int chunks_per_thread, size_t &chunk, size_t &window) const {
    const size_t kAlign = 64 << 10;
    const size_t copiers = (size_t)std::max(1, caller_copies ? pool_.threads() : pool_.threads() - 1);
    window = std::min<size_t>(kMaxWindow, copiers * (size_t)std::max(1, chunks_per_thread));
    size_t c = (bytes + window - 1) / window;
    c = std::min(std::max(c, tuning_.min_chunk), std::max(tuning_.max_chunk, tuning_.min_chunk));
    chunk = (c + kAlign - 1) / kAlign * kAlign;
}

void HostStaging::ensure(Ring &r, size_t chunk, size_t window) {
    const size_t need = 2 * window * chunk;
    if (chunk != r.chunk || r.bytes < need) {
        // the slots move with the chunk size: every earlier DMA must have ended
        for (int s = 0; s < 2 * kMaxWindow; s++)
            if (r.used[s]) check_cuda(cudaEventSynchronize(r.ev[s]), "staging event synchronize");
        std::fill(std::begin(r.used), std::end(r.used), false);
        r.chunk = chunk;
    }
    if (r.bytes < need) {
        if (r.buf) check_cuda(cudaFreeHost(r.buf), "pinned staging free");
        r.buf = nullptr;
        r.bytes = 0;
        check_cuda(cudaHostAlloc(reinterpret_cast<void **>(&r.buf), need, cudaHostAllocDefault),
                   "pinned staging allocation");
        r.bytes = need;
    }
    for (cudaEvent_t &e : r.ev)
        if (!e) check_cuda(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "staging event creation");
}

void HostStaging::upload(void *dst, const void *src, size_t bytes, cudaStream_t stream) {
    if (bytes == 0) return;
    const bool solo = pool_.threads() == 1;
    size_t C, W;
    plan(bytes, solo, tuning_.up_chunks_per_thread, C, W);
    ensure(up_, C, W);
    const size_t nchunks = (bytes + C - 1) / C;
    const auto *s = static_cast<const unsigned char *>(src);
    auto *d = static_cast<unsigned char *>(dst);
    // windows of W chunks in alternate halves of the ring: the CPU copies of a window
    // overlap the DMAs of the one before; a half is rewritten only after the DMAs of its
    // last window ended (one event per half).  The workers copy; this thread queues each
    // chunk's DMA in order as soon as the chunk is in the ring (copy calls into one stream
    // from several threads measured slower).
    for (size_t w0 = 0, win = 0; w0 < nchunks; w0 += W, win++) {
        const size_t count = std::min(W, nchunks - w0);
        const int h = (int)(win & 1);
        if (up_.used[h]) check_cuda(cudaEventSynchronize(up_.ev[h]), "staging event synchronize");
        unsigned char *half = up_.buf + (size_t)h * W * C;
        auto copy = [&](size_t i) {
            const size_t off = (w0 + i) * C;
            std::memcpy(half + i * C, s + off, std::min(C, bytes - off));
        };
        auto queue = [&](size_t i) {
            const size_t off = (w0 + i) * C;
            check_cuda(cudaMemcpyAsync(d + off, half + i * C, std::min(C, bytes - off), cudaMemcpyHostToDevice, stream),
                       "input upload");
        };
        if (solo) {
            for (size_t i = 0; i < count; i++) {
                copy(i);
                queue(i);
            }
        } else {
            for (size_t i = 0; i < count; i++) ready_[i].store(0, std::memory_order_relaxed);
            const std::function<void(size_t)> job = [&](size_t i) {
                copy(i);
                ready_[i].store(1, std::memory_order_release);
            };
            pool_.start(count, job);
            try {
                for (size_t i = 0; i < count; i++) {
                    while (!ready_[i].load(std::memory_order_acquire)) cpu_relax();
                    queue(i);
                }
            } catch (...) {
                pool_.finish();  // the workers still use the ring
                throw;
            }
            pool_.finish();
        }
        check_cuda(cudaEventRecord(up_.ev[h], stream), "staging event record");
        up_.used[h] = true;
    }
}

void HostStaging::download(void *dst, const void *src, size_t bytes, cudaStream_t stream) {
    if (bytes == 0) return;
    size_t C, W;
    plan(bytes, true, tuning_.down_chunks_per_thread, C, W);
    ensure(down_, C, W);
    const size_t nchunks = (bytes + C - 1) / C;
    const auto *s = static_cast<const unsigned char *>(src);
    auto *d = static_cast<unsigned char *>(dst);
    auto issue = [&](size_t w0, size_t win) {  // DMAs of one window into its half, an event each
        const size_t count = std::min(W, nchunks - w0);
        const size_t base = (win & 1) * W;
        for (size_t i = 0; i < count; i++) {
            const size_t off = (w0 + i) * C, len = std::min(C, bytes - off);
            check_cuda(cudaMemcpyAsync(down_.buf + (base + i) * C, s + off, len, cudaMemcpyDeviceToHost, stream),
                       "output download");
            check_cuda(cudaEventRecord(down_.ev[base + i], stream), "staging event record");
            down_.used[base + i] = true;
        }
    };
    issue(0, 0);
    for (size_t w0 = 0, win = 0; w0 < nchunks; w0 += W, win++) {
        // the next window's DMAs go to the other half, whose chunks were copied out already
        if (w0 + W < nchunks) issue(w0 + W, win + 1);
        const size_t count = std::min(W, nchunks - w0);
        const size_t base = (win & 1) * W;
        pool_.run(count, [&](size_t i) {
            const size_t off = (w0 + i) * C, len = std::min(C, bytes - off);
            check_cuda(cudaEventSynchronize(down_.ev[base + i]), "staging event synchronize");
            std::memcpy(d + off, down_.buf + (base + i) * C, len);
        });
    }
}

}  // namespace b200fft
