// Host arrays in ordinary (pageable) memory through pinned staging.
//
// The copy engines read and write only page-locked host memory; a cudaMemcpyAsync from a
// pageable array is staged by the driver through its own small pinned buffers, one piece
// at a time, on the calling thread (≈15–18 GB/s measured on the B200 hosts, against
// ≈44 GB/s from pinned memory and ≈17 GB/s for one thread's memcpy).  The host API of
// this library takes the caller's arrays as they are (execute_transform_f32 / _f64 take
// Rust slices, native_runtime.rs:339-359), so for large arrays it stages them itself: the
// array is cut into chunks, the threads of a small copy pool copy chunks into a pinned
// ring, and each chunk's DMA is queued as soon as its copy lands, so the CPU copies of
// later chunks overlap the transfers of earlier ones (and the reverse on the way back).
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <condition_variable>
#include <cstddef>
#include <cstdint>
#include <exception>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace b200fft {

// True when `p` is host memory that CUDA has not page-locked (malloc'd, numpy, a Vec).
bool host_is_pageable(const void *p);

// A fixed set of host threads that run the items of one job, with or without the caller.
class CopyPool {
public:
    // spin_us: how long an idle worker polls for the next job before it sleeps
    CopyPool(int device, int workers, int spin_us);
    ~CopyPool();
    CopyPool(const CopyPool &) = delete;
    CopyPool &operator=(const CopyPool &) = delete;
    int threads() const { return (int)workers_.size() + 1; }
    // Runs fn(k) for every k in [0, n) (n < 2^20) on the workers and the calling thread;
    // returns when all items have finished and rethrows the first exception an item raised.
    void run(size_t n, const std::function<void(size_t)> &fn);
    // The same on the workers alone (there must be some): start() returns at once, so the
    // caller can act on items as they finish; finish() waits for the job and rethrows.
    void start(size_t n, const std::function<void(size_t)> &fn);
    void finish();

private:
    // the claim word: job generation (high 24 bits) | item count (20 bits) | next item
    // (low 20 bits), so a claim is checked against the count of its own job
    static constexpr int kGenShift = 40, kCountShift = 20;
    static constexpr uint64_t kField = (1ull << 20) - 1;
    void worker_main();
    void claim_items(uint64_t gen);

    int device_;
    int spin_us_;
    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable cv_;
    bool stop_ = false;
    // next item of the current job with its count and generation: a worker that wakes
    // late cannot claim an item of a later job by mistake
    std::atomic<uint64_t> next_{0};
    std::atomic<size_t> done_{0};
    uint64_t gen_ = 0;
    size_t job_n_ = 0;
    const std::function<void(size_t)> *fn_ = nullptr;
    std::mutex err_mu_;
    std::exception_ptr err_;
};

// How a HostStaging cuts its copies.  The defaults are the measured best on the B200
// hosts (16 Xeon threads; ≈17 GB/s memcpy per thread; ≈44 GB/s pinned DMA; the driver's
// pageable copy ≈18 GB/s up, ≈14 GB/s down): a staged download beats the driver's from
// 1 MiB (2 MiB 155 → 105 µs, 32 MiB 2.05 → 0.9–1.0 ms), a staged upload only for large
// arrays (128 MiB 12.4 → 4.8 ms; from 2 to 32 MiB it measured no better), since below
// that the driver already overlaps one thread's memcpy with the DMA at memcpy speed.
struct StagingTuning {
    int workers = 3;                    // pool threads besides the caller
    int spin_us = 0;                    // idle polling of a worker before it sleeps
    int up_chunks_per_thread = 1;       // chunks of one upload window per copying thread
    int down_chunks_per_thread = 4;     // the same for downloads
    size_t min_chunk = 256 << 10;       // bytes
    size_t max_chunk = 4 << 20;
    size_t min_staged_upload = 32 << 20;   // smaller pageable copies use the driver's path
    size_t min_staged_download = 1 << 20;
};

// Pinned rings and events of one context's staged host copies (one host call at a time:
// the context's host lock serialises them).
class HostStaging {
public:
    explicit HostStaging(int device, const StagingTuning &tuning = StagingTuning());
    ~HostStaging();
    HostStaging(const HostStaging &) = delete;
    HostStaging &operator=(const HostStaging &) = delete;
    // Copies `bytes` of pageable host memory to device memory `dst` in stream order.
    // Returns once every byte is in the pinned ring and its DMA is queued on `stream`
    // (the source array may then change; later work on `stream` sees the data).
    void upload(void *dst, const void *src, size_t bytes, cudaStream_t stream);
    // Copies `bytes` of device memory `src` into pageable host memory after the work
    // queued on `stream` so far; returns when every byte has been written to `dst`.
    void download(void *dst, const void *src, size_t bytes, cudaStream_t stream);
    // A page-locked word for small device-to-host reads (the kernels' error word).
    int *pinned_word() { return word_; }

private:
    static constexpr int kMaxWindow = 32;  // chunks per window; the ring holds two windows
    struct Ring {
        unsigned char *buf = nullptr;
        size_t bytes = 0;
        size_t chunk = 0;                     // chunk size of the slots' last use
        cudaEvent_t ev[2 * kMaxWindow] = {};  // download: per chunk; upload: per half
        bool used[2 * kMaxWindow] = {};
    };
    void plan(size_t bytes, bool caller_copies, int chunks_per_thread, size_t &chunk, size_t &window) const;
    void ensure(Ring &r, size_t chunk, size_t window);

    int device_;
    StagingTuning tuning_;
    CopyPool pool_;
    Ring up_, down_;
    std::atomic<int> ready_[kMaxWindow];  // upload: chunk i of the window is in the ring
    int *word_ = nullptr;
};

}  // namespace b200fft
