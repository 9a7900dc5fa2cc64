// Host-side bulk byte movement for large updates (hundreds of MB): copies split over a
// persistent pool of worker threads, which also spreads the first-touch page faults of a freshly
// allocated destination over cores.
#include <sys/mman.h>

#include <algorithm>
#include <cstdlib>
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "host_codec.h"

namespace crx {

namespace {

// Runs fn(0..n_tasks) on the calling thread plus the pool's workers; every worker takes part in
// every run and run() returns only after all of them left it, so no worker can still be working
// on one run when the next begins.
class Pool {
public:
    Pool() {
        // one process per GPU shares the host: split the cores between the local processes
        unsigned hw = std::max(1u, std::thread::hardware_concurrency());
        if (const char* lw = std::getenv("LOCAL_WORLD_SIZE")) {
            const long k = std::strtol(lw, nullptr, 10);
            if (k > 1) hw = std::max(2u, hw / unsigned(k));
        }
        const unsigned n = std::min(hw, 32u) - 1;
        for (unsigned k = 0; k < n; ++k) workers_.emplace_back([this] { loop(); });
    }
    ~Pool() {
        {
            std::lock_guard<std::mutex> g(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (auto& t : workers_) t.join();
    }

    void run(size_t n_tasks, const std::function<void(size_t)>& fn) {
        std::lock_guard<std::mutex> serial(run_mu_);
        {
            std::lock_guard<std::mutex> g(mu_);
            fn_ = &fn;
            n_ = n_tasks;
            next_.store(0);
            active_ = workers_.size();
            ++gen_;
        }
        cv_.notify_all();
        work(fn, n_tasks);
        std::unique_lock<std::mutex> g(mu_);
        done_cv_.wait(g, [&] { return active_ == 0; });
    }

private:
    void work(const std::function<void(size_t)>& fn, size_t n) {
        for (;;) {
            const size_t k = next_.fetch_add(1);
            if (k >= n) return;
            fn(k);
        }
    }
    void loop() {
        uint64_t seen = 0;
        for (;;) {
            const std::function<void(size_t)>* f;
            size_t n;
            {
                std::unique_lock<std::mutex> g(mu_);
                cv_.wait(g, [&] { return stop_ || gen_ != seen; });
                if (stop_) return;
                seen = gen_;
                f = fn_;
                n = n_;
            }
            work(*f, n);
            std::lock_guard<std::mutex> g(mu_);
            if (--active_ == 0) done_cv_.notify_all();
        }
    }

    std::vector<std::thread> workers_;
    std::mutex mu_, run_mu_;
    std::condition_variable cv_, done_cv_;
    const std::function<void(size_t)>* fn_ = nullptr;
    size_t n_ = 0;
    size_t active_ = 0;
    std::atomic<size_t> next_{0};
    uint64_t gen_ = 0;
    bool stop_ = false;
};

Pool& pool() {
    static Pool p;   // created on first large copy, joined at process exit
    return p;
}

}  // namespace

void parallel_copy(void* dst, const void* src, size_t n) {
    constexpr size_t kPiece = size_t(1) << 20;
    if (n < 4 * kPiece) {
        std::memcpy(dst, src, n);
        return;
    }
    // fewer, larger page faults when transparent huge pages are available on request
    const uintptr_t a = (reinterpret_cast<uintptr_t>(dst) + (size_t(2) << 20) - 1) & ~((uintptr_t(2) << 20) - 1);
    const uintptr_t b = (reinterpret_cast<uintptr_t>(dst) + n) & ~((uintptr_t(2) << 20) - 1);
    if (b > a) madvise(reinterpret_cast<void*>(a), b - a, MADV_HUGEPAGE);
    const size_t pieces = (n + kPiece - 1) / kPiece;
    pool().run(pieces, [&](size_t k) {
        const size_t lo = k * kPiece, len = std::min(kPiece, n - lo);
        std::memcpy(static_cast<uint8_t*>(dst) + lo, static_cast<const uint8_t*>(src) + lo, len);
    });
}

void parallel_for(size_t n, const std::function<void(size_t)>& fn) { pool().run(n, fn); }

void prefault(void* dst, size_t n) {
    constexpr size_t kPiece = size_t(2) << 20;
    if (n < 4 * kPiece) return;
    const uintptr_t a = (reinterpret_cast<uintptr_t>(dst) + kPiece - 1) & ~uintptr_t(kPiece - 1);
    const uintptr_t b = (reinterpret_cast<uintptr_t>(dst) + n) & ~uintptr_t(kPiece - 1);
    if (b > a) madvise(reinterpret_cast<void*>(a), b - a, MADV_HUGEPAGE);
    const size_t pieces = (n + kPiece - 1) / kPiece;
    pool().run(pieces, [&](size_t k) {
        volatile uint8_t* p = static_cast<uint8_t*>(dst) + k * kPiece;
        const size_t len = std::min(kPiece, n - k * kPiece);
        for (size_t off = 0; off < len; off += 4096) p[off] = 0;
    });
}

}  // namespace crx
