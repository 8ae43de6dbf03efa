// A persistent pool of host threads for the per-structure host work of a
// call (periodic geometry, cell plans).  Threads are started once per process
// and sleep between calls; parallel_for hands out fixed-size chunks through
// an atomic counter and the calling thread takes chunks too.  The caller
// returns as soon as every chunk is done: a worker that wakes late finds no
// chunk left and goes back to sleep, so a call never waits for a thread to be
// scheduled.  Workers poll briefly before sleeping, because the parallel
// loops of one neighbor-list call follow each other within a millisecond.
// Calls from several host threads are serialised.
#pragma once

#include <algorithm>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <cstdlib>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace tnr {

class HostPool {
public:
    // Never destroyed: the sleeping threads end with the process.
    static HostPool& instance() {
        static HostPool* pool = new HostPool;
        return *pool;
    }

    // Runs body(begin, end) over [0, n) in chunks of `grain`.  body must not
    // throw; report failures through its own state.
    void parallel_for(int64_t n, int64_t grain, const std::function<void(int64_t, int64_t)>& body) {
        if (n <= 0) return;
        grain = std::max<int64_t>(grain, 1);
        const int64_t chunks = (n + grain - 1) / grain;
        if (chunks == 1 || workers_.empty()) {
            body(0, n);
            return;
        }
        std::lock_guard<std::mutex> call(call_mutex_);
        {
            std::lock_guard<std::mutex> lock(mutex_);
            body_ = &body;
            n_ = n;
            grain_ = grain;
            next_.store(0, std::memory_order_relaxed);
            remaining_.store(chunks, std::memory_order_relaxed);
            generation_.fetch_add(1, std::memory_order_release);
        }
        wake_.notify_all();
        run_chunks(body, n, grain);
        std::unique_lock<std::mutex> lock(mutex_);
        done_.wait(lock, [&] {
            return remaining_.load(std::memory_order_acquire) == 0 && in_flight_ == 0;
        });
        body_ = nullptr;
    }

    // Wakes the workers without work, so that they poll (instead of
    // sleeping) when a parallel loop follows shortly: a caller about to
    // block on the device calls this first, and the loop after the wait
    // does not pay the threads' wake-up latency.
    void prewake() {
        if (workers_.empty()) return;
        std::lock_guard<std::mutex> call(call_mutex_);
        {
            std::lock_guard<std::mutex> lock(mutex_);
            body_ = nullptr;
            generation_.fetch_add(1, std::memory_order_release);
        }
        wake_.notify_all();
    }

    HostPool(const HostPool&) = delete;
    HostPool& operator=(const HostPool&) = delete;

private:
    // One process per GPU shares the host: under a launcher that sets
    // LOCAL_WORLD_SIZE (torchrun does) each process takes its share of the
    // cores, so the ranks' pools do not oversubscribe the host.
    HostPool() {
        unsigned hardware = std::max(1u, std::thread::hardware_concurrency());
        if (const char* local = std::getenv("LOCAL_WORLD_SIZE")) {
            const long ranks = std::strtol(local, nullptr, 10);
            if (ranks > 1) hardware = std::max(1u, hardware / static_cast<unsigned>(ranks));
        }
        const unsigned count = std::min(hardware, 64u) - 1;
        for (unsigned k = 0; k < count; ++k) {
            workers_.emplace_back([this] { loop(); });
            workers_.back().detach();
        }
    }
    ~HostPool() = default;

    void run_chunks(const std::function<void(int64_t, int64_t)>& body, int64_t n, int64_t grain) {
        for (;;) {
            const int64_t begin = next_.fetch_add(grain, std::memory_order_relaxed);
            if (begin >= n) return;
            body(begin, std::min(n, begin + grain));
            if (remaining_.fetch_sub(1, std::memory_order_acq_rel) == 1) {
                std::lock_guard<std::mutex> lock(mutex_);
                done_.notify_all();
            }
        }
    }

    void loop() {
        uint64_t seen = generation_.load(std::memory_order_acquire);
        for (;;) {
            // Poll for up to 500 us, then sleep until the next generation.
            const auto poll_until = std::chrono::steady_clock::now() + std::chrono::microseconds(500);
            while (generation_.load(std::memory_order_acquire) == seen &&
                   std::chrono::steady_clock::now() < poll_until) {
                std::this_thread::yield();
            }
            const std::function<void(int64_t, int64_t)>* body;
            int64_t n, grain;
            {
                std::unique_lock<std::mutex> lock(mutex_);
                wake_.wait(lock, [&] { return generation_.load(std::memory_order_relaxed) != seen; });
                seen = generation_.load(std::memory_order_relaxed);
                if (body_ == nullptr || remaining_.load(std::memory_order_relaxed) == 0) continue;
                body = body_;
                n = n_;
                grain = grain_;
                ++in_flight_;
            }
            run_chunks(*body, n, grain);
            {
                std::lock_guard<std::mutex> lock(mutex_);
                --in_flight_;
                done_.notify_all();
            }
        }
    }

    std::vector<std::thread> workers_;
    std::mutex call_mutex_;
    std::mutex mutex_;
    std::condition_variable wake_;
    std::condition_variable done_;
    const std::function<void(int64_t, int64_t)>* body_ = nullptr;
    int64_t n_ = 0;
    int64_t grain_ = 1;
    std::atomic<int64_t> next_{0};
    std::atomic<int64_t> remaining_{0};
    int in_flight_ = 0;
    std::atomic<uint64_t> generation_{0};
};

}  // namespace tnr
