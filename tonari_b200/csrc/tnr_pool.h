// A persistent pool of host threads for the per-structure host work of a
// call (periodic geometry, cell plans).  Threads are started once per process
// and sleep between calls; parallel_for hands out fixed-size chunks through
// an atomic counter and the calling thread takes chunks too.  Calls from
// several host threads are serialised.
#pragma once

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdint>
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
            active_ = static_cast<int>(std::min<int64_t>(chunks - 1, static_cast<int64_t>(workers_.size())));
            pending_ = active_;
            ++generation_;
        }
        wake_.notify_all();
        run_chunks(body, n, grain);
        std::unique_lock<std::mutex> lock(mutex_);
        done_.wait(lock, [&] { return pending_ == 0; });
        body_ = nullptr;
    }

    HostPool(const HostPool&) = delete;
    HostPool& operator=(const HostPool&) = delete;

private:
    HostPool() {
        const unsigned hardware = std::max(1u, std::thread::hardware_concurrency());
        const unsigned count = std::min(hardware, 64u) - 1;
        for (unsigned k = 0; k < count; ++k) {
            workers_.emplace_back([this, k] { loop(static_cast<int>(k)); });
            workers_.back().detach();
        }
    }
    ~HostPool() = default;

    void run_chunks(const std::function<void(int64_t, int64_t)>& body, int64_t n, int64_t grain) {
        for (;;) {
            const int64_t begin = next_.fetch_add(grain, std::memory_order_relaxed);
            if (begin >= n) return;
            body(begin, std::min(n, begin + grain));
        }
    }

    void loop(int index) {
        uint64_t seen = 0;
        for (;;) {
            const std::function<void(int64_t, int64_t)>* body;
            int64_t n, grain;
            {
                std::unique_lock<std::mutex> lock(mutex_);
                wake_.wait(lock, [&] { return generation_ != seen; });
                seen = generation_;
                if (index >= active_) continue;
                body = body_;
                n = n_;
                grain = grain_;
            }
            run_chunks(*body, n, grain);
            {
                std::lock_guard<std::mutex> lock(mutex_);
                if (--pending_ == 0) done_.notify_one();
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
    int active_ = 0;
    int pending_ = 0;
    uint64_t generation_ = 0;
};

}  // namespace tnr
