// A small pool of persistent host threads for the data plane's per-call
// host work (the padded batch page table of paged_attention_batch): the
// caller and up to kMaxWorkers threads take chunks of rows from a shared
// counter. One job runs at a time; concurrent callers queue on a mutex.
// The pool is sized to the CPUs this process may run on, shared among the
// processes of one node when a launcher says how many there are
// (LOCAL_WORLD_SIZE, one process per GPU): a worker preempted while it holds
// a chunk would hold up the whole job.
#include <sched.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdlib>
#include <exception>
#include <mutex>
#include <thread>

#include "runtime.h"

namespace kvflux::v2::detail {
namespace {

constexpr unsigned kMaxWorkers = 7;

// CPUs in this process's affinity mask (all CPUs if it cannot be read),
// divided among LOCAL_WORLD_SIZE processes when that is set above 1.
unsigned usable_cpus() {
    unsigned cpus = std::thread::hardware_concurrency();
    cpu_set_t set;
    CPU_ZERO(&set);
    if (sched_getaffinity(0, sizeof(set), &set) == 0 && CPU_COUNT(&set) > 0) {
        cpus = static_cast<unsigned>(CPU_COUNT(&set));
    }
    if (const char* s = std::getenv("LOCAL_WORLD_SIZE")) {
        const long procs = std::strtol(s, nullptr, 10);
        if (procs > 1) cpus = std::max(1u, cpus / static_cast<unsigned>(procs));
    }
    return cpus;
}

class Pool {
public:
    Pool() {
        const unsigned cpus = usable_cpus();
        const unsigned n = cpus > 1 ? std::min(kMaxWorkers, cpus - 1) : 0;
        for (unsigned i = 0; i < n; ++i) workers_.emplace_back([this] { loop(); });
    }

    ~Pool() {
        {
            std::lock_guard<std::mutex> lock(mu_);
            stop_ = true;
        }
        cv_.notify_all();
        for (std::thread& t : workers_) t.join();
    }

    void run(std::size_t n, std::size_t grain, const std::function<void(std::size_t, std::size_t)>& fn) {
        std::lock_guard<std::mutex> job_lock(job_mu_);
        {
            std::lock_guard<std::mutex> lock(mu_);
            fn_ = &fn;
            n_ = n;
            grain_ = grain;
            next_.store(0, std::memory_order_relaxed);
            busy_ = workers_.size();
            error_ = nullptr;
            ++generation_;
        }
        cv_.notify_all();
        work();
        std::unique_lock<std::mutex> lock(mu_);
        done_cv_.wait(lock, [this] { return busy_ == 0; });
        fn_ = nullptr;
        if (error_) std::rethrow_exception(error_);
    }

private:
    // Takes chunks until none is left; the first exception is kept.
    void work() {
        for (;;) {
            const std::size_t begin = next_.fetch_add(grain_, std::memory_order_relaxed);
            if (begin >= n_) return;
            try {
                (*fn_)(begin, std::min(n_, begin + grain_));
            } catch (...) {
                std::lock_guard<std::mutex> lock(mu_);
                if (!error_) error_ = std::current_exception();
            }
        }
    }

    void loop() {
        std::uint64_t seen = 0;
        for (;;) {
            {
                std::unique_lock<std::mutex> lock(mu_);
                cv_.wait(lock, [&] { return stop_ || generation_ != seen; });
                if (stop_) return;
                seen = generation_;
            }
            work();
            {
                std::lock_guard<std::mutex> lock(mu_);
                --busy_;
            }
            done_cv_.notify_one();
        }
    }

    std::vector<std::thread> workers_;
    std::mutex job_mu_;
    std::mutex mu_;
    std::condition_variable cv_, done_cv_;
    const std::function<void(std::size_t, std::size_t)>* fn_ = nullptr;
    std::size_t n_ = 0, grain_ = 1;
    std::atomic<std::size_t> next_{0};
    std::size_t busy_ = 0;
    std::uint64_t generation_ = 0;
    bool stop_ = false;
    std::exception_ptr error_;
};

}  // namespace

void parallel_for(std::size_t n, std::size_t grain, const std::function<void(std::size_t, std::size_t)>& fn) {
    if (grain == 0) grain = 1;
    if (n <= grain) {
        if (n != 0) fn(0, n);
        return;
    }
    static Pool pool;
    pool.run(n, grain, fn);
}

} // namespace kvflux::v2::detail
