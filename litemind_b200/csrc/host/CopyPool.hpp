// CopyPool.hpp -- a small fixed set of host threads for parallel copies into pinned
// staging memory (weight upload), so host-side copying keeps pace with the
// host-to-device DMA.
#pragma once

#include <condition_variable>
#include <cstdint>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

namespace lm {

// run(n, fn) calls fn(0) .. fn(n - 1) on the pool's threads and the caller's own,
// and returns once all have finished.  One run at a time.
class CopyPool {
public:
    explicit CopyPool(int threads);
    ~CopyPool();
    CopyPool(const CopyPool&) = delete;
    CopyPool& operator=(const CopyPool&) = delete;

    int threads() const { return static_cast<int>(workers_.size()) + 1; }
    void run(int n, const std::function<void(int)>& fn);

private:
    void loop();
    bool claim(int* index);  // under mu_

    std::vector<std::thread> workers_;
    std::mutex mu_;
    std::condition_variable work_cv_;
    std::condition_variable done_cv_;
    const std::function<void(int)>* fn_ = nullptr;
    int n_ = 0;
    int next_ = 0;
    int active_ = 0;
    bool stop_ = false;
};

}  // namespace lm
