// CopyPool.cpp -- see CopyPool.hpp.
#include "CopyPool.hpp"

namespace lm {

CopyPool::CopyPool(int threads) {
    for (int i = 1; i < threads; ++i) workers_.emplace_back([this] { loop(); });
}

CopyPool::~CopyPool() {
    {
        std::lock_guard<std::mutex> lock(mu_);
        stop_ = true;
    }
    work_cv_.notify_all();
    for (std::thread& t : workers_) t.join();
}

bool CopyPool::claim(int* index) {
    if (fn_ == nullptr || next_ >= n_) return false;
    *index = next_++;
    ++active_;
    return true;
}

void CopyPool::run(int n, const std::function<void(int)>& fn) {
    std::unique_lock<std::mutex> lock(mu_);
    fn_ = &fn;
    n_ = n;
    next_ = 0;
    active_ = 0;
    lock.unlock();
    work_cv_.notify_all();
    lock.lock();
    int i = 0;
    while (claim(&i)) {
        lock.unlock();
        fn(i);
        lock.lock();
        --active_;
    }
    done_cv_.wait(lock, [&] { return next_ >= n_ && active_ == 0; });
    fn_ = nullptr;
}

void CopyPool::loop() {
    std::unique_lock<std::mutex> lock(mu_);
    for (;;) {
        work_cv_.wait(lock, [&] { return stop_ || (fn_ != nullptr && next_ < n_); });
        if (stop_) return;
        int i = 0;
        while (claim(&i)) {
            const std::function<void(int)>* fn = fn_;
            lock.unlock();
            (*fn)(i);
            lock.lock();
            --active_;
        }
        done_cv_.notify_all();
    }
}

}  // namespace lm
