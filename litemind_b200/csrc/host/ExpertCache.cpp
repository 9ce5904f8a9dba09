// ExpertCache.cpp -- litemind::b200::ExpertCache: the reference's working-set
// bookkeeping (src/ExpertCache.cpp:5-76: LRU order, make room before loading, the
// same counters) with loads becoming host-to-HBM uploads when attached to a layer.
#include "litemind_b200/ExpertCache.hpp"

#include "litemind_b200/MoeLayer.hpp"

namespace litemind::b200 {

void ExpertCache::configure(std::uint64_t budget_bytes) noexcept { budget_bytes_ = budget_bytes; }

void ExpertCache::touch(std::uint64_t key, const Block& block) {
    if (!enabled()) return;
    if (auto found = entries_.find(key); found != entries_.end()) {
        recency_.splice(recency_.begin(), recency_, found->second.position);
        found->second.position = recency_.begin();
        ++hits_;
        return;
    }
    const std::uint64_t bytes = block.byte_size();
    while (resident_bytes_ + bytes > budget_bytes_ && !recency_.empty()) evict_oldest();
    if (layer_ != nullptr)
        layer_->upload_expert(static_cast<int32_t>(key >> 32U), static_cast<int32_t>(key & 0xffffffffU), block.gate,
                              block.up, block.down);
    recency_.push_front(key);
    entries_.emplace(key, Entry{bytes, recency_.begin()});
    resident_bytes_ += bytes;
    bytes_streamed_ += bytes;
    ++loads_;
}

void ExpertCache::evict_oldest() {
    if (recency_.empty()) return;
    const std::uint64_t key = recency_.back();
    recency_.pop_back();
    if (auto found = entries_.find(key); found != entries_.end()) {
        resident_bytes_ -= found->second.bytes;
        entries_.erase(found);
        ++evictions_;
    }
}

void ExpertCache::clear() {
    while (!recency_.empty()) evict_oldest();
    entries_.clear();
    resident_bytes_ = 0U;
}

}  // namespace litemind::b200
