// ExpertCache.cpp -- litemind::b200::ExpertCache, the reference ExpertCache's
// bookkeeping contract (include/ExpertCache.hpp:29-89 of the reference) over a
// residency ledger of its own: a touch of a resident expert counts a hit and makes
// it the most recent; a touch of a new one first drops least-recently-touched
// experts until it fits the budget (or nothing is left), then loads it -- an upload
// into the attached layer's HBM -- and counts a load and its bytes.  A zero budget
// disables the bookkeeping altogether.  The counters match the reference's after
// every touch (tests/golden/cache.json holds a sequence recorded from it).
#include "litemind_b200/ExpertCache.hpp"

#include "litemind_b200/MoeLayer.hpp"

namespace litemind::b200 {

void ExpertCache::configure(std::uint64_t budget_bytes) noexcept { budget_bytes_ = budget_bytes; }

void ExpertCache::touch(std::uint64_t key, const Block& block) {
    if (budget_bytes_ == 0U) return;
    const std::uint64_t now = ++clock_;
    if (const auto it = slot_of_.find(key); it != slot_of_.end()) {
        Slot& slot = slots_[it->second];
        by_last_touch_.erase(slot.last_touch);
        slot.last_touch = now;
        by_last_touch_.emplace(now, it->second);
        ++hits_;
        return;
    }
    const std::uint64_t bytes = block.byte_size();
    while (!by_last_touch_.empty() && resident_bytes_ + bytes > budget_bytes_) drop_least_recent();
    if (layer_ != nullptr)
        layer_->upload_expert(static_cast<int32_t>(key >> 32U), static_cast<int32_t>(key & 0xffffffffU), block.gate,
                              block.up, block.down);
    std::uint32_t index;
    if (free_slots_.empty()) {
        index = static_cast<std::uint32_t>(slots_.size());
        slots_.push_back(Slot{});
    } else {
        index = free_slots_.back();
        free_slots_.pop_back();
    }
    slots_[index] = Slot{key, bytes, now};
    slot_of_.emplace(key, index);
    by_last_touch_.emplace(now, index);
    resident_bytes_ += bytes;
    bytes_streamed_ += bytes;
    ++loads_;
}

void ExpertCache::drop_least_recent() {
    const auto oldest = by_last_touch_.begin();
    const std::uint32_t index = oldest->second;
    by_last_touch_.erase(oldest);
    slot_of_.erase(slots_[index].key);
    resident_bytes_ -= slots_[index].bytes;
    free_slots_.push_back(index);
    ++evictions_;
}

void ExpertCache::clear() {
    while (!by_last_touch_.empty()) drop_least_recent();
    slots_.clear();
    free_slots_.clear();
    resident_bytes_ = 0U;
}

}  // namespace litemind::b200
