// ExpertCache.hpp -- litemind::ExpertCache's interface (include/ExpertCache.hpp:29-89 of
// the reference) over HBM residency.
//
// The reference keeps an LRU working set of experts in RAM under a byte budget,
// streaming them from SSD on touch() and releasing them on eviction.  On the B200
// every expert of every resident layer lives in HBM, so paging disappears; this
// class keeps the same bookkeeping and counters (loads, hits, evictions,
// bytes_streamed, resident bytes and experts, with the reference's LRU order and
// evict-before-load rule) so callers and their reports keep working.  When attached
// to a MoeLayer, a touch() that loads an expert uploads it to the device (the
// reference's SSD read becomes a host-to-HBM copy); evictions are bookkeeping only,
// since device memory for every expert is reserved up front.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <unordered_map>
#include <vector>

namespace litemind::b200 {

class MoeLayer;

class ExpertCache final {
public:
    /** The three matrices of one expert's SwiGLU block, as host pointers and sizes. */
    struct Block final {
        const std::uint16_t* gate{nullptr};  ///< [inter, hidden] bf16
        const std::uint16_t* up{nullptr};    ///< [inter, hidden] bf16
        const std::uint16_t* down{nullptr};  ///< [hidden, inter] bf16
        std::uint64_t gate_bytes{};
        std::uint64_t up_bytes{};
        std::uint64_t down_bytes{};

        [[nodiscard]] std::uint64_t byte_size() const noexcept { return gate_bytes + up_bytes + down_bytes; }
    };

    ExpertCache() = default;

    /** Sets the residency budget in bytes.  Zero disables the bookkeeping. */
    void configure(std::uint64_t budget_bytes) noexcept;

    /** Uploads loaded experts into `layer` from now on (nullptr: bookkeeping only). */
    void attach(MoeLayer* layer) noexcept { layer_ = layer; }

    /** Marks an expert as needed now, evicting least-recently-used ones first if it would not fit. */
    void touch(std::uint64_t key, const Block& block);

    /** Evicts everything. */
    void clear();

    [[nodiscard]] bool enabled() const noexcept { return budget_bytes_ != 0U; }
    [[nodiscard]] std::uint64_t budget_bytes() const noexcept { return budget_bytes_; }
    [[nodiscard]] std::uint64_t resident_bytes() const noexcept { return resident_bytes_; }
    [[nodiscard]] std::size_t resident_experts() const noexcept { return slot_of_.size(); }
    [[nodiscard]] std::uint64_t loads() const noexcept { return loads_; }
    [[nodiscard]] std::uint64_t hits() const noexcept { return hits_; }
    [[nodiscard]] std::uint64_t evictions() const noexcept { return evictions_; }
    [[nodiscard]] std::uint64_t bytes_streamed() const noexcept { return bytes_streamed_; }

    /** The reference's key: layer in the high 32 bits, expert in the low 32. */
    [[nodiscard]] static std::uint64_t make_key(std::size_t layer, std::size_t expert) noexcept {
        return (static_cast<std::uint64_t>(layer) << 32U) | static_cast<std::uint32_t>(expert);
    }

private:
    // The residency ledger: one slot per resident expert in a flat vector (slots of
    // evicted experts are reused), the key -> slot index, and the slots ordered by
    // the tick of their last touch -- the smallest tick is the least recently used.
    struct Slot final {
        std::uint64_t key{};
        std::uint64_t bytes{};
        std::uint64_t last_touch{};
    };

    void drop_least_recent();

    MoeLayer* layer_{nullptr};
    std::uint64_t budget_bytes_{};
    std::uint64_t resident_bytes_{};
    std::uint64_t clock_{};
    std::vector<Slot> slots_;
    std::vector<std::uint32_t> free_slots_;
    std::unordered_map<std::uint64_t, std::uint32_t> slot_of_;
    std::map<std::uint64_t, std::uint32_t> by_last_touch_;
    std::uint64_t loads_{};
    std::uint64_t hits_{};
    std::uint64_t evictions_{};
    std::uint64_t bytes_streamed_{};
};

}  // namespace litemind::b200
