// ExpertCacheTest.cpp -- litemind::b200::ExpertCache against the reference's own
// counters.  Reads a touch sequence and the reference ExpertCache's statistics after
// every touch (tests/golden/cache.json, flattened by the pytest driver into
// `layer expert resident_bytes resident_experts loads hits evictions streamed`
// lines, the last one -- layer 999999 -- after clear()), replays it and compares.
// Also: a zero budget keeps no books, an expert larger than the budget empties the
// ledger and is still loaded (as the reference's evict-then-load loop does), and slots
// freed by eviction are reused.  No GPU: the cache is not attached to a layer.
#include <cstdint>
#include <fstream>
#include <iostream>
#include <string>

#include "Expect.hpp"
#include "litemind_b200/ExpertCache.hpp"

using litemind::b200::ExpertCache;

int main(int argc, char** argv) {
    Expect expect("ExpertCacheTest (B200 residency)");
    if (argc != 2) {
        std::cerr << "usage: ExpertCacheTest <sequence.txt>\n";
        return 2;
    }
    std::ifstream in(argv[1]);
    std::uint64_t budget = 0, block = 0;
    in >> budget >> block;
    ExpertCache cache;
    expect(!cache.enabled(), "a fresh cache is disabled");
    cache.configure(budget);
    expect(cache.enabled() && cache.budget_bytes() == budget, "configure sets the budget");
    const ExpertCache::Block b{nullptr, nullptr, nullptr, block / 3, block / 3, block - 2 * (block / 3)};
    std::uint64_t layer, expert, rb, re, loads, hits, ev, streamed;
    int step = 0;
    while (in >> layer >> expert >> rb >> re >> loads >> hits >> ev >> streamed) {
        if (layer == 999999U) {
            cache.clear();
        } else {
            cache.touch(ExpertCache::make_key(layer, expert), b);
        }
        const std::string at = " at step " + std::to_string(step++);
        expect(cache.resident_bytes() == rb, "resident bytes" + at);
        expect(cache.resident_experts() == re, "resident experts" + at);
        expect(cache.loads() == loads, "loads" + at);
        expect(cache.hits() == hits, "hits" + at);
        expect(cache.evictions() == ev, "evictions" + at);
        expect(cache.bytes_streamed() == streamed, "bytes streamed" + at);
    }
    expect(step > 10, "the sequence was read");

    ExpertCache off;
    off.touch(1U, b);
    expect(off.loads() == 0U && off.resident_experts() == 0U, "a zero budget keeps no books");

    ExpertCache small;
    small.configure(block / 2);  // smaller than one expert
    small.touch(ExpertCache::make_key(0, 1), b);
    small.touch(ExpertCache::make_key(0, 2), b);
    expect(small.resident_experts() == 1U && small.evictions() == 1U && small.loads() == 2U,
           "an expert larger than the budget empties the ledger and is loaded anyway");
    small.touch(ExpertCache::make_key(0, 2), b);
    expect(small.hits() == 1U && small.resident_bytes() == block, "a hit keeps the one resident expert");

    ExpertCache lru;
    lru.configure(3 * block);
    for (std::uint64_t e : {1U, 2U, 3U, 1U, 4U, 5U}) lru.touch(ExpertCache::make_key(7, e), b);
    // 1 2 3 loaded; 1 hit (now most recent); 4 drops 2; 5 drops 3.
    expect(lru.loads() == 5U && lru.hits() == 1U && lru.evictions() == 2U && lru.resident_experts() == 3U,
           "least recently touched experts leave first");
    lru.touch(ExpertCache::make_key(7, 1), b);
    expect(lru.hits() == 2U, "the re-touched expert survived both evictions");
    lru.clear();
    expect(lru.resident_experts() == 0U && lru.resident_bytes() == 0U && lru.evictions() == 5U,
           "clear evicts every resident expert");
    return expect.finish();
}
