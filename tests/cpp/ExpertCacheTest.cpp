// ExpertCacheTest.cpp -- litemind::b200::ExpertCache against the reference's own
// counters.  Reads a touch sequence and the reference ExpertCache's statistics after
// every touch (tests/golden/cache.json, flattened by the pytest driver into
// `layer expert resident_bytes resident_experts loads hits evictions streamed`
// lines), replays it and compares.  No GPU: the cache is not attached to a layer.
#include <cstdint>
#include <fstream>
#include <iostream>
#include <string>

#include "TestSupport.hpp"
#include "litemind_b200/ExpertCache.hpp"

using namespace test_support;

int main(int argc, char** argv) {
    if (argc != 2) {
        std::cerr << "usage: ExpertCacheTest <sequence.txt>\n";
        return 2;
    }
    std::ifstream in(argv[1]);
    std::uint64_t budget = 0, block = 0;
    in >> budget >> block;
    litemind::b200::ExpertCache cache;
    check(!cache.enabled(), "a fresh cache is disabled");
    cache.configure(budget);
    check(cache.enabled() && cache.budget_bytes() == budget, "configure sets the budget");
    const litemind::b200::ExpertCache::Block b{nullptr, nullptr, nullptr, block / 3, block / 3, block - 2 * (block / 3)};
    std::uint64_t layer, expert, rb, re, loads, hits, ev, streamed;
    int step = 0;
    while (in >> layer >> expert >> rb >> re >> loads >> hits >> ev >> streamed) {
        if (layer == 999999U) {  // the final line: statistics after clear()
            cache.clear();
        } else {
            cache.touch(litemind::b200::ExpertCache::make_key(layer, expert), b);
        }
        const std::string at = " at step " + std::to_string(step++);
        check(cache.resident_bytes() == rb, "resident bytes" + at);
        check(cache.resident_experts() == re, "resident experts" + at);
        check(cache.loads() == loads, "loads" + at);
        check(cache.hits() == hits, "hits" + at);
        check(cache.evictions() == ev, "evictions" + at);
        check(cache.bytes_streamed() == streamed, "bytes streamed" + at);
    }
    check(step > 10, "the sequence was read");
    litemind::b200::ExpertCache off;
    off.touch(1U, b);
    check(off.loads() == 0U && off.resident_experts() == 0U, "a zero budget leaves paging alone (no bookkeeping)");
    return report("ExpertCacheTest (B200 residency)");
}
