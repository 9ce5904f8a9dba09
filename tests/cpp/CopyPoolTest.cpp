// The weight upload's host copy pool (litemind_b200/csrc/host/CopyPool.cpp): every
// index runs exactly once per run, runs can follow one another and be empty, a
// one-thread pool runs everything on the caller, and pieces copied in parallel
// reassemble the source.
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>

#include "CopyPool.hpp"
#include "TestSupport.hpp"

using test_support::check;

int main() {
    lm::CopyPool pool(8);
    check(pool.threads() == 8, "thread count");
    for (int rep = 0; rep < 500; ++rep) {
        const int n = 1 + rep % 97;
        std::vector<int> hits(static_cast<size_t>(n), 0);
        pool.run(n, [&](int i) { hits[static_cast<size_t>(i)] += 1; });
        bool once = true;
        for (int v : hits) once = once && v == 1;
        check(once, "every index exactly once");
        pool.run(0, [&](int) { check(false, "empty run calls nothing"); });
    }
    lm::CopyPool single(1);
    int sum = 0;
    single.run(10, [&](int i) { sum += i; });  // caller only: no race on sum
    check(sum == 45, "one-thread pool");
    // Pieces of 1 KiB copied in parallel reassemble a 1 MiB buffer.
    std::vector<uint16_t> src(1 << 19), dst(1 << 19, 0);
    std::iota(src.begin(), src.end(), uint16_t{7});
    const size_t piece = 512;
    pool.run(static_cast<int>(src.size() / piece), [&](int i) {
        std::memcpy(dst.data() + static_cast<size_t>(i) * piece, src.data() + static_cast<size_t>(i) * piece,
                    piece * sizeof(uint16_t));
    });
    check(src == dst, "parallel pieces reassemble the source");
    return test_support::report("CopyPoolTest");
}
