// The weight upload's host copy pool (litemind_b200/csrc/host/CopyPool.cpp): every
// index runs exactly once per run, runs can follow one another and be empty, a
// one-thread pool runs everything on the caller, and pieces copied in parallel
// reassemble the source.
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>

#include "CopyPool.hpp"
#include "Expect.hpp"

int main() {
    Expect expect("CopyPoolTest");
    lm::CopyPool pool(8);
    expect(pool.threads() == 8, "thread count");
    for (int rep = 0; rep < 500; ++rep) {
        const int n = 1 + rep % 97;
        std::vector<int> hits(static_cast<size_t>(n), 0);
        pool.run(n, [&](int i) { hits[static_cast<size_t>(i)] += 1; });
        bool once = true;
        for (int v : hits) once = once && v == 1;
        expect(once, "every index exactly once");
        pool.run(0, [&](int) { expect(false, "empty run calls nothing"); });
    }
    lm::CopyPool single(1);
    int sum = 0;
    single.run(10, [&](int i) { sum += i; });  // caller only: no race on sum
    expect(sum == 45, "one-thread pool");
    // Pieces of 1 KiB copied in parallel reassemble a 1 MiB buffer.
    std::vector<uint16_t> src(1 << 19), dst(1 << 19, 0);
    std::iota(src.begin(), src.end(), uint16_t{7});
    const size_t piece = 512;
    pool.run(static_cast<int>(src.size() / piece), [&](int i) {
        std::memcpy(dst.data() + static_cast<size_t>(i) * piece, src.data() + static_cast<size_t>(i) * piece,
                    piece * sizeof(uint16_t));
    });
    expect(src == dst, "parallel pieces reassemble the source");
    return expect.finish();
}
