// TestSupport.hpp -- minimal check/report helpers for the C++ mirror tests, in the
// style of the reference's tests (one executable per test, exit code = result).
#pragma once

#include <cmath>
#include <iostream>
#include <string>

namespace test_support {

inline int failures = 0;

inline void check(bool condition, const std::string& what) {
    if (!condition) {
        std::cerr << "  FAILED: " << what << "\n";
        ++failures;
    }
}

inline void check_close(double actual, double expected, double tolerance, const std::string& what) {
    if (!(std::abs(actual - expected) <= tolerance)) {
        std::cerr << "  FAILED: " << what << " (expected " << expected << ", got " << actual << ")\n";
        ++failures;
    }
}

inline int report(const std::string& name) {
    if (failures == 0) {
        std::cout << name << ": all checks passed.\n";
        return 0;
    }
    std::cerr << name << ": " << failures << " check(s) failed.\n";
    return 1;
}

}  // namespace test_support
