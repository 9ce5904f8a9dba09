// Expect.hpp -- the expectation recorder of the C++ mirror tests.  A test executable
// states its expectations through one Expect object: a missed expectation is printed
// with its description (and the values, for numeric ones) when it is evaluated, and
// finish() prints a tally and returns the process exit status, 0 when every
// expectation held.  Not thread-safe: state expectations from one thread.
#pragma once

#include <cmath>
#include <cstdio>
#include <string>
#include <string_view>
#include <utility>

class Expect {
public:
    explicit Expect(std::string suite) : suite_(std::move(suite)) {}

    /** Records one yes/no expectation; returns it. */
    bool operator()(bool held, std::string_view what) {
        ++stated_;
        if (!held) miss(what, "");
        return held;
    }

    /** Records |got - want| <= tolerance. */
    bool near(double got, double want, double tolerance, std::string_view what) {
        ++stated_;
        const bool held = std::fabs(got - want) <= tolerance;
        if (!held) {
            char detail[160];
            std::snprintf(detail, sizeof(detail), " (got %.9g, want %.9g +- %.3g)", got, want, tolerance);
            miss(what, detail);
        }
        return held;
    }

    /** Prints the tally; the exit status for main(). */
    [[nodiscard]] int finish() const {
        if (missed_ == 0) {
            std::printf("%s: all %d expectations held\n", suite_.c_str(), stated_);
            return 0;
        }
        std::fprintf(stderr, "%s: %d of %d expectations missed\n", suite_.c_str(), missed_, stated_);
        return 1;
    }

private:
    void miss(std::string_view what, const char* detail) {
        ++missed_;
        std::fprintf(stderr, "[%s] missed: %.*s%s\n", suite_.c_str(), static_cast<int>(what.size()), what.data(),
                     detail);
    }

    std::string suite_;
    int stated_{0};
    int missed_{0};
};
