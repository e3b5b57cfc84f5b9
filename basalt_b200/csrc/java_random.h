// java.util.Random for the host side of the engine, from the JDK's published specification:
// a 48-bit linear congruential generator x' = (0x5DEECE66D * x + 0xB) mod 2^48, seeded by
// setSeed(s) = (s ^ 0x5DEECE66D) mod 2^48. TextEngine owns one (TextEngine.java:43) and draws one
// nextDouble (two generator steps) per sampled token (TextEngine.java:417).
#pragma once

#include <cmath>
#include <cstdint>

namespace bst {
namespace jrand {

constexpr uint64_t kMultiplier = 0x5DEECE66DULL;
constexpr uint64_t kAddend = 0xBULL;
constexpr uint64_t kMask = (1ULL << 48) - 1;

inline uint64_t scramble(int64_t seed) { return (static_cast<uint64_t>(seed) ^ kMultiplier) & kMask; }

// The state after `n` generator steps, by squaring the affine map (x -> a x + c) n's bits at a time.
inline uint64_t advance(uint64_t state, uint64_t n) {
    uint64_t mul = 1, add = 0;                    // accumulated map
    uint64_t step_mul = kMultiplier, step_add = kAddend;  // map for 2^i steps
    while (n) {
        if (n & 1) {
            mul = (mul * step_mul) & kMask;
            add = (add * step_mul + step_add) & kMask;
        }
        step_add = (step_add * step_mul + step_add) & kMask;
        step_mul = (step_mul * step_mul) & kMask;
        n >>= 1;
    }
    return (state * mul + add) & kMask;
}

struct Random {
    uint64_t state = 0;
    bool have_next_gaussian = false;
    double next_gaussian_value = 0.0;

    explicit Random(int64_t seed) : state(scramble(seed)) {}

    int32_t next(int bits) {
        state = (state * kMultiplier + kAddend) & kMask;
        return static_cast<int32_t>(static_cast<int64_t>(state) >> (48 - bits));
    }
    double next_double() {
        const int64_t hi = next(26);
        const int64_t lo = next(27);
        return static_cast<double>((hi << 27) + lo) * 0x1.0p-53;
    }
    int32_t next_int(int32_t bound) {
        int32_t r = next(31);
        const int32_t m = bound - 1;
        if ((bound & m) == 0) return static_cast<int32_t>((static_cast<int64_t>(bound) * r) >> 31);
        for (int32_t u = r;; u = next(31)) {
            r = u % bound;
            if (static_cast<int32_t>(static_cast<uint32_t>(u) - static_cast<uint32_t>(r) +
                                     static_cast<uint32_t>(m)) >= 0) {
                return r;
            }
        }
    }
    // Marsaglia polar method, as Random.nextGaussian specifies.
    double next_gaussian() {
        if (have_next_gaussian) {
            have_next_gaussian = false;
            return next_gaussian_value;
        }
        double v1, v2, s;
        do {
            v1 = 2 * next_double() - 1;
            v2 = 2 * next_double() - 1;
            s = v1 * v1 + v2 * v2;
        } while (s >= 1 || s == 0);
        const double multiplier = std::sqrt(-2 * std::log(s) / s);
        next_gaussian_value = v2 * multiplier;
        have_next_gaussian = true;
        return v1 * multiplier;
    }
};

}  // namespace jrand
}  // namespace bst
