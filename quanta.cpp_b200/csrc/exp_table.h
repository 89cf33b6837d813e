// Host-measured exceptions of the libm's expf (see exp_table.cpp) and the device-side e^x that uses them.
#pragma once

#include <stdint.h>

#include <string>
#include <vector>

namespace qb {

// An input is looked up only when the double-precision e^x lies within this fraction of a half-ulp of a rounding
// midpoint (the libm's error bound, 0.502 ulp, allows a different choice only within 0.002 ulp of one).
constexpr double kExpNearMidpoint = 0.008;

#if defined(__CUDACC__)
__host__ __device__
#endif
inline uint32_t exp_hash(uint32_t key) {
    return (key * 2654435761u) ^ (key >> 15);
}

// Open-addressing table: slot = (x bits << 32) | expf(x) bits, empty = all ones; size a power of two.
struct ExpTab {
    const unsigned long long* slots = nullptr;
    unsigned mask = 0;
};

// Builds (once per process) the table of every float x in (-104, 89) whose libm expf differs from the correctly
// rounded double exp.  note receives "cached <file>" or "scanned (...)".
const std::vector<uint64_t>& expf_exception_slots(std::string* note);

#if defined(__CUDACC__)
// e^x with the host libm's bits: the double exp rounded once, corrected from the table near rounding midpoints.
// The table holds every input whose expf differs from that rounding, so probing a superset of the near-midpoint
// inputs is still exact (a miss returns the rounding).  For y >= 2^-126 the float keeps the top 23 of the double's 52
// mantissa bits, and the dropped 29 bits r place y against the midpoint at r = 2^28: |r - 2^28| < 2^22 (0.0078 ulp)
// covers the window above (0.004 ulp); tests/test_exp_midpoint.py checks every r of two edge binades.  Smaller y
// (a subnormal float) keeps the direct test.
__device__ __forceinline__ float exp_ref(float x, const ExpTab& tab) {
    const double y = exp(double(x));
    const float f = float(y);
    if (tab.slots != nullptr && f != 0.f && !isinf(f)) {
        const unsigned long long yb = static_cast<unsigned long long>(__double_as_longlong(y));
        bool near;
        if ((yb >> 52) >= 1023ull - 126ull) {  // y >= 2^-126 (y > 0)
            const int r = int(yb & 0x1fffffffull);
            near = abs(r - (1 << 28)) < (1 << 22);
        } else {
            const double df = double(f), e = y - df;
            const float nb = e >= 0 ? nextafterf(f, INFINITY) : nextafterf(f, -INFINITY);
            const double half = fabs(double(nb) - df) * 0.5;
            near = half - fabs(e) < half * kExpNearMidpoint;
        }
        if (near) {
            const unsigned key = __float_as_uint(x);
            unsigned h = exp_hash(key) & tab.mask;
            for (int probe = 0; probe <= int(tab.mask); ++probe) {
                const unsigned long long s = __ldg(tab.slots + h);
                if (s == ~0ULL) break;
                if (unsigned(s >> 32) == key) return __uint_as_float(unsigned(s));
                h = (h + 1) & tab.mask;
            }
        }
    }
    return f;
}
#endif

}  // namespace qb
