// The platform libm's expf, reproduced on the device.
//
// The reference computes softmax and MoE routing weights with the C library's
// expf (sml/sml-run.c:280-288, :3024-3032). For the GPU to pick the same
// tokens bit for bit it must produce the same floats. The device computes
// exp in double precision and rounds once to float -- the correctly rounded
// result except where the double is within a few units of its last place of
// a float rounding midpoint -- and corrects the arguments where the host's
// expf rounds differently: a table, built once per process on the host by
// calling the host's expf, of every negative argument x >= -104 (below it both
// give 0) whose libm result differs from the rounded double, or whose rounded
// double is that close to a midpoint. About 1e5 of the 1.1e9 negative floats
// (glibc's expf is within 0.502 ulp, not correctly rounded); softmax and
// routing only ever take exp of x - max <= 0.
//
// The table is an open-addressing hash of 2^kExpfBits slots (x bits, expf(x)
// bits), empty slots keyed 0xffffffff (a NaN: never an argument). libm's
// expf only rounds differently where the exact exp(x) lies very near a float
// rounding midpoint (glibc's worst case here: 0.0016 of a float ulp), so the
// device looks an argument up only when its double exp lies within `near` ulp
// of one -- about 0.2 % of arguments; the build checks that every entry
// qualifies.
#pragma once

#include <cstdint>
#include <vector>

namespace sb {

constexpr int kExpfBits = 18;

struct ExpfEntry { uint32_t x, y; };

// Slot of key k (multiplicative hash); probes continue linearly.
__host__ __device__ inline uint32_t expf_slot(uint32_t k) { return (k * 0x9E3779B1u) >> (32 - kExpfBits); }

struct ExpfTable {
    std::vector<ExpfEntry> slots;   // empty if the table could not be built
    float near;                     // midpoint distance (float ulps) below which to look up
};

// The table for this process's libm (built on first use, then shared). Empty
// if more entries than half the slots were found, or an entry lies farther
// from its midpoint than the lookup threshold could allow.
const ExpfTable & expf_libm_table();

}  // namespace sb
