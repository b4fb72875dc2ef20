// Host side of expf_libm.h: the correction table, built by calling this
// process's libm over every negative float down to -104 (threads share the
// range; ~2 s of CPU on 8 cores, once per process).
#include "expf_libm.h"

#include <cmath>
#include <cstring>
#include <mutex>
#include <thread>

namespace sb {

namespace {

float bits_f(uint32_t b) { float f; std::memcpy(&f, &b, 4); return f; }
uint32_t f_bits(float f) { uint32_t b; std::memcpy(&b, &f, 4); return b; }

// Distance of d from the float rounding midpoint nearest it, in float ulps (of
// the spacing on d's side of its rounding c).
double mid_dist(double d, float c) {
    if ((double) c == d) return 0.5;
    const float nb = nextafterf(c, d > (double) c ? INFINITY : 0.0f);
    const double mid = 0.5 * ((double) c + (double) nb);
    return fabs(d - mid) / fabs((double) nb - (double) c);
}

// libm's expf differs from exp rounded to float, or that rounding sits within
// 8 double ulps of a float midpoint (so a device exp one ulp off could round
// the other way). *dist: the midpoint distance in float ulps.
bool needs_entry(float x, float * libm, double * dist) {
    const float a = expf(x);
    const double d = exp((double) x);
    const float c = (float) d;
    *libm = a;
    *dist = mid_dist(d, c);
    if (f_bits(a) != f_bits(c)) return true;
    if ((double) c == d) return false;
    const float nb = nextafterf(c, d > (double) c ? INFINITY : 0.0f);
    const double mid = 0.5 * ((double) c + (double) nb);
    const double ulp = nextafter(d, INFINITY) - d;
    return fabs(d - mid) <= 8.0 * ulp;
}

ExpfTable build() {
    const uint32_t lo = 0x80000001u;                 // -smallest denormal
    const uint32_t hi = f_bits(-104.0f);             // ... down to -104
    unsigned nt = std::thread::hardware_concurrency();
    if (nt < 1) nt = 1;
    if (nt > 64) nt = 64;
    std::vector<std::vector<ExpfEntry>> part(nt);
    std::vector<double> far(nt, 0.0);   // the largest midpoint distance of an entry
    std::vector<std::thread> th;
    const uint64_t span = (uint64_t) hi - lo + 1;
    for (unsigned t = 0; t < nt; t++)
        th.emplace_back([&, t] {
            const uint64_t b0 = lo + span * t / nt, b1 = lo + span * (t + 1) / nt;
            for (uint64_t b = b0; b < b1; b++) {
                float y;
                double dist;
                if (needs_entry(bits_f((uint32_t) b), &y, &dist)) {
                    part[t].push_back({(uint32_t) b, f_bits(y)});
                    if (dist > far[t]) far[t] = dist;
                }
            }
        });
    for (auto & x : th) x.join();
    ExpfTable out;
    double worst = 0.0;
    for (double f : far) worst = f > worst ? f : worst;
    // look up everything within twice the worst entry's distance (at least
    // 0.001 ulp); an entry near 0.25 ulp would make lookups too frequent
    out.near = (float) (2.0 * worst > 1e-3 ? 2.0 * worst : 1e-3);
    const uint32_t slots = 1u << kExpfBits;
    size_t n = 0;
    for (auto & p : part) n += p.size();
    if (n > slots / 2 || out.near > 0.05f) return out;
    out.slots.assign(slots, ExpfEntry{0xffffffffu, 0u});
    for (auto & p : part)
        for (const ExpfEntry & e : p) {
            uint32_t h = expf_slot(e.x);
            while (out.slots[h].x != 0xffffffffu) h = (h + 1) & (slots - 1);
            out.slots[h] = e;
        }
    return out;
}

}  // namespace

const ExpfTable & expf_libm_table() {
    static std::once_flag once;
    static ExpfTable tab;
    std::call_once(once, [] { tab = build(); });
    return tab;
}

}  // namespace sb
