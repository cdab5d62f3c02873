// vb_synth.cpp -- seeded synthetic weights: N(0, std) f32.
//
// Counter-based so any slice can be produced independently and the result
// does not depend on the thread count: element pair p uses the SplitMix64
// finaliser (Steele, Lea & Flood, "Fast splittable pseudorandom number
// generators", OOPSLA 2014) of seed + (p+1)*golden-gamma as two 24-bit
// uniforms in (0,1), turned into two normals by the Box-Muller transform.
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <thread>
#include <vector>

#include "verbum_b200.h"

namespace {

inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

void fill_range(float* out, uint64_t n, uint64_t seed, float stdv, uint64_t p0, uint64_t p1) {
    const double two_pi = 6.283185307179586476925286766559;
    for (uint64_t p = p0; p < p1; p++) {
        const uint64_t z = mix64(seed + (p + 1) * 0x9E3779B97F4A7C15ull);
        const double u1 = ((double)(z >> 40) + 0.5) * (1.0 / 16777216.0);
        const double u2 = ((double)(z & 0xFFFFFFull) + 0.5) * (1.0 / 16777216.0);
        const double r = sqrt(-2.0 * log(u1));
        const double a = two_pi * u2;
        const uint64_t i = 2 * p;
        out[i] = (float)(r * cos(a) * stdv);
        if (i + 1 < n) out[i + 1] = (float)(r * sin(a) * stdv);
    }
}

}  // namespace

extern "C" void vb_synth_normal(float* out, uint64_t n, uint64_t seed, float stdv) {
    if (!out || n == 0) return;
    const uint64_t pairs = (n + 1) / 2;
    unsigned hw = std::thread::hardware_concurrency();
    unsigned nt = std::max(1u, std::min(hw ? hw : 1u, 64u));
    if (pairs < (1u << 16)) nt = 1;
    std::vector<std::thread> th;
    const uint64_t per = (pairs + nt - 1) / nt;
    for (unsigned t = 0; t < nt; t++) {
        const uint64_t a = t * per, b = std::min(pairs, a + per);
        if (a >= b) break;
        th.emplace_back(fill_range, out, n, seed, stdv, a, b);
    }
    for (auto& t : th) t.join();
}
