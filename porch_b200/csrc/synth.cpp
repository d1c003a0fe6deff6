// Seeded synthetic inputs (pb_fill_synthetic in include/porch_b200.h).
//
// Counter-based: element i is a SplitMix64 hash of (seed, i), so the stream
// does not depend on how the work is split across threads. Uniform values use
// 24 random mantissa bits; normal values use Box-Muller in double on two
// per-element uniforms, rounded once to float. This file has no dependency on
// the rest of the library so the reference-side benchmark runner can compile
// the same generator and see bit-identical inputs.
#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <thread>
#include <vector>

namespace {

    uint64_t splitmix(uint64_t x) {
        x += 0x9e3779b97f4a7c15ULL;
        x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
        x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
        return x ^ (x >> 31);
    }

    double unit(uint64_t seed, uint64_t i) {
        return static_cast<double>(splitmix(seed * 0xd1b54a32d192ed03ULL + i) >> 40) *
               (1.0 / 16777216.0);
    }

} // namespace

extern "C" int pb_fill_synthetic(float* values, size_t count, uint64_t seed, int dist,
                                 double a, double b) {
    if (count != 0 && values == nullptr) return 1;
    if (dist != 0 && dist != 1) return 1;
    auto work = [&](size_t begin, size_t end) {
        for (size_t i = begin; i < end; ++i) {
            double v;
            if (dist == 0) {
                v = a + (b - a) * unit(seed, i);
            } else {
                const double u1 = unit(seed, 2 * static_cast<uint64_t>(i));
                const double u2 = unit(seed, 2 * static_cast<uint64_t>(i) + 1);
                const double r = std::sqrt(-2.0 * std::log(1.0 - u1));
                v = a + b * r * std::cos(6.283185307179586476925 * u2);
            }
            values[i] = static_cast<float>(v);
        }
    };
    const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t nthreads = std::min<size_t>(hw, std::max<size_t>(1, count >> 16));
    if (nthreads <= 1) {
        work(0, count);
        return 0;
    }
    std::vector<std::thread> pool;
    const size_t chunk = (count + nthreads - 1) / nthreads;
    for (size_t t = 0; t < nthreads; ++t) {
        const size_t begin = t * chunk;
        const size_t end = std::min(count, begin + chunk);
        if (begin < end) pool.emplace_back(work, begin, end);
    }
    for (auto& th : pool) th.join();
    return 0;
}
