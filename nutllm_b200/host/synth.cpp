/* Seeded synthetic inputs for benchmarks and parity runs.
 *
 * The reference has no seeded N(0, sigma) initialiser (its tests draw from
 * std::mt19937 + uniform_real_distribution), and std::normal_distribution
 * output is specific to a standard library.  Inputs are therefore generated
 * once on the host by this documented, counter-based generator and the
 * identical bytes are fed to every implementation:
 *
 *   key      = splitmix64(seed ^ splitmix64(stream))
 *   u1, u2   = 53-bit uniforms in (0, 1] from splitmix64(key + 2j),
 *              splitmix64(key + 2j + 1)
 *   z0, z1   = Box-Muller in double: r = sqrt(-2 ln u1), t = 2 pi u2,
 *              z0 = r cos t, z1 = r sin t
 *   out[2j]  = float(sigma * z0), out[2j+1] = float(sigma * z1)
 *
 * Element i depends only on (seed, stream, i), so a matrix can be generated
 * by any number of threads, and streams (one per tensor) are independent.
 */
#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <thread>
#include <vector>

namespace {

inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

inline double unit(uint64_t bits) {
    return double((bits >> 11) + 1) * (1.0 / 9007199254740992.0);
}

void normal_range(uint64_t key, double sigma, float *out, size_t begin,
                  size_t end) {
    const double two_pi = 6.283185307179586476925286766559;
    for (size_t pair = begin / 2; pair * 2 < end; pair++) {
        const double u1 = unit(splitmix64(key + 2 * pair));
        const double u2 = unit(splitmix64(key + 2 * pair + 1));
        const double r = std::sqrt(-2.0 * std::log(u1));
        const double t = two_pi * u2;
        const size_t i = pair * 2;
        if (i >= begin)
            out[i] = float(sigma * (r * std::cos(t)));
        if (i + 1 < end)
            out[i + 1] = float(sigma * (r * std::sin(t)));
    }
}

template <typename F> void split(size_t n, F &&body) {
    const size_t hw = std::max(1u, std::thread::hardware_concurrency());
    const size_t threads = std::min<size_t>(hw, std::max<size_t>(1, n >> 16));
    if (threads <= 1) {
        body(size_t(0), n);
        return;
    }
    std::vector<std::thread> pool;
    for (size_t t = 1; t < threads; t++) {
        /* keep pair boundaries on even indices */
        const size_t b = (n * t / threads) & ~size_t(1);
        const size_t e = t + 1 == threads ? n : (n * (t + 1) / threads) & ~size_t(1);
        pool.emplace_back([&body, b, e] { body(b, e); });
    }
    body(0, (n / threads) & ~size_t(1));
    for (auto &th : pool)
        th.join();
}

} // namespace

extern "C" {

/* Fills out[0..n) with N(0, sigma^2) samples of stream `stream`. */
void nut_synth_normal(uint64_t seed, uint64_t stream, float sigma, float *out,
                      size_t n) {
    const uint64_t key = splitmix64(seed ^ splitmix64(stream));
    split(n, [&](size_t b, size_t e) { normal_range(key, sigma, out, b, e); });
}

/* Token ids uniform in [lo, hi] (inclusive) of stream `stream`. */
void nut_synth_tokens(uint64_t seed, uint64_t stream, int lo, int hi, int *out,
                      size_t n) {
    const uint64_t key = splitmix64(seed ^ splitmix64(stream ^ 0x746f6b656eull));
    const uint64_t span = uint64_t(int64_t(hi) - int64_t(lo) + 1);
    for (size_t i = 0; i < n; i++)
        out[i] = int(int64_t(lo) + int64_t(splitmix64(key + i) % span));
}

} // extern "C"
