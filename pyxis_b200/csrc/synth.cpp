// synth.cpp -- seeded synthetic tensors (see include/pyxis_synth.h).
#include "../../include/pyxis_synth.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

inline uint64_t mix64(uint64_t z) {  // splitmix64 output function
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

inline uint64_t stream_at(uint64_t seed, uint64_t k) { return mix64(seed + (k + 1) * kGolden); }

inline double normal_at(uint64_t seed, uint64_t i) {
    const double u1 = ((double)(stream_at(seed, 2 * i) >> 11) + 0.5) * (1.0 / 9007199254740992.0);
    const double u2 = (double)(stream_at(seed, 2 * i + 1) >> 11) * (1.0 / 9007199254740992.0);
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t b;
    std::memcpy(&b, &f, 4);
    if ((b & 0x7f800000u) == 0x7f800000u && (b & 0x7fffffu)) return (uint16_t)((b >> 16) | 0x40);
    b += 0x7fffu + ((b >> 16) & 1u);
    return (uint16_t)(b >> 16);
}

template <typename F>
void parallel_for(size_t n, F f) {
    unsigned nt = std::max(1u, std::thread::hardware_concurrency());
    if (n < (1u << 16)) nt = 1;
    nt = (unsigned)std::min<size_t>(nt, 64);
    if (nt == 1) {
        f(0, n);
        return;
    }
    std::vector<std::thread> th;
    size_t per = (n + nt - 1) / nt;
    for (unsigned t = 0; t < nt; ++t) {
        size_t b = t * per, e = std::min(n, b + per);
        if (b >= e) break;
        th.emplace_back([=] { f(b, e); });
    }
    for (auto &x : th) x.join();
}

}  // namespace

extern "C" void pyxis_synth_normal_f32(uint64_t seed, size_t n, float sigma, float *out) {
    parallel_for(n, [&](size_t b, size_t e) {
        for (size_t i = b; i < e; ++i) out[i] = (float)((double)sigma * normal_at(seed, i));
    });
}

extern "C" void pyxis_synth_normal_bf16(uint64_t seed, size_t n, float sigma, uint16_t *out) {
    parallel_for(n, [&](size_t b, size_t e) {
        for (size_t i = b; i < e; ++i)
            out[i] = f32_to_bf16_rne((float)((double)sigma * normal_at(seed, i)));
    });
}

extern "C" void pyxis_synth_tokens(uint64_t seed, size_t n, uint32_t vocab, int32_t *out) {
    for (size_t i = 0; i < n; ++i) out[i] = (int32_t)(stream_at(seed, i) % vocab);
}
