/* Seeded synthetic inputs for the optimizer-step workloads (host side, used by
 * the benchmark and the tests; not part of the optimizer itself).
 *
 * Normal(0, 1) samples: SplitMix64 over a counter (state_k = seed + k * gamma,
 * k = 1, 2, ...), two 53-bit uniforms per pair, Box-Muller in double
 * (r = sqrt(-2 ln u1), z0 = r cos(2 pi u2), z1 = r sin(2 pi u2)), scaled by
 * std and rounded to float once. Element 2i uses outputs 2i+1 and 2i+2.
 * Parallel over pairs with OpenMP; the result does not depend on the thread
 * count. */
#include <math.h>
#include <stddef.h>
#include <stdint.h>

#define SOAR_SYNTH_API __attribute__((visibility("default")))

static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static const uint64_t kGamma = 0x9E3779B97F4A7C15ull;

SOAR_SYNTH_API void soar_synth_splitmix64(uint64_t seed, uint64_t n, uint64_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = mix64(seed + (uint64_t)(i + 1) * kGamma);
}

SOAR_SYNTH_API void soar_synth_normal_f32(uint64_t seed, uint64_t n, double std, double mean,
                                          float* out) {
    const double inv53 = 1.0 / 9007199254740992.0;
    const double two_pi = 6.283185307179586476925286766559;
    const int64_t pairs = (int64_t)((n + 1) / 2);
#pragma omp parallel for schedule(static)
    for (int64_t p = 0; p < pairs; ++p) {
        const uint64_t a = mix64(seed + (uint64_t)(2 * p + 1) * kGamma);
        const uint64_t b = mix64(seed + (uint64_t)(2 * p + 2) * kGamma);
        const double u1 = ((double)(a >> 11) + 1.0) * inv53; /* (0, 1] */
        const double u2 = (double)(b >> 11) * inv53;         /* [0, 1) */
        const double r = sqrt(-2.0 * log(u1));
        const double th = two_pi * u2;
        out[2 * p] = (float)(r * cos(th) * std + mean);
        if ((uint64_t)(2 * p + 1) < n) out[2 * p + 1] = (float)(r * sin(th) * std + mean);
    }
}
