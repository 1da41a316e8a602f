/*
 * datagen.c -- seeded synthetic inputs for the tests and the benchmark.
 *
 * Counter-based, so any element can be produced independently (threads,
 * shards) and the stream is identical on every machine:
 *   z_i     = splitmix64_finalise(seed * 0xD1B54A32D192ED03 + (i + 1) * 0x9E3779B97F4A7C15)
 *   uniform = a + (b - a) * ((z_i >> 40) * 2^-24)          (binary64, rounded once)
 *   normal  = mean + std * sqrt(-2 ln u1) * cos(2 pi u2)   (Box-Muller in binary64,
 *             u1 = ((z_2i >> 11) + 1) * 2^-53, u2 = (z_2i+1 >> 11) * 2^-53)
 * The SplitMix64 finaliser constants are Steele, Lea and Flood's (OOPSLA 2014).
 */
#include <math.h>
#include <stdint.h>

#define EXPORT __attribute__((visibility("default")))

static inline uint64_t mix(uint64_t seed, uint64_t i) {
    uint64_t z = seed * 0xD1B54A32D192ED03ull + (i + 1) * 0x9E3779B97F4A7C15ull;
    z ^= z >> 30;
    z *= 0xBF58476D1CE4E5B9ull;
    z ^= z >> 27;
    z *= 0x94D049BB133111EBull;
    z ^= z >> 31;
    return z;
}

EXPORT uint64_t qsml_gen_bits(uint64_t seed, uint64_t i) { return mix(seed, i); }

/* out[j] = uniform element (offset + j), j < n */
EXPORT void qsml_gen_uniform_f32(uint64_t seed, int64_t offset, int64_t n, double a, double b, float* out) {
#pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < n; ++j) {
        uint64_t z = mix(seed, (uint64_t)(offset + j));
        double u = (double)(z >> 40) * 0x1.0p-24;
        out[j] = (float)(a + (b - a) * u);
    }
}

EXPORT void qsml_gen_normal_f32(uint64_t seed, int64_t offset, int64_t n, double mean, double stdv, float* out) {
    const double two_pi = 6.283185307179586476925286766559;
#pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < n; ++j) {
        uint64_t i = (uint64_t)(offset + j);
        uint64_t z1 = mix(seed, 2 * i), z2 = mix(seed, 2 * i + 1);
        double u1 = ((double)(z1 >> 11) + 1.0) * 0x1.0p-53;
        double u2 = (double)(z2 >> 11) * 0x1.0p-53;
        double g = sqrt(-2.0 * log(u1)) * cos(two_pi * u2);
        out[j] = (float)(mean + stdv * g);
    }
}

/* out[j] = (int32)(offset + j): X[i, j] = i * cols + j for a row-major X. */
EXPORT void qsml_gen_iota_i32(int64_t offset, int64_t n, int32_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < n; ++j) out[j] = (int32_t)(offset + j);
}
