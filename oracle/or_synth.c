/* or_synth.c — the seeded synthetic-checkpoint generator, restated for the CPU oracle.
 * TEST INFRASTRUCTURE: used by tests/ and by bench.py's reference arm so that the CPU
 * baseline builds its weights without mapping the CUDA library.
 *
 * The generator is this repository's own input generator (not reference code): element i
 * of stream `sid` under `seed` is a pure function of (seed, sid, i):
 *   key  = splitmix64(seed ^ splitmix64(sid))
 *   h(i) = splitmix64(key + i * 0xD1B54A32D192ED03)
 * SplitMix64 is the published finaliser (Steele, Lea, Flood 2014).  Normals use
 * Box-Muller on two 24-bit fields of h(i); bytes are the eight bytes of h(i >> 3).
 * Compiled without fp contraction and without vector ISA flags, so that every float
 * operation rounds exactly as the library's host generator does (same formula, same
 * libm): tests/test_oracle.py checks the two bit for bit. */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "dm_oracle.h"

static uint64_t sm64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static uint64_t key_of(uint64_t seed, uint64_t sid) { return sm64(seed ^ sm64(sid)); }
static uint64_t hash_at(uint64_t key, uint64_t i) { return sm64(key + i * 0xD1B54A32D192ED03ull); }

static float normal_of(uint64_t h) {
    const float u1 = (float)((h >> 40) + 1) * (1.0f / 16777216.0f);
    const float u2 = (float)((h >> 16) & 0xFFFFFFull) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cosf(6.28318530717958647692f * u2);
}

static uint32_t bits_of(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof u);
    return u;
}

static uint16_t to_bf16(float f) { /* round to nearest even; NaN stays NaN */
    const uint32_t u = bits_of(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}

static uint16_t to_f16(float f) { /* round to nearest even, subnormals included */
    uint32_t x = bits_of(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    x &= 0x7fffffffu;
    if (x >= 0x47800000u) return (uint16_t)(sign | (x > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (x < 0x38800000u) {
        if (x < 0x33000000u) return (uint16_t)sign;
        const uint32_t sh = 126u - (x >> 23);
        const uint32_t m = (x & 0x7fffffu) | 0x800000u;
        uint32_t q = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1u);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    const uint32_t r = x - 0x38000000u;
    return (uint16_t)(sign | ((r + 0xfffu + ((r >> 13) & 1u)) >> 13));
}

int or_synth_bf16(uint64_t seed, uint64_t sid, uint64_t n, float mean, float std, uint16_t* out) {
    if (!out) return 1;
    const uint64_t key = key_of(seed, sid);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = to_bf16(mean + std * normal_of(hash_at(key, (uint64_t)i)));
    return 0;
}

int or_synth_f32(uint64_t seed, uint64_t sid, uint64_t n, float mean, float std, float* out) {
    if (!out) return 1;
    const uint64_t key = key_of(seed, sid);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = mean + std * normal_of(hash_at(key, (uint64_t)i));
    return 0;
}

int or_synth_u8(uint64_t seed, uint64_t sid, uint64_t n, uint8_t* out) {
    if (!out) return 1;
    const uint64_t key = key_of(seed, sid);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i)
        out[i] = (uint8_t)(hash_at(key, (uint64_t)i >> 3) >> (8 * ((uint64_t)i & 7)));
    return 0;
}

int or_synth_f16_absnormal(uint64_t seed, uint64_t sid, uint64_t n, float std, uint16_t* out) {
    if (!out) return 1;
    const uint64_t key = key_of(seed, sid);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = to_f16(fabsf(std * normal_of(hash_at(key, (uint64_t)i))));
    return 0;
}
