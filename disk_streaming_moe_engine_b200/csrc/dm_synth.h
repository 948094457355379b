// dm_synth.h — counter-based synthetic checkpoint generator (host and device).
//
// Element i of stream `stream_id` under `seed` is a pure function of (seed, stream_id, i):
//   key  = splitmix64(seed ^ splitmix64(stream_id))
//   h(i) = splitmix64(key + i * 0xD1B54A32D192ED03)
// splitmix64 is the published SplitMix64 finaliser (Steele, Lea, Flood 2014; constants of
// Vigna's reference implementation).  Normals use Box-Muller on the two 24-bit halves of
// h(i): u1 = (h >> 40 + 1) / 2^24 in (0, 1], u2 = ((h >> 16) & 0xffffff) / 2^24,
// z = sqrt(-2 ln u1) cos(2 pi u2).  Host and device evaluate the same formula; they can
// differ in the last bits of logf/cosf, so tests generate on the host and upload.
//
// Stream ids of the synthetic model (benchmark / parity configs):
//   dense tensor (layer l or -1, tensor id t):   ((l + 1) << 8) | t
//   expert (layer l, expert e or -1, proj p, part q in {0 nibbles, 1 scales, 2 zeros}):
//        (1 << 40) | (l << 20) | ((e + 1) << 4) | (3 p + q)
// Distributions:
//   norm weights (input/post/final/gdn/q/k norms)   N(1, 0.02)
//   router rows                                      N(0, 1/sqrt(H))  (logits ~ N(0, 1))
//   every other dense weight, dt_bias, A_log         N(0, 0.02)
//   expert nibbles and zero points                   uniform 0..15 (uniform bytes)
//   expert scales                                    |N(0, 0.02)| as fp16
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define DM_SYN_FN __host__ __device__ __forceinline__
#else
#define DM_SYN_FN static inline
#endif
#include <math.h>

namespace dm {

DM_SYN_FN uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
DM_SYN_FN uint64_t synth_key(uint64_t seed, uint64_t stream_id) {
    return splitmix64(seed ^ splitmix64(stream_id));
}
DM_SYN_FN uint64_t synth_hash(uint64_t key, uint64_t i) {
    return splitmix64(key + i * 0xD1B54A32D192ED03ull);
}
DM_SYN_FN float synth_normal(uint64_t h) {
    const float u1 = static_cast<float>((h >> 40) + 1) * (1.0f / 16777216.0f);
    const float u2 = static_cast<float>((h >> 16) & 0xFFFFFFull) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cosf(6.28318530717958647692f * u2);
}
DM_SYN_FN uint8_t synth_byte(uint64_t key, uint64_t i) {
    return static_cast<uint8_t>(synth_hash(key, i >> 3) >> (8 * (i & 7)));
}

// fp32 -> bf16 / fp16 bit patterns, round to nearest even (host and device).
DM_SYN_FN uint32_t synth_bits(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    __builtin_memcpy(&u, &f, sizeof u);
    return u;
#endif
}
DM_SYN_FN uint16_t synth_f32_to_bf16(float f) {
    const uint32_t u = synth_bits(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);
    const uint32_t lsb = (u >> 16) & 1u;
    return static_cast<uint16_t>((u + 0x7fffu + lsb) >> 16);
}
DM_SYN_FN uint16_t synth_f32_to_f16(float f) {
    uint32_t x = synth_bits(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    x &= 0x7fffffffu;
    if (x >= 0x47800000u) return static_cast<uint16_t>(sign | (x > 0x7f800000u ? 0x7e00u : 0x7c00u));
    if (x < 0x38800000u) {  // below the smallest fp16 normal: subnormal or zero
        if (x < 0x33000000u) return static_cast<uint16_t>(sign);
        const uint32_t e = x >> 23;                 // biased fp32 exponent, <= 112
        const uint32_t m = (x & 0x7fffffu) | 0x800000u;
        const uint32_t sh = 126u - e;               // value / 2^-24 = m >> sh
        uint32_t q = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u);
        const uint32_t halfv = 1u << (sh - 1u);
        if (rem > halfv || (rem == halfv && (q & 1u))) ++q;
        return static_cast<uint16_t>(sign | q);
    }
    uint32_t r = x - 0x38000000u;                   // rebias exponent 127 -> 15
    const uint32_t lsb = (r >> 13) & 1u;
    r = (r + 0xfffu + lsb) >> 13;
    return static_cast<uint16_t>(sign | r);
}

DM_SYN_FN uint64_t synth_dense_stream(int layer, int tensor_id) {
    return (static_cast<uint64_t>(layer + 1) << 8) | static_cast<uint64_t>(tensor_id);
}
DM_SYN_FN uint64_t synth_expert_stream(int layer, int expert, int proj, int part) {
    return (1ull << 40) | (static_cast<uint64_t>(layer) << 20) |
           (static_cast<uint64_t>(expert + 1) << 4) | static_cast<uint64_t>(3 * proj + part);
}

}  // namespace dm
