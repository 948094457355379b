/*
 * or_formats.c — CPU restatement of the reference's on-disk weight formats
 * (TEST INFRASTRUCTURE: the checker of libdismoen_cuda.so's loaders, never the product).
 *
 *   GGUF block dequantisation   reference src/format/gguf.mojo:414-561 and
 *                               tools/oracle/oracle_port.py:68-159 (Q8_0, Q4_K, Q3_K;
 *                               F32 / F16 / BF16 as oracle_port.py:185-203 converts them)
 *   custom 4-bit -> pool        the exact conversion of the loader (nibble n -> n XOR 8,
 *                               zero 8, the group's scale)
 *   re-quantisation -> pool     the loader's round-to-nearest rule (stated in
 *                               include/dismoen_cuda.h and the loader source)
 *
 * Compiled with -ffp-contract=off: every product and difference rounds on its own, as in
 * the reference's fp32 loops and in the CUDA kernels (__fmul_rn / __fsub_rn).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "dm_oracle.h"

float or_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const int exp = (h >> 10) & 0x1F;
    const uint32_t man = h & 0x3FFu;
    float f;
    if (exp == 0) {
        f = ldexpf((float)man, -24); /* zero and subnormals: man * 2^-24, exact */
        uint32_t u;
        memcpy(&u, &f, 4);
        u |= sign;
        memcpy(&f, &u, 4);
        return f;
    }
    uint32_t u;
    if (exp == 31)
        u = sign | 0x7F800000u | (man << 13);
    else
        u = sign | ((uint32_t)(exp - 15 + 127) << 23) | (man << 13);
    memcpy(&f, &u, 4);
    return f;
}

/* fp32 -> fp16, round to nearest even (IEEE 754 convertFormat). */
uint16_t or_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    x &= 0x7FFFFFFFu;
    if (x >= 0x7F800000u) return sign | (x > 0x7F800000u ? 0x7E00u : 0x7C00u);
    if (x >= 0x477FF000u) return sign | 0x7C00u; /* >= 65520 rounds to infinity */
    if (x < 0x38800000u) {                      /* below 2^-14: a subnormal result */
        float ax;
        memcpy(&ax, &x, 4);
        const double m = nearbyint((double)ax * 16777216.0); /* exact product; RNE */
        return sign | (uint16_t)m;
    }
    uint32_t h = ((x >> 23) - 127 + 15) << 10 | ((x & 0x7FFFFFu) >> 13);
    const uint32_t rem = x & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
    return sign | (uint16_t)h;
}

static float f16_at(const uint8_t* p) { return or_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

/* Element e of one block (see the per-type references above). */
static float gguf_elem(int type, const uint8_t* blk, int e, unsigned flags) {
    switch (type) {
        case 0: { /* F32 */
            float v;
            memcpy(&v, blk, 4);
            return v;
        }
        case 1: return f16_at(blk); /* F16 */
        case 30: {                  /* BF16: the high half of an fp32 */
            const uint32_t u = (uint32_t)(blk[0] | (blk[1] << 8)) << 16;
            float v;
            memcpy(&v, &u, 4);
            return v;
        }
        case 8: /* Q8_0, gguf.mojo:414-441 / oracle_port.py:68-83: scale * int8 */
            return f16_at(blk) * (float)(int8_t)blk[2 + e];
        case 12: { /* Q4_K, gguf.mojo:444-506 / oracle_port.py:86-127 */
            const float d = f16_at(blk), dmin = f16_at(blk + 2);
            const uint8_t* sc = blk + 4;
            const int j = e / 32, i = e % 32;
            int s6, m6;
            if (j < 4) {
                s6 = sc[j] & 63;
                m6 = sc[j + 4] & 63;
            } else if (flags & 1u) { /* gguf.mojo:478-485 */
                const int b4 = sc[j - 4], b8 = sc[j];
                s6 = (b8 & 0xF) | ((b4 >> 6) << 4);
                m6 = (b8 >> 4) | ((b8 >> 6) << 4);
            } else { /* oracle_port.py:108-112, the GGUF layout */
                s6 = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
                m6 = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
            }
            const float scv = (float)s6 * d;
            const float mv = (float)m6 * dmin;
            const uint8_t b = blk[16 + j * 16 + (i % 16)];
            const int q = i < 16 ? (b & 0xF) : (b >> 4);
            return scv * (float)q - mv;
        }
        case 11: { /* Q3_K, gguf.mojo:509-560 / oracle_port.py:130-159 */
            const float d = f16_at(blk + 112);
            const float scv = (float)((int)blk[96 + e / 16] - 32) * d;
            const int h = (blk[e / 8] >> (e % 8)) & 1;
            const int lo = (blk[32 + e / 4] >> (2 * (e % 4))) & 3;
            return scv * (float)(((h << 2) | lo) - 4);
        }
        default: return 0.0f;
    }
}

int or_gguf_dequant(int type, const uint8_t* raw, long long n, unsigned flags, float* out) {
    int bs, bpb;
    switch (type) {
        case 0: bs = 1; bpb = 4; break;
        case 1: case 30: bs = 1; bpb = 2; break;
        case 8: bs = 32; bpb = 34; break;
        case 11: bs = 256; bpb = 114; break;
        case 12: bs = 256; bpb = 144; break;
        default: return -1;
    }
    if (n % bs) return -2;
    for (long long e = 0; e < n; ++e) out[e] = gguf_elem(type, raw + (e / bs) * bpb, (int)(e % bs), flags);
    return 0;
}

/* The custom signed 4-bit format -> the pool's asymmetric form.  Returns the flags of the
 * CUDA conversion: 1 reserved nibble, 2 invalid scale, 4 different scales inside one pool
 * group. */
unsigned or_sym4_to_pool(const uint8_t* packed, const uint16_t* scales, long long e0, int rows, int cols, int gf,
                         int gp, uint8_t* q, uint16_t* s, uint8_t* z) {
    unsigned f = 0;
    const int ngp = cols / gp;
    for (int r = 0; r < rows; ++r)
        for (int g = 0; g < ngp; ++g) {
            const long long base = e0 + (long long)r * cols + (long long)g * gp;
            for (int k = 0; k < gp / 2; ++k) {
                const uint8_t b = packed[base / 2 + k];
                if ((b & 0xF) == 8 || (b >> 4) == 8) f |= 1u;
                q[(size_t)r * (cols / 2) + g * (gp / 2) + k] = b ^ 0x88;
            }
            const uint16_t s0 = scales[base / gf];
            for (long long e = base; e < base + gp; e += gf) {
                const uint16_t u = scales[e / gf];
                if (((u >> 10) & 0x1F) == 0x1F || (u & 0x8000u) || (u & 0x7FFFu) == 0) f |= 2u;
                if (u != s0) f |= 4u;
            }
            s[(size_t)r * ngp + g] = s0;
            if ((g & 1) == 0) z[(size_t)r * (ngp / 2) + g / 2] = 0x88;
        }
    return f;
}

/* Round-to-nearest re-quantisation into the pool's form (groups of gp along each row):
 * lo = min(0, min w), hi = max(0, max w); s = fp16(RN((hi - lo) / 15)) saturated to
 * [2^-24, 65504] (1 when hi == lo); z = clamp(rint(-lo / s), 0, 15);
 * q = clamp(rint(w / s) + z, 0, 15).  Returns 8 when a weight is not finite; *max_err the
 * largest |w - s (q - z)|. */
unsigned or_requant_pool(const float* w, int rows, int cols, int gp, uint8_t* q, uint16_t* s, uint8_t* z,
                         float* max_err) {
    unsigned f = 0;
    float err = 0.0f;
    const int ng = cols / gp;
    for (int r = 0; r < rows; ++r)
        for (int g = 0; g < ng; ++g) {
            const float* src = w + (size_t)r * cols + (size_t)g * gp;
            float lo = 0.0f, hi = 0.0f;
            for (int k = 0; k < gp; ++k) {
                if (!isfinite(src[k])) f |= 8u;
                lo = fminf(lo, src[k]);
                hi = fmaxf(hi, src[k]);
            }
            const float s32 = (hi - lo) / 15.0f;
            uint16_t s16;
            if (s32 == 0.0f || !isfinite(s32)) {
                s16 = isfinite(s32) ? 0x3C00 : 0x7BFF;
            } else {
                s16 = or_f32_to_f16(s32);
                if ((s16 & 0x7FFF) == 0x7C00) s16 = 0x7BFF;
                if (s16 == 0) s16 = 0x0001;
            }
            const float sf = or_f16_to_f32(s16);
            const float zf = fminf(fmaxf(rintf(-lo / sf), 0.0f), 15.0f);
            const int zi = (int)zf;
            for (int k = 0; k < gp; ++k) {
                const float v = src[k];
                const float qf = fminf(fmaxf(rintf(v / sf) + zf, 0.0f), 15.0f);
                const int qi = isfinite(v) ? (int)qf : zi;
                if (isfinite(v)) {
                    const float d = fabsf(v - sf * (float)(qi - zi));
                    if (d > err) err = d;
                }
                uint8_t* dst = q + (size_t)r * (cols / 2) + ((size_t)g * gp + k) / 2;
                if (k & 1)
                    *dst = (uint8_t)((*dst & 0x0F) | (qi << 4));
                else
                    *dst = (uint8_t)qi;
            }
            s[(size_t)r * ng + g] = s16;
            uint8_t* zd = z + (size_t)r * (ng / 2) + g / 2;
            if (g & 1)
                *zd = (uint8_t)((*zd & 0x0F) | (zi << 4));
            else
                *zd = (uint8_t)zi;
        }
    if (max_err) *max_err = err;
    return f;
}
