// dm_sha256.cu — SHA-256 (FIPS 180-4) for the session files' trailing checksum.
//
// Written from the standard: message padded with 0x80, zeros and the 64-bit big-endian bit
// length to a multiple of 64 bytes; each block expanded to 64 words and compressed with
// the eight working variables; the round constants are the first 32 bits of the
// fractional parts of the cube roots of the first 64 primes, the initial hash those of
// the square roots of the first 8 primes (both generated once at run time from the
// primes, not tabulated).
#include <cmath>
#include <cstdint>
#include <cstring>

#include "dismoen_cuda.h"
#include "dm_internal.h"

namespace {

struct Sha256Tables {
    uint32_t k[64];
    uint32_t h0[8];
    Sha256Tables() {
        int primes[64];
        int n = 0;
        for (int c = 2; n < 64; ++c) {
            bool p = true;
            for (int d = 2; d * d <= c; ++d)
                if (c % d == 0) {
                    p = false;
                    break;
                }
            if (p) primes[n++] = c;
        }
        // first 32 fractional bits of cbrt / sqrt, in long double with an integer fix-up
        for (int i = 0; i < 64; ++i) k[i] = frac_bits(primes[i], 3);
        for (int i = 0; i < 8; ++i) h0[i] = frac_bits(primes[i], 2);
    }
    // floor(frac(p^(1/r)) * 2^32), exact: integer root of p * 2^(32 r) by correction
    static uint32_t frac_bits(int p, int r) {
        const long double x = std::pow(static_cast<long double>(p), 1.0L / r);
        unsigned __int128 v = static_cast<unsigned __int128>(x * 4294967296.0L);
        auto pw = [r](unsigned __int128 a) {
            unsigned __int128 t = a;
            for (int i = 1; i < r; ++i) t *= a;
            return t;
        };
        unsigned __int128 target = static_cast<unsigned __int128>(p);
        for (int i = 0; i < r; ++i) target <<= 32;
        while (pw(v + 1) <= target) ++v;
        while (pw(v) > target) --v;
        return static_cast<uint32_t>(v & 0xFFFFFFFFu);
    }
};

const Sha256Tables& tables() {
    static const Sha256Tables t;
    return t;
}

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void compress(uint32_t h[8], const uint8_t* blk, const uint32_t* k) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
        w[i] = (uint32_t(blk[4 * i]) << 24) | (uint32_t(blk[4 * i + 1]) << 16) | (uint32_t(blk[4 * i + 2]) << 8) |
               uint32_t(blk[4 * i + 3]);
    for (int i = 16; i < 64; ++i) {
        const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
        const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
        w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
        const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
        const uint32_t ch = (e & f) ^ (~e & g);
        const uint32_t t1 = hh + S1 + ch + k[i] + w[i];
        const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
        const uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
        const uint32_t t2 = S0 + mj;
        hh = g;
        g = f;
        f = e;
        e = d + t1;
        d = c;
        c = b;
        b = a;
        a = t1 + t2;
    }
    h[0] += a;
    h[1] += b;
    h[2] += c;
    h[3] += d;
    h[4] += e;
    h[5] += f;
    h[6] += g;
    h[7] += hh;
}

}  // namespace

namespace dm {

// Incremental SHA-256 over several buffers (header, payload parts).
struct Sha256 {
    uint32_t h[8];
    uint8_t buf[64];
    size_t fill = 0;
    uint64_t total = 0;
    Sha256() { memcpy(h, tables().h0, sizeof h); }
    void update(const uint8_t* p, size_t n) {
        total += n;
        while (n) {
            const size_t take = (64 - fill) < n ? (64 - fill) : n;
            memcpy(buf + fill, p, take);
            fill += take;
            p += take;
            n -= take;
            if (fill == 64) {
                compress(h, buf, tables().k);
                fill = 0;
            }
        }
    }
    void finish(uint8_t out[32]) {
        const uint64_t bits = total * 8;
        const uint8_t one = 0x80, zero = 0;
        update(&one, 1);
        while (fill != 56) update(&zero, 1);
        uint8_t len[8];
        for (int i = 0; i < 8; ++i) len[i] = static_cast<uint8_t>(bits >> (56 - 8 * i));
        update(len, 8);
        for (int i = 0; i < 8; ++i)
            for (int j = 0; j < 4; ++j) out[4 * i + j] = static_cast<uint8_t>(h[i] >> (24 - 8 * j));
    }
};

void sha256_parts(const uint8_t* const* parts, const size_t* sizes, int n, uint8_t out[32]) {
    Sha256 s;
    for (int i = 0; i < n; ++i) s.update(parts[i], sizes[i]);
    s.finish(out);
}

}  // namespace dm

extern "C" int32_t dm_sha256(const uint8_t* data, uint64_t n, uint8_t* out32) {
    if ((!data && n) || !out32) return DM_ERR_INVALID_ARG;
    const uint8_t* parts[1] = {data};
    const size_t sizes[1] = {static_cast<size_t>(n)};
    dm::sha256_parts(parts, sizes, 1, out32);
    return DM_OK;
}
