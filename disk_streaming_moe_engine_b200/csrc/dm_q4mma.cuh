// dm_q4mma.cuh — 4-bit expert rows times activation vectors with integer mma.sync
// (u8 x s8 -> s32) on sm_100a: the chunk geometry of the expert records, the activation
// digits (two signed 8-bit digits per element with a unit per 64-element scale group) and
// the per-set product with the zero point and scale applied per group.  Shared by the
// fused single-row MoE kernel and the batched small-segment expert kernels.
//
// Reference format: asymmetric 4-bit, w = s * (q - z), fp16 scale s and 4-bit zero z per
// group of 64 along K, nibbles low first (quant_format.md:831-854).
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

#include "dm_common.cuh"

namespace dm {
// ---------------------------------------------------------------------------------------
// 4-bit chunk geometry: 16 rows of `K` columns, group G.
template <int K, int G>
struct Q4 {
    static constexpr int NV = K / 32;                 // 16-byte vectors per row
    static constexpr int LPR = NV < 32 ? NV : 32;     // lanes per row
    static constexpr int RPP = 32 / LPR;              // rows per warp pass
    static constexpr int VPL = NV / LPR;              // vectors per lane per row
    static constexpr int Q_BYTES = 16 * K / 2;
    static constexpr int S_OFF = Q_BYTES;
    static constexpr int S_BYTES = 16 * (K / G) * 2;
    static constexpr int Z_OFF = S_OFF + S_BYTES;
    static constexpr int Z_BYTES = 16 * (K / G) / 2;
    static constexpr int CHUNK = Z_OFF + Z_BYTES;
    static_assert(G % 32 == 0 && K % (2 * G) == 0, "group geometry");
};

// ---- 4-bit rows times a vector on the tensor cores: integer mma.sync m16n8k32 (u8 x s8,
// s32 accumulation, exact) ----
// A: a chunk's 16 rows as their raw nibbles q.  B: the vector v as two signed 8-bit digits
// per element with a scale per scale group g (the 64 columns that share a row's scale s
// and zero point z): S_g = max |v| over the group, u = v * 127 / S_g, d0 = rint(u),
// d1 = rint((u - d0) * 254), so v = unit_g (254 d0 + d1) with unit_g = S_g / (127 * 254),
// to within unit_g / 2 (1.6e-5 S_g).  Per group the integer sums C_i = sum q d_i are exact
// and the zero point enters exactly as C_i - z D_i (D_i = sum of the group's digits i):
//   row += s * unit_g * ((C_0 - z D_0) * 254 + (C_1 - z D_1))      (|.| < 2^25)
//
// Sets of four groups (256 columns, 128 bytes of a row) are eight MMAs into one
// accumulator.  Lane (r = lane / 4, t = lane % 4) supplies group t of the set: its 32
// bytes of rows r and r + 8, byte word m (columns 8m .. 8m + 7 of the group) to MMA m,
// low nibbles (even columns) at the lane's k positions 4t..4t+3, high nibbles (odd
// columns) at 4t+16..4t+19.  B column 2j + i carries digit i of group j at group j's k
// positions and zeros elsewhere, so after the set lane (r, t) holds C_0 and C_1 of group
// t for rows r and r + 8 and finishes that group itself.
//
// Rows are K/2 bytes apart (a multiple of 128): the same bytes of different rows share
// banks.  Lane (r, t) reads its two 16-byte units in the order (2t + (r & 1), the other),
// so each quarter-warp's 16-byte loads cover 8 different units (conflict-free), then
// swaps them back for odd rows.
//
// Vector fragments, per set S of four groups and MMA pair q = m / 2: 128 bytes, 16 for
// each (group t, digit i) at (2t + i) * 16, holding MMA 2q then 2q + 1: b0 = digit i of
// columns 8m + {0, 2, 4, 6}, b1 = of 8m + {1, 3, 5, 7}.  2 bytes per element.
constexpr int kQ4G = 64;  // the only group size these kernels take
// bytes of a K-element vector's fragments (whole sets of four groups)
__host__ __device__ constexpr int vfrag_bytes(int K) { return (K / kQ4G + 3) / 4 * 512; }
DM_DEV void mma_u8s8_16832(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                           uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Per-group vector data beside the fragments, kept per half (the 32 elements one warp
// holds) so that every slot has one writer and nothing needs an atomic.  A half's digit
// sums are at most 32 * 127 in magnitude: 16 bits each.  vgroup_build gives both halves
// the group's unit; vgroup_build_half gives each half its own.
struct alignas(16) VGroup {
    int16_t d0[2], d1[2];  // digit sums of each half
    float unit[2];         // S / (127 * 254) of each half
};
static_assert(sizeof(VGroup) == 16, "VGroup layout");

// Element k of a vector (whole warps: lane l holds k = 32w + l of a 32-aligned run, which
// lies in one scale group) given v = its value and vp = the value at k ^ 32, the other
// half of its group: the group max, its two digits into the fragments, and the half's
// digit sums and the group's unit into the group record (lane 0).  One pass, no barrier:
// both halves' warps compute the same maximum.  A zero group gives zero digits; a
// non-finite group max gives a non-finite unit, so non-finite inputs reach the outputs.
DM_DEV void vgroup_build(int8_t* vf, VGroup* vg, int k, float v, float vp) {
    const float S = __uint_as_float(
        __reduce_max_sync(0xffffffffu, max(__float_as_uint(fabsf(v)), __float_as_uint(fabsf(vp)))));
    const float inv = S > 0.0f && S <= 3.0e38f ? 127.0f / S : 0.0f;
    // round to nearest even through 1.5 * 2^23 (|u|, |e| <= 127.5): the sum's low bits are
    // the integer
    constexpr float kRound = 12582912.0f;
    const float u = v * inv;
    const float t0 = u + kRound;
    const int d0 = __float_as_int(t0) - 0x4B400000;
    const float t1 = (u - (t0 - kRound)) * 254.0f + kRound;
    const int d1 = __float_as_int(t1) - 0x4B400000;
    const int grp = k / kQ4G, col = k & (kQ4G - 1), m = col >> 3, p = col & 7;
    const int o = (((grp >> 2) * 4 + (m >> 1)) * 128) + ((grp & 3) * 2) * 16 + (m & 1) * 8 + (p & 1) * 4 + (p >> 1);
    vf[o] = static_cast<int8_t>(d0);
    vf[o + 16] = static_cast<int8_t>(d1);  // digit 1: the next 16 bytes
    // both sums in one reduction: |sum d0|, |sum d1| <= 32 * 127 < 2^15
    const int pk = __reduce_add_sync(0xffffffffu, d0 + d1 * 65536);
    if ((threadIdx.x & 31) == 0) {
        VGroup& g = vg[grp];
        const int h = (k >> 5) & 1;
        const int s0 = static_cast<int16_t>(pk & 0xFFFF);
        g.d0[h] = static_cast<int16_t>(s0);
        g.d1[h] = static_cast<int16_t>((pk - s0) >> 16);
        g.unit[h] = S * (1.0f / (127.0f * 254.0f));  // both halves: the group's unit
    }
}

// Set S (groups 4S .. 4S + ng - 1, ng <= 4) of a chunk's 16 rows (Q4 layout in shared
// memory) against the vector fragments: adds s * unit * T of group 4S + lane % 4 (if
// < ng) to rows lane / 4 (ya) and lane / 4 + 8 (yb).  The caller sums the four lanes of
// each row.
template <int K>
DM_DEV void q4_set_mma(const uint8_t* chunk, const uint4* vf, const VGroup* vg, int S, int ng, int lane, float& ya,
                       float& yb) {
    using Q = Q4<K, kQ4G>;
    constexpr int NG = K / kQ4G, RB = K / 2;
    const int r = lane >> 2, t = lane & 3;
    const bool have = t < ng;
    const int g = 4 * S + t;  // this lane's group
    // A: 32 bytes of rows r and r + 8 (units in row-parity order, then swapped back)
    uint4 a0 = make_uint4(0u, 0u, 0u, 0u), a1 = a0, b0 = a0, b1 = a0;
    if (have) {
        const int u0 = r & 1;
        const uint8_t* pa = chunk + r * RB + g * 32;
        const uint8_t* pb = chunk + (r + 8) * RB + g * 32;
        a0 = *reinterpret_cast<const uint4*>(pa + 16 * u0);
        a1 = *reinterpret_cast<const uint4*>(pa + 16 * (1 - u0));
        b0 = *reinterpret_cast<const uint4*>(pb + 16 * u0);
        b1 = *reinterpret_cast<const uint4*>(pb + 16 * (1 - u0));
        if (u0) {
            const uint4 x = a0; a0 = a1; a1 = x;
            const uint4 y = b0; b0 = b1; b1 = y;
        }
    }
    const uint32_t wa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const uint32_t wb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    // B: lanes (n, t) with n / 2 == t carry digit n % 2 of their group; the rest zeros
    const bool bl = (r >> 1) == t && have;
    int c[4] = {0, 0, 0, 0};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint4 v = bl ? vf[(S * 4 + q) * 8 + r] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int m = 2 * q + h;
            mma_u8s8_16832(c, wa[m] & 0x0F0F0F0Fu, wb[m] & 0x0F0F0F0Fu, (wa[m] >> 4) & 0x0F0F0F0Fu,
                           (wb[m] >> 4) & 0x0F0F0F0Fu, h ? v.z : v.x, h ? v.w : v.y);
        }
    }
    if (have) {
        const VGroup G = vg[g];
        const int D0 = G.d0[0] + G.d0[1], D1 = G.d1[0] + G.d1[1];
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(chunk + Q::S_OFF);
        const uint8_t* zp = chunk + Q::Z_OFF;
        const uint32_t zba = zp[r * (NG / 2) + (g >> 1)], zbb = zp[(r + 8) * (NG / 2) + (g >> 1)];
        const int za = static_cast<int>((g & 1) ? (zba >> 4) : (zba & 15u));
        const int zb = static_cast<int>((g & 1) ? (zbb >> 4) : (zbb & 15u));
        const float sa = __half2float(__ushort_as_half(sc[r * NG + g]));
        const float sb = __half2float(__ushort_as_half(sc[(r + 8) * NG + g]));
        const int ta = (c[0] - za * D0) * 254 + (c[1] - za * D1);
        const int tb = (c[2] - zb * D0) * 254 + (c[3] - zb * D1);
        ya = fmaf(sa * G.unit[0], static_cast<float>(ta), ya);
        yb = fmaf(sb * G.unit[0], static_cast<float>(tb), yb);
    }
}

// Element k of a vector whose digits take a unit per half group (the 32 elements one warp
// holds, k = 32w + lane): the half's max, its two digits into the fragments, its digit
// sums and unit into the group record (lane 0).  Same digits as vgroup_build with S the
// half's own max.
DM_DEV void vgroup_build_half(int8_t* vf, VGroup* vg, int k, float v) {
    const float S = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v))));
    const float inv = S > 0.0f && S <= 3.0e38f ? 127.0f / S : 0.0f;
    constexpr float kRound = 12582912.0f;
    const float u = v * inv;
    const float t0 = u + kRound;
    const int d0 = __float_as_int(t0) - 0x4B400000;
    const float t1 = (u - (t0 - kRound)) * 254.0f + kRound;
    const int d1 = __float_as_int(t1) - 0x4B400000;
    const int grp = k / kQ4G, col = k & (kQ4G - 1), m = col >> 3, p = col & 7;
    const int o = (((grp >> 2) * 4 + (m >> 1)) * 128) + ((grp & 3) * 2) * 16 + (m & 1) * 8 + (p & 1) * 4 + (p >> 1);
    vf[o] = static_cast<int8_t>(d0);
    vf[o + 16] = static_cast<int8_t>(d1);
    const int pk = __reduce_add_sync(0xffffffffu, d0 + d1 * 65536);
    if ((threadIdx.x & 31) == 0) {
        VGroup& g = vg[grp];
        const int h = (k >> 5) & 1;
        const int s0 = static_cast<int16_t>(pk & 0xFFFF);
        g.d0[h] = static_cast<int16_t>(s0);
        g.d1[h] = static_cast<int16_t>((pk - s0) >> 16);
        g.unit[h] = S * (1.0f / (127.0f * 254.0f));
    }
}

// One activation vector as the batched small-segment kernels keep it: its fragments
// (vfrag_bytes(K)), then its K / 64 scale-group records.
__host__ __device__ constexpr int vrec_bytes(int K) {
    return vfrag_bytes(K) + (K / kQ4G) * static_cast<int>(sizeof(VGroup));
}

// mma_u8s8_16832 without `volatile`: the compiler may interleave independent MMAs (other
// accumulators, other vectors) with each other and with the shared-memory loads.
DM_DEV void mma_u8s8_16832_nv(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                              uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Set S of a chunk's 16 rows against TT (1, 2 or 4) vectors (records of vrec_bytes(K)
// bytes at xr, xr + vrec_bytes(K), ...) whose digits take a unit per half group
// (vgroup_build_half): the rows' nibbles, scales and zeros are read once, then per vector
// the eight MMAs of q4_set_mma and the group epilogue
//   row += s * (unit_0 T_0 + unit_1 T_1),  T_h = (C_0h - z D_0h) * 254 + (C_1h - z D_1h),
// h the half of the group (columns 0-31, 32-63).  The MMA latency, not its throughput,
// bounds a set, so no MMA waits for another: one vector takes an accumulator per MMA (8),
// two vectors one per MMA pair (4 each), four vectors one per half (2 each); the integer
// partial sums are added at the end (exact).
template <int K, int TT>
DM_DEV void q4_set_mma_tok(const uint8_t* chunk, const uint8_t* xr, int S, int ng, int lane, float (&ya)[TT],
                           float (&yb)[TT]) {
    static_assert(TT == 1 || TT == 2 || TT == 4, "vectors per call");
    using Q = Q4<K, kQ4G>;
    constexpr int NG = K / kQ4G, RB = K / 2, VFB = vfrag_bytes(K), RBY = vrec_bytes(K);
    constexpr int NA = TT == 1 ? 8 : (TT == 2 ? 4 : 2);  // accumulators per vector
    const int r = lane >> 2, t = lane & 3;
    const bool have = t < ng;
    const int g = 4 * S + t;
    uint4 a0 = make_uint4(0u, 0u, 0u, 0u), a1 = a0, b0 = a0, b1 = a0;
    float sa = 0.0f, sb = 0.0f;
    int za = 0, zb = 0;
    if (have) {
        const int u0 = r & 1;
        const uint8_t* pa = chunk + r * RB + g * 32;
        const uint8_t* pb = chunk + (r + 8) * RB + g * 32;
        a0 = *reinterpret_cast<const uint4*>(pa + 16 * u0);
        a1 = *reinterpret_cast<const uint4*>(pa + 16 * (1 - u0));
        b0 = *reinterpret_cast<const uint4*>(pb + 16 * u0);
        b1 = *reinterpret_cast<const uint4*>(pb + 16 * (1 - u0));
        if (u0) {
            const uint4 x = a0; a0 = a1; a1 = x;
            const uint4 y = b0; b0 = b1; b1 = y;
        }
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(chunk + Q::S_OFF);
        const uint8_t* zp = chunk + Q::Z_OFF;
        const uint32_t zba = zp[r * (NG / 2) + (g >> 1)], zbb = zp[(r + 8) * (NG / 2) + (g >> 1)];
        za = static_cast<int>((g & 1) ? (zba >> 4) : (zba & 15u));
        zb = static_cast<int>((g & 1) ? (zbb >> 4) : (zbb & 15u));
        sa = __half2float(__ushort_as_half(sc[r * NG + g]));
        sb = __half2float(__ushort_as_half(sc[(r + 8) * NG + g]));
    }
    const uint32_t wa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const uint32_t wb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    const bool bl = (r >> 1) == t && have;
    int acc[TT][NA][4];
#pragma unroll
    for (int j = 0; j < TT; ++j)
#pragma unroll
        for (int i = 0; i < NA; ++i) acc[j][i][0] = acc[j][i][1] = acc[j][i][2] = acc[j][i][3] = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint4 v[TT];
#pragma unroll
        for (int j = 0; j < TT; ++j)
            v[j] = bl ? reinterpret_cast<const uint4*>(xr + j * RBY)[(S * 4 + q) * 8 + r] : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int m = 2 * q + h;
            const uint32_t al = wa[m] & 0x0F0F0F0Fu, bl2 = wb[m] & 0x0F0F0F0Fu;
            const uint32_t ah = (wa[m] >> 4) & 0x0F0F0F0Fu, bh = (wb[m] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
            for (int j = 0; j < TT; ++j)
                mma_u8s8_16832_nv(acc[j][TT == 1 ? m : (TT == 2 ? q : q >> 1)], al, bl2, ah, bh, h ? v[j].z : v[j].x,
                                  h ? v[j].w : v[j].y);
        }
    }
    if (have) {
#pragma unroll
        for (int j = 0; j < TT; ++j) {
            int c[4], e[4];  // halves 0 (MMA pairs 0, 1) and 1 (pairs 2, 3)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                c[i] = acc[j][0][i];
                e[i] = acc[j][NA / 2][i];
#pragma unroll
                for (int u = 1; u < NA / 2; ++u) {
                    c[i] += acc[j][u][i];
                    e[i] += acc[j][NA / 2 + u][i];
                }
            }
            const VGroup G = reinterpret_cast<const VGroup*>(xr + j * RBY + VFB)[g];
            // per half C_i - z D_i = sum (q - z) d_i: at most 32 * 15 * 127, so |T| < 2^24 (exact in fp32)
            const int ta0 = (c[0] - za * G.d0[0]) * 254 + (c[1] - za * G.d1[0]);
            const int ta1 = (e[0] - za * G.d0[1]) * 254 + (e[1] - za * G.d1[1]);
            const int tb0 = (c[2] - zb * G.d0[0]) * 254 + (c[3] - zb * G.d1[0]);
            const int tb1 = (e[2] - zb * G.d0[1]) * 254 + (e[3] - zb * G.d1[1]);
            ya[j] = fmaf(sa, fmaf(G.unit[0], static_cast<float>(ta0), G.unit[1] * static_cast<float>(ta1)), ya[j]);
            yb[j] = fmaf(sb, fmaf(G.unit[0], static_cast<float>(tb0), G.unit[1] * static_cast<float>(tb1)), yb[j]);
        }
    }
}

}  // namespace dm
