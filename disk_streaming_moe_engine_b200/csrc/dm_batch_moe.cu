// dm_batch_moe.cu — routed + shared experts of the batched decode step on the tensor
// cores (sm_100a, mma.sync m16n8k16 bf16 -> fp32), dequantising the asymmetric 4-bit
// format in registers.
//
// Work: the (expert, row) pairs of a layer are grouped by expert into segments of at
// most kSegTok rows (one n8 tile).  An item is a segment and 16 consecutive 16-row chunks
// of the projection; the CTA (16 warps, one chunk each) stages the segment's activations
// in shared memory and every warp streams its chunk: A = the 16 weight rows, B = the
// activation rows, so the weights are read once per segment straight from HBM with
// 8 groups of loads in flight per thread.
//
// Exact dequantisation.  Within a group of 64 columns every weight is s * (q - z) with one
// fp16 scale s and one 4-bit zero z (reference quant_format.md:831-854, low nibble first).
// A nibble q is turned into the bf16 number 128 + q by OR-ing it into the bits of 128.0
// (bf16 has 7 mantissa bits, so 128..255 are exact); subtracting 128 + z in packed bf16
// gives q - z exactly.  The tensor cores therefore multiply exact integers by the
// activation, split as x = hi + lo (two bf16 terms, |x - hi - lo| <= 2^-16 |x|), and the
// group's partial sum is scaled by s in fp32.  The columns a lane supplies to one MMA
// are a permutation of the group's columns (8 nibbles of one 32-bit word feed two MMAs);
// the activations are staged in the same permuted order, which leaves every dot product
// unchanged.
//
// gate/up (K = H): chunk c holds gate rows 8c..8c+7 then up rows 8c..8c+7, so the lane
//   holding C[g][*] also holds the matching up row C[g+8][*]: h = SiLU(gate) * up
//   (reference swiglu.mojo:52) is formed in registers and stored per pair.
// down (K = I): chunk c holds output rows 16c..16c+15 -> part[pair][row].
#include <cuda.h>
#include <cuda_fp16.h>

#include "dm_common.cuh"
#include "dm_kernels.h"

namespace dm {

constexpr int kXThreads = 512;
constexpr int kXWarps = kXThreads / 32;

struct BExpArgs {
    const uint8_t* experts;   // [E] records
    const uint8_t* shared;    // shared-expert record
    int64_t expert_bytes;
    int64_t proj_off;         // offset of this projection inside a record
    int64_t chunk_bytes;
    int E, n_chunks;
    const int4* segs;         // (expert, first pair, rows, 0)
    int* work;                // [0] segments; [slot] work counter of this launch
    int work_slot;
    const int* pair_src;      // (source rank * n + row) * 32 + k of each pair
    int n, topk;
    EpView ep;                // gate/up reads ep.xn[source rank]; down writes ep.eout[source rank]
    const float* h_in;        // down: h [pairs][K]
    float* h_out;             // gate/up: h [pairs][I]
    int H;
    // tensor-map kernel: the projection's nibble rows of the layer's whole expert pool as a
    // 4-D byte tensor (row bytes, 16 rows, chunk, expert; the shared expert is expert E)
    CUtensorMap wmap;
    uint32_t* err;
};


// (q_j, q_{j+4}) of a word of 8 nibbles as bf16 (128 + q) pairs, minus the zero pair.
DM_DEV uint32_t nib_pair_minus(uint32_t w, int shift, uint32_t zpair) {
    const uint32_t p = ((w >> shift) & 0x000F000Fu) | 0x43004300u;
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(p), "r"(zpair));
    return d;
}

DM_DEV uint2 ldg_nc_v2(const void* p) {
    uint2 r;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
    return r;
}
DM_DEV uint32_t ldg_nc_u16(const void* p) {
    unsigned short r;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}
DM_DEV uint4 lds128(const void* p) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(smem_u32(p)));
    return r;
}

// Staged order of a 16-column run: [0,4,1,5,2,6,3,7, 8,12,9,13,10,14,11,15], so that
// 32-bit word m holds the columns (j, j + 4) that MMA m/2 takes from lane ft (see above).
template <int K>
struct XGeom {
    static constexpr int NG = K / 64;                  // groups of a row
    static constexpr int PD = NG < 8 ? NG : 8;         // groups of loads in flight
    static constexpr int ROWB = K * 2 + 16;            // bytes of a staged activation row
    static constexpr int S_OFF = 16 * K / 2;           // scales [16][NG] fp16
    static constexpr int Z_OFF = S_OFF + 16 * NG * 2;  // zeros [16][NG/2] bytes
    static constexpr int ZB = NG / 2;                  // zero bytes per row
    static constexpr int ZW = (ZB + 3) / 4;            // ... as 32-bit words
    static constexpr size_t SMEM = 2 * kSegTok * ROWB;
    static_assert(K % 128 == 0, "whole zero bytes per row");
};

template <int K>
DM_DEV void load_zero_words(const uint8_t* zrow, uint32_t (&zw)[XGeom<K>::ZW]) {
    using XG = XGeom<K>;
    if (XG::ZB >= 4) {
#pragma unroll
        for (int i = 0; i < XG::ZW; ++i) zw[i] = __ldg(reinterpret_cast<const uint32_t*>(zrow) + i);
    } else {
        uint32_t v = 0;
#pragma unroll
        for (int i = 0; i < XG::ZB; ++i) v |= static_cast<uint32_t>(__ldg(zrow + i)) << (8 * i);
        zw[0] = v;
    }
}

template <int K, bool GATEUP>
__global__ void __launch_bounds__(kXThreads, 1) b_expert_kernel(const __grid_constant__ BExpArgs a) {
    using XG = XGeom<K>;
    extern __shared__ __align__(16) uint8_t xsm[];  // hi rows [kSegTok][ROWB], then lo rows
    __shared__ int s_item;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int fg = lane >> 2, ft = lane & 3;
    const int ips = (a.n_chunks + kXWarps - 1) / kXWarps;  // items per segment
    pdl_wait();
    const int nitems = a.work[0] * ips;
    pdl_launch_dependents();
    uint8_t* xhi = xsm;
    uint8_t* xlo = xsm + kSegTok * XG::ROWB;

    while (true) {
        if (tid == 0) s_item = atomicAdd(a.work + a.work_slot, 1);
        __syncthreads();
        const int item = s_item;
        if (item >= nitems) break;
        const int4 sg = a.segs[item / ips];
        const int part = item % ips;
        const int ex = sg.x, pair0 = sg.y, ntok = sg.z;

        // ---- stage the segment's activation rows: 16 columns per task ----
        for (int t = tid; t < kSegTok * (K / 16); t += kXThreads) {
            const int r = t / (K / 16), c16 = t % (K / 16);
            float v[16];
            if (r < ntok) {
                const float* row;
                if (GATEUP) {  // the normalised row of its source rank (peer memory in a group)
                    const int src = a.pair_src[pair0 + r] >> 5;
                    row = a.ep.xn[src / a.n] + static_cast<size_t>(src % a.n) * K;
                } else {
                    row = a.h_in + static_cast<size_t>(pair0 + r) * K;
                }
                const float4* src = reinterpret_cast<const float4*>(row + 16 * c16);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 f = src[i];
                    v[4 * i] = f.x;
                    v[4 * i + 1] = f.y;
                    v[4 * i + 2] = f.z;
                    v[4 * i + 3] = f.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = 0.0f;
            }
            // word m of the staged run = (x[j], x[j + 4]), j = (m & 3) + 8 (m >> 2)
            uint32_t hw[8], lw[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const int j = (m & 3) + 8 * (m >> 2);
                const uint16_t h0 = f32_to_bf16(v[j]), h1 = f32_to_bf16(v[j + 4]);
                const uint16_t l0 = f32_to_bf16(v[j] - bf16_to_f32(h0)), l1 = f32_to_bf16(v[j + 4] - bf16_to_f32(h1));
                hw[m] = static_cast<uint32_t>(h0) | (static_cast<uint32_t>(h1) << 16);
                lw[m] = static_cast<uint32_t>(l0) | (static_cast<uint32_t>(l1) << 16);
            }
            uint4* dh = reinterpret_cast<uint4*>(xhi + r * XG::ROWB + 32 * c16);
            uint4* dl = reinterpret_cast<uint4*>(xlo + r * XG::ROWB + 32 * c16);
            dh[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            dh[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
            dl[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            dl[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
        }
        __syncthreads();

        const int c = part * kXWarps + warp;
        if (c < a.n_chunks) {
            const uint8_t* rec = ex < a.E ? a.experts + static_cast<int64_t>(ex) * a.expert_bytes : a.shared;
            const uint8_t* ch = rec + a.proj_off + static_cast<int64_t>(c) * a.chunk_bytes;
            const uint8_t* q0 = ch + fg * (K / 2) + 8 * ft;
            const uint8_t* q1 = ch + (fg + 8) * (K / 2) + 8 * ft;
            const uint16_t* s0 = reinterpret_cast<const uint16_t*>(ch + XG::S_OFF) + fg * XG::NG;
            const uint16_t* s1 = reinterpret_cast<const uint16_t*>(ch + XG::S_OFF) + (fg + 8) * XG::NG;
            uint2 qa[XG::PD], qb[XG::PD];
            uint32_t sa[XG::PD], sb[XG::PD];
#pragma unroll
            for (int i = 0; i < XG::PD; ++i) {
                qa[i] = ldg_nc_v2(q0 + 32 * i);
                qb[i] = ldg_nc_v2(q1 + 32 * i);
                sa[i] = ldg_nc_u16(s0 + i);
                sb[i] = ldg_nc_u16(s1 + i);
            }
            uint32_t za[XG::ZW], zb[XG::ZW];
            load_zero_words<K>(ch + XG::Z_OFF + fg * XG::ZB, za);
            load_zero_words<K>(ch + XG::Z_OFF + (fg + 8) * XG::ZB, zb);
            const uint8_t* bh = xhi + fg * XG::ROWB + 32 * ft;
            const uint8_t* bl = xlo + fg * XG::ROWB + 32 * ft;
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int g0 = 0; g0 < XG::NG; g0 += XG::PD) {
#pragma unroll
                for (int u = 0; u < XG::PD; ++u) {
                    const int g = g0 + u;
                    const uint2 wa = qa[u], wb = qb[u];
                    const float sca = __half2float(__ushort_as_half(static_cast<unsigned short>(sa[u])));
                    const float scb = __half2float(__ushort_as_half(static_cast<unsigned short>(sb[u])));
                    if (g + XG::PD < XG::NG) {
                        qa[u] = ldg_nc_v2(q0 + 32 * (g + XG::PD));
                        qb[u] = ldg_nc_v2(q1 + 32 * (g + XG::PD));
                        sa[u] = ldg_nc_u16(s0 + g + XG::PD);
                        sb[u] = ldg_nc_u16(s1 + g + XG::PD);
                    }
                    const uint32_t zqa = (za[g >> 3] >> (4 * (g & 7))) & 15u;
                    const uint32_t zqb = (zb[g >> 3] >> (4 * (g & 7))) & 15u;
                    const uint32_t zpa = 0x43004300u | zqa | (zqa << 16);
                    const uint32_t zpb = 0x43004300u | zqb | (zqb << 16);
                    const uint4 h0 = lds128(bh + 128 * g), h1 = lds128(bh + 128 * g + 16);
                    const uint4 l0 = lds128(bl + 128 * g), l1 = lds128(bl + 128 * g + 16);
                    float ch_[4] = {0.0f, 0.0f, 0.0f, 0.0f}, cl_[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    // MMA 0..3: word x (shifts 0/4, 8/12) then word y
                    {
                        const uint32_t a0 = nib_pair_minus(wa.x, 0, zpa), a1 = nib_pair_minus(wb.x, 0, zpb);
                        const uint32_t a2 = nib_pair_minus(wa.x, 4, zpa), a3 = nib_pair_minus(wb.x, 4, zpb);
                        mma_bf16_m16n8k16(ch_, a0, a1, a2, a3, h0.x, h0.y);
                        mma_bf16_m16n8k16(cl_, a0, a1, a2, a3, l0.x, l0.y);
                    }
                    {
                        const uint32_t a0 = nib_pair_minus(wa.x, 8, zpa), a1 = nib_pair_minus(wb.x, 8, zpb);
                        const uint32_t a2 = nib_pair_minus(wa.x, 12, zpa), a3 = nib_pair_minus(wb.x, 12, zpb);
                        mma_bf16_m16n8k16(ch_, a0, a1, a2, a3, h0.z, h0.w);
                        mma_bf16_m16n8k16(cl_, a0, a1, a2, a3, l0.z, l0.w);
                    }
                    {
                        const uint32_t a0 = nib_pair_minus(wa.y, 0, zpa), a1 = nib_pair_minus(wb.y, 0, zpb);
                        const uint32_t a2 = nib_pair_minus(wa.y, 4, zpa), a3 = nib_pair_minus(wb.y, 4, zpb);
                        mma_bf16_m16n8k16(ch_, a0, a1, a2, a3, h1.x, h1.y);
                        mma_bf16_m16n8k16(cl_, a0, a1, a2, a3, l1.x, l1.y);
                    }
                    {
                        const uint32_t a0 = nib_pair_minus(wa.y, 8, zpa), a1 = nib_pair_minus(wb.y, 8, zpb);
                        const uint32_t a2 = nib_pair_minus(wa.y, 12, zpa), a3 = nib_pair_minus(wb.y, 12, zpb);
                        mma_bf16_m16n8k16(ch_, a0, a1, a2, a3, h1.z, h1.w);
                        mma_bf16_m16n8k16(cl_, a0, a1, a2, a3, l1.z, l1.w);
                    }
                    acc[0] = fmaf(sca, ch_[0] + cl_[0], acc[0]);
                    acc[1] = fmaf(sca, ch_[1] + cl_[1], acc[1]);
                    acc[2] = fmaf(scb, ch_[2] + cl_[2], acc[2]);
                    acc[3] = fmaf(scb, ch_[3] + cl_[3], acc[3]);
                }
            }
            // C rows fg / fg + 8, columns (rows of the segment) 2 ft, 2 ft + 1
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int t = 2 * ft + e;
                if (t < ntok) {
                    if (GATEUP) {
                        // h row length I = 8 rows per gate/up chunk
                        a.h_out[static_cast<size_t>(pair0 + t) * (a.n_chunks * 8) + 8 * c + fg] =
                            silu_f(acc[e]) * acc[2 + e];
                    } else {  // into the source rank's expert-output row (peer memory in a group)
                        const int ps = a.pair_src[pair0 + t];
                        const int src = ps >> 5, k = ps & 31;
                        float* dst = a.ep.eout[src / a.n] + (static_cast<size_t>(src % a.n) * (a.topk + 1) + k) * a.H;
                        dst[16 * c + fg] = acc[e];
                        dst[16 * c + fg + 8] = acc[2 + e];
                    }
                }
            }
        }
        __syncthreads();  // staged rows free; s_item read by every thread
    }
    if (!GATEUP && a.ep.world > 1) __threadfence_system();  // results stored into peers
}

// ---------------------------------------------------------------------------------------
// Tensor-map variant (K <= 2048).  Same items, tiles and MMA fragments as b_expert_kernel;
// the weights move differently:
//   * every warp streams its chunk's nibble rows in K-blocks of 4 groups (16 rows x 128
//     bytes, one 2-D box of the pool's tensor map, 128-byte swizzle) through its own
//     kVStages-deep ring, and the chunk's scales and zeros (contiguous) with one bulk copy;
//     lane 0 issues, every lane waits on the stage's mbarrier.  Copies of an item are
//     issued before its activation rows are staged.
//   * the zero point leaves the inner loop: A = 128 + q (exact in bf16), and per group
//     sum_k (q - z) x = sum_k (128 + q) x - (128 + z) sum_k x, with sum_k x of the staged
//     hi + lo terms (16-column partial sums added in a fixed order).
constexpr int kVStages = 3;        // K-blocks in flight per warp
constexpr int kVBox = 16 * 128;    // bytes of one K-block box

template <int K>
struct VGeom {
    using XG = XGeom<K>;
    static constexpr int NKB = K / 256;                       // K-blocks (4 groups) of a chunk
    static constexpr int SZ = XG::Z_OFF - XG::S_OFF + 16 * XG::ZB;  // scales + zeros bytes
    static constexpr int SZP = (SZ + 127) / 128 * 128;
    static constexpr int RING = kVStages * kVBox;             // one warp's ring (1024-aligned)
    static constexpr int XS_LD = K / 16 + 4;                  // padded row of the partial sums
    static constexpr size_t ACT = 2 * kSegTok * XG::ROWB;
    static constexpr size_t XSUM = static_cast<size_t>(kSegTok) * XS_LD * 4;  // 16-column partials
    static constexpr size_t SMEM = 1024 + static_cast<size_t>(kXWarps) * (RING + SZP) + ACT + XSUM;
    static_assert(SMEM <= 227 * 1024, "shared memory of the expert kernel");
    static_assert(K % 256 == 0, "whole K-blocks");
};

DM_DEV void tma_load_4d(void* smem_dst, const CUtensorMap* map, int x, int y, int z, int w, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
        : "memory");
}


template <int K, bool GATEUP>
__global__ void __launch_bounds__(kXThreads, 1) b_expert_tma_kernel(const __grid_constant__ BExpArgs a) {
    using XG = XGeom<K>;
    using VG = VGeom<K>;
    extern __shared__ __align__(1024) uint8_t vsm_raw[];
    uint8_t* vsm = vsm_raw + ((1024u - (smem_u32(vsm_raw) & 1023u)) & 1023u);
    __shared__ __align__(8) uint64_t bar[kXWarps][kVStages + 1];  // K-block stages, then scales
    __shared__ int s_item;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int fg = lane >> 2, ft = lane & 3;
    const int ips = (a.n_chunks + kXWarps - 1) / kXWarps;
    uint8_t* wring = vsm + static_cast<size_t>(warp) * VG::RING;           // this warp's ring
    uint8_t* wsz = vsm + static_cast<size_t>(kXWarps) * VG::RING + warp * VG::SZP;  // its scales + zeros
    uint8_t* xhi = vsm + static_cast<size_t>(kXWarps) * (VG::RING + VG::SZP);
    uint8_t* xlo = xhi + kSegTok * XG::ROWB;
    float* xsum = reinterpret_cast<float*>(xlo + kSegTok * XG::ROWB);     // [token][XS_LD]
    if (lane == 0) {
        for (int i = 0; i <= kVStages; ++i) mbar_init(&bar[warp][i], 1);
        mbar_fence_init();
    }
    __syncwarp();
    uint32_t phase = 0;  // bit i: parity of the next wait on bar[warp][i]
    pdl_wait();
    const int nitems = a.work[0] * ips;
    pdl_launch_dependents();

    while (true) {
        if (tid == 0) s_item = atomicAdd(a.work + a.work_slot, 1);
        __syncthreads();
        const int item = s_item;
        if (item >= nitems) break;
        const int4 sg = a.segs[item / ips];
        const int part = item % ips;
        const int ex = sg.x, pair0 = sg.y, ntok = sg.z;
        const int c = part * kXWarps + warp;
        const bool has_chunk = c < a.n_chunks;
        const uint8_t* ch = nullptr;
        if (has_chunk) {
            const uint8_t* rec = ex < a.E ? a.experts + static_cast<int64_t>(ex) * a.expert_bytes : a.shared;
            ch = rec + a.proj_off + static_cast<int64_t>(c) * a.chunk_bytes;
        }
        // ---- this warp's copies: scales + zeros, the first kVStages K-blocks ----
        auto issue_kb = [&](int kb) {
            const int st = kb % kVStages;
            mbar_arrive_expect_tx(&bar[warp][st], kVBox);
            tma_load_4d(wring + st * kVBox, &a.wmap, 128 * kb, 0, c, ex, &bar[warp][st]);
        };
        if (has_chunk && lane == 0) {
            fence_proxy_async_smem();  // the previous item's reads of the ring come first
            mbar_arrive_expect_tx(&bar[warp][kVStages], VG::SZ);
            bulk_g2s(wsz, ch + XG::S_OFF, VG::SZ, &bar[warp][kVStages]);
            for (int kb = 0; kb < VG::NKB && kb < kVStages; ++kb) issue_kb(kb);
        }

        // ---- stage the segment's activation rows (hi, lo) and their 16-column sums ----
        for (int t = tid; t < kSegTok * (K / 16); t += kXThreads) {
            const int r = t / (K / 16), c16 = t % (K / 16);
            float v[16];
            if (r < ntok) {
                const float* row;
                if (GATEUP) {
                    const int src = a.pair_src[pair0 + r] >> 5;
                    row = a.ep.xn[src / a.n] + static_cast<size_t>(src % a.n) * K;
                } else {
                    row = a.h_in + static_cast<size_t>(pair0 + r) * K;
                }
                const float4* src = reinterpret_cast<const float4*>(row + 16 * c16);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float4 f = src[i];
                    v[4 * i] = f.x;
                    v[4 * i + 1] = f.y;
                    v[4 * i + 2] = f.z;
                    v[4 * i + 3] = f.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; ++i) v[i] = 0.0f;
            }
            uint32_t hw[8], lw[8];
            float sum = 0.0f;
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const int j = (m & 3) + 8 * (m >> 2);
                const uint16_t h0 = f32_to_bf16(v[j]), h1 = f32_to_bf16(v[j + 4]);
                const uint16_t l0 = f32_to_bf16(v[j] - bf16_to_f32(h0)), l1 = f32_to_bf16(v[j + 4] - bf16_to_f32(h1));
                hw[m] = static_cast<uint32_t>(h0) | (static_cast<uint32_t>(h1) << 16);
                lw[m] = static_cast<uint32_t>(l0) | (static_cast<uint32_t>(l1) << 16);
                sum += (bf16_to_f32(h0) + bf16_to_f32(l0)) + (bf16_to_f32(h1) + bf16_to_f32(l1));
            }
            uint4* dh = reinterpret_cast<uint4*>(xhi + r * XG::ROWB + 32 * c16);
            uint4* dl = reinterpret_cast<uint4*>(xlo + r * XG::ROWB + 32 * c16);
            dh[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            dh[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
            dl[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            dl[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
            xsum[r * VG::XS_LD + c16] = sum;
        }
        __syncthreads();

        if (has_chunk) {
            bool ok = mbar_wait_bounded(&bar[warp][kVStages], (phase >> kVStages) & 1u, a.err, nullptr);
            phase ^= 1u << kVStages;
            // zero words of rows fg, fg + 8; scales read per group from the staged block
            uint32_t za[XG::ZW], zb[XG::ZW];
            {
                const uint8_t* z0 = wsz + (XG::Z_OFF - XG::S_OFF) + fg * XG::ZB;
                const uint8_t* z1 = wsz + (XG::Z_OFF - XG::S_OFF) + (fg + 8) * XG::ZB;
                if (XG::ZB >= 4) {
#pragma unroll
                    for (int i = 0; i < XG::ZW; ++i) {
                        za[i] = reinterpret_cast<const uint32_t*>(z0)[i];
                        zb[i] = reinterpret_cast<const uint32_t*>(z1)[i];
                    }
                } else {
                    uint32_t va = 0, vb = 0;
#pragma unroll
                    for (int i = 0; i < XG::ZB; ++i) {
                        va |= static_cast<uint32_t>(z0[i]) << (8 * i);
                        vb |= static_cast<uint32_t>(z1[i]) << (8 * i);
                    }
                    za[0] = va;
                    zb[0] = vb;
                }
            }
            const uint16_t* sa = reinterpret_cast<const uint16_t*>(wsz) + fg * XG::NG;
            const uint16_t* sb = reinterpret_cast<const uint16_t*>(wsz) + (fg + 8) * XG::NG;
            const uint8_t* bh = xhi + fg * XG::ROWB + 32 * ft;
            const uint8_t* bl = xlo + fg * XG::ROWB + 32 * ft;
            const float* xs0 = xsum + (2 * ft) * VG::XS_LD;      // token 2ft
            const float* xs1 = xsum + (2 * ft + 1) * VG::XS_LD;  // token 2ft + 1
            float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
            for (int kb = 0; kb < VG::NKB; ++kb) {
                const int st = kb % kVStages;
                ok = mbar_wait_bounded(&bar[warp][st], (phase >> st) & 1u, a.err, nullptr) && ok;
                phase ^= 1u << st;
                const uint8_t* tile = wring + st * kVBox;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int g = 4 * kb + j;
                    // lane's 8 bytes of the group: unit (2j + ft / 2) of the row, swizzled
                    const int u = 2 * j + (ft >> 1);
                    const uint2 wa = *reinterpret_cast<const uint2*>(tile + fg * 128 + ((u ^ (fg & 7)) << 4) + (ft & 1) * 8);
                    const uint2 wb =
                        *reinterpret_cast<const uint2*>(tile + (fg + 8) * 128 + ((u ^ ((fg + 8) & 7)) << 4) + (ft & 1) * 8);
                    const float sca = __half2float(__ushort_as_half(sa[g]));
                    const float scb = __half2float(__ushort_as_half(sb[g]));
                    const float zqa = static_cast<float>(128u + ((za[g >> 3] >> (4 * (g & 7))) & 15u));
                    const float zqb = static_cast<float>(128u + ((zb[g >> 3] >> (4 * (g & 7))) & 15u));
                    const uint4 h0 = lds128(bh + 128 * g), h1 = lds128(bh + 128 * g + 16);
                    const uint4 l0 = lds128(bl + 128 * g), l1 = lds128(bl + 128 * g + 16);
                    float ch_[4] = {0.0f, 0.0f, 0.0f, 0.0f}, cl_[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                    const uint32_t ax4 = wa.x >> 4, bx4 = wb.x >> 4, ay4 = wa.y >> 4, by4 = wb.y >> 4;
                    {
                        const uint32_t a0 = nib_pair128(wa.x), a1 = nib_pair128(wb.x);
                        const uint32_t a2 = nib_pair128(ax4), a3 = nib_pair128(bx4);
                        mma_bf16_m16n8k16(ch_, a0, a1, a2, a3, h0.x, h0.y);
                        mma_bf16_m16n8k16(cl_, a0, a1, a2, a3, l0.x, l0.y);
                    }
                    {
                        const uint32_t a0 = nib_pair128(wa.x >> 8), a1 = nib_pair128(wb.x >> 8);
                        const uint32_t a2 = nib_pair128(ax4 >> 8), a3 = nib_pair128(bx4 >> 8);
                        mma_bf16_m16n8k16(ch_, a0, a1, a2, a3, h0.z, h0.w);
                        mma_bf16_m16n8k16(cl_, a0, a1, a2, a3, l0.z, l0.w);
                    }
                    {
                        const uint32_t a0 = nib_pair128(wa.y), a1 = nib_pair128(wb.y);
                        const uint32_t a2 = nib_pair128(ay4), a3 = nib_pair128(by4);
                        mma_bf16_m16n8k16(ch_, a0, a1, a2, a3, h1.x, h1.y);
                        mma_bf16_m16n8k16(cl_, a0, a1, a2, a3, l1.x, l1.y);
                    }
                    {
                        const uint32_t a0 = nib_pair128(wa.y >> 8), a1 = nib_pair128(wb.y >> 8);
                        const uint32_t a2 = nib_pair128(ay4 >> 8), a3 = nib_pair128(by4 >> 8);
                        mma_bf16_m16n8k16(ch_, a0, a1, a2, a3, h1.z, h1.w);
                        mma_bf16_m16n8k16(cl_, a0, a1, a2, a3, l1.z, l1.w);
                    }
                    // group sums of the two tokens: the 4 staged 16-column partials in order
                    const float4 p0 = *reinterpret_cast<const float4*>(xs0 + 4 * g);
                    const float4 p1 = *reinterpret_cast<const float4*>(xs1 + 4 * g);
                    const float s0 = ((p0.x + p0.y) + p0.z) + p0.w;
                    const float s1 = ((p1.x + p1.y) + p1.z) + p1.w;
                    acc[0] = fmaf(sca, fmaf(-zqa, s0, ch_[0] + cl_[0]), acc[0]);
                    acc[1] = fmaf(sca, fmaf(-zqa, s1, ch_[1] + cl_[1]), acc[1]);
                    acc[2] = fmaf(scb, fmaf(-zqb, s0, ch_[2] + cl_[2]), acc[2]);
                    acc[3] = fmaf(scb, fmaf(-zqb, s1, ch_[3] + cl_[3]), acc[3]);
                }
                __syncwarp();  // every lane is done with the stage
                if (lane == 0 && kb + kVStages < VG::NKB) {
                    fence_proxy_async_smem();
                    issue_kb(kb + kVStages);
                }
            }
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int t = 2 * ft + e;
                if (t < ntok) {
                    if (GATEUP) {
                        a.h_out[static_cast<size_t>(pair0 + t) * (a.n_chunks * 8) + 8 * c + fg] =
                            silu_f(acc[e]) * acc[2 + e];
                    } else {
                        const int ps = a.pair_src[pair0 + t];
                        const int src = ps >> 5, k = ps & 31;
                        float* dst = a.ep.eout[src / a.n] + (static_cast<size_t>(src % a.n) * (a.topk + 1) + k) * a.H;
                        dst[16 * c + fg] = acc[e];
                        dst[16 * c + fg + 8] = acc[2 + e];
                    }
                }
            }
        }
        __syncthreads();  // staged rows free; s_item read by every thread
    }
    if (!GATEUP && a.ep.world > 1) __threadfence_system();
}

#define DM_XK_INSTANCES(X) X(128) X(256) X(512) X(1024) X(2048) X(4096)
#define DM_VK_INSTANCES(X) X(256) X(512) X(1024) X(2048)

cudaError_t b_experts_set_attrs() {
    cudaError_t e = cudaSuccess;
#define DM_XK_ATTR(KK)                                                                                        \
    if (e == cudaSuccess)                                                                                     \
        e = cudaFuncSetAttribute(b_expert_kernel<KK, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,       \
                                 static_cast<int>(XGeom<KK>::SMEM));                                          \
    if (e == cudaSuccess)                                                                                     \
        e = cudaFuncSetAttribute(b_expert_kernel<KK, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,      \
                                 static_cast<int>(XGeom<KK>::SMEM));
    DM_XK_INSTANCES(DM_XK_ATTR)
#undef DM_XK_ATTR
#define DM_VK_ATTR(KK)                                                                                        \
    if (e == cudaSuccess)                                                                                     \
        e = cudaFuncSetAttribute(b_expert_tma_kernel<KK, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                                 static_cast<int>(VGeom<KK>::SMEM));                                          \
    if (e == cudaSuccess)                                                                                     \
        e = cudaFuncSetAttribute(b_expert_tma_kernel<KK, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                                 static_cast<int>(VGeom<KK>::SMEM));
    DM_VK_INSTANCES(DM_VK_ATTR)
#undef DM_VK_ATTR
    return e;
}

static cudaError_t launch_expert_proj(const LaunchCfg& lc, int K, bool gateup, const BExpArgs& a, bool tma) {
    const dim3 grid(lc.num_sms), block(kXThreads);
    if (tma) {
#define DM_VK_LAUNCH(KK)                                                                                      \
        if (K == KK)                                                                                          \
            return gateup ? launch_kernel(lc, b_expert_tma_kernel<KK, true>, grid, block, VGeom<KK>::SMEM, a)  \
                          : launch_kernel(lc, b_expert_tma_kernel<KK, false>, grid, block, VGeom<KK>::SMEM, a);
        DM_VK_INSTANCES(DM_VK_LAUNCH)
#undef DM_VK_LAUNCH
        return cudaErrorInvalidValue;
    }
#define DM_XK_LAUNCH(KK)                                                                                      \
    if (K == KK)                                                                                              \
        return gateup ? launch_kernel(lc, b_expert_kernel<KK, true>, grid, block, XGeom<KK>::SMEM, a)          \
                      : launch_kernel(lc, b_expert_kernel<KK, false>, grid, block, XGeom<KK>::SMEM, a);
    DM_XK_INSTANCES(DM_XK_LAUNCH)
#undef DM_XK_LAUNCH
    return cudaErrorInvalidValue;
}

bool expert_tma_supported(int K) { return K == 256 || K == 512 || K == 1024 || K == 2048; }

cudaError_t launch_b_experts(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& bb,
                             const Buffers& b, int n) {
    BExpArgs a{};
    a.experts = w.experts;
    a.shared = w.shared;
    a.expert_bytes = d.expert_bytes;
    a.E = d.E_res;  // routed records before the shared one
    a.segs = bb.segs;
    a.work = bb.work;
    a.pair_src = bb.pair_src;
    a.n = n;
    a.topk = d.topk;
    a.ep = bb.ep;
    a.H = d.H;
    a.err = b.err;
    // gate/up: K = H, chunks of 8 gate + 8 up rows
    a.proj_off = 0;
    a.chunk_bytes = d.gu_chunk_bytes;
    a.n_chunks = d.gu_chunks;
    a.work_slot = 1;
    a.h_out = bb.h;
    const bool tma_gu = w.tm_gu != nullptr && expert_tma_supported(d.H);
    if (tma_gu) a.wmap = *static_cast<const CUtensorMap*>(w.tm_gu);
    cudaError_t e = launch_expert_proj(lc, d.H, true, a, tma_gu);
    if (e != cudaSuccess) return e;
    // down: K = I, chunks of 16 output rows
    a.proj_off = static_cast<int64_t>(d.gu_chunks) * d.gu_chunk_bytes;
    a.chunk_bytes = d.d_chunk_bytes;
    a.n_chunks = d.d_chunks;
    a.work_slot = 2;
    a.h_in = bb.h;
    const bool tma_dn = w.tm_dn != nullptr && expert_tma_supported(d.I);
    if (tma_dn) a.wmap = *static_cast<const CUtensorMap*>(w.tm_dn);
    return launch_expert_proj(lc, d.I, false, a, tma_dn);
}

}  // namespace dm
