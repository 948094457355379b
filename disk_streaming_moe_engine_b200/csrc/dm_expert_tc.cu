// dm_expert_tc.cu — routed + shared experts of the batched decode step on the 5th-generation
// tensor cores (tcgen05, accumulators in tensor memory), fed by TMA, with the 4-bit weights
// dequantised exactly in shared memory.
//
// Reference: parallel_moe_experts (src/core/worker_pool.mojo:383) running swiglu_forward
// (src/layers/swiglu.mojo:52) per expert over the tokens routed to it; weights in the
// asymmetric 4-bit format w = s * (q - z), one fp16 scale s and one 4-bit zero z per
// group of 64 along K, nibbles low first (quant_format.md:831-854).
//
// Work.  The (token, expert) pairs of a layer are grouped by expert into segments of at
// most kSegTok = 64 tokens.  A segment's activations are staged once, before the expert
// kernels, as a bf16 operand of 2T rows (row 2t = hi(x_t), row 2t + 1 = lo(x_t) with
// x = hi + lo to 2^-16), padded to N = a multiple of 16 rows, in 64-column group tiles
// laid out exactly as the MMA reads them (128-byte swizzle).  An item is one segment and
// one M-tile of 128 weight rows; CTAs take items c, c + grid, ... in order.
//
// Per 64-column group g of the item (one fp16 scale per row):
//   producer warp   TMA: the 8 chunks' nibble boxes of the current 256-column K-block,
//                   the group's B tile (1-D bulk copy of N x 128 bytes), and once per item
//                   the 8 chunks' scales and zeros;
//   math warps 0-3  thread r owns weight row r: A[r][k] = bf16(q - z), exact (integers in
//                   -15..15), written into a swizzled 128 x 64 tile; then, for the group
//                   before, acc[n] += s[r][g] * D[r][n] read from tensor memory (fp32);
//   MMA warp        one thread: D = A B^T over K = 64 (4 x tcgen05.mma, M = 128, N) into
//                   one of 4 tensor-memory accumulators (128 columns each), committed to
//                   mbarriers that release the accumulator, the A tile and the B tile.
// Every product is exact and accumulates in fp32; the group scale multiplies the group's
// fp32 partial, as the format defines.  Each wait is bounded (1 s of %globaltimer): on a
// timeout the kernel raises the error bit, every role stops, the producer waits for its
// copies in flight, the MMA thread for its MMAs, and the tensor memory is freed.
//
// gate/up (K = H): chunk c of a record holds gate rows 8c..8c+7, then up rows 8c..8c+7, so
//   tile t covers intermediate indices 64t..64t+63 and lane r + 8 holds the up row of the
//   gate row in lane r: h = SiLU(gate) * up is formed with one shuffle and written, split
//   hi/lo, straight into group t of the down projection's staged operand.
// down (K = I): tile t is output rows 128t..128t+127 of every token, stored into the
//   expert-output rows of the token's source rank (peer memory in an expert-parallel
//   group: plain stores, no TMA on peer memory).
#include <cuda.h>

#include "dm_kernels.h"
#include "dm_tc.cuh"

namespace dm {

constexpr int kTcThreads = 192;   // warps 0-3 math, warp 4 producer, warp 5 MMA + allocator
constexpr int kTcNKS = 3;         // nibble K-block stages
constexpr int kTcNAS = 3;         // dequantised A tiles
constexpr int kTcNBS = 4;         // B group tiles
constexpr int kTcNACC = 4;        // tensor-memory accumulators
constexpr int kTcAccCols = 128;   // columns of one accumulator (N <= 128: 64 tokens, hi + lo)
constexpr int kTcTile = 16384;    // bytes of one A or B tile buffer (128 rows x 128 bytes)

static_assert(2 * kSegTok <= kTcAccCols, "a segment's hi and lo rows fit one accumulator");

template <int K>
struct TcGeom {
    static constexpr int NG = K / 64;                      // scale groups along K
    static constexpr int KB = K < 256 ? K : 256;           // columns of one nibble stage
    static constexpr int GPB = KB / 64;                    // groups per stage
    static constexpr int RB = KB / 2;                      // bytes of one row in a stage box
    static constexpr bool SWZ = RB == 128;                 // 128-byte swizzle, else plain 64-byte rows
    static constexpr int BOX = 16 * RB;                    // one chunk's box
    static constexpr int NIB = 8 * BOX;                    // one stage: 8 chunks = 128 rows
    static constexpr int NIB_AL = (NIB + 1023) / 1024 * 1024;
    static constexpr int SZC = 16 * NG * 2 + 16 * NG / 2;  // scales + zeros of one chunk
    static constexpr int SZ = 8 * SZC;
    static constexpr int S_OFF = 16 * K / 2;               // scales inside a chunk
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = A_OFF + kTcNAS * kTcTile;
    static constexpr int N_OFF = B_OFF + kTcNBS * kTcTile;
    static constexpr int SZ_OFF = N_OFF + kTcNKS * NIB_AL;
    static constexpr size_t SMEM = SZ_OFF + 2 * SZ + 1024;  // + alignment slack
    static_assert(K % 128 == 0 && K >= 128, "whole zero bytes and 64-column groups");
    static_assert(SZC % 16 == 0, "bulk copies of scales and zeros");
    static_assert(SMEM <= 227 * 1024, "shared memory of the expert kernel");
};

struct TcExpArgs {
    const uint8_t* experts;   // record 0 of the layer's pool; the shared record follows the routed ones
    int64_t expert_bytes, proj_off, chunk_bytes;
    const int4* segs;         // (record, first pair, tokens, first staged column)
    const int* work;          // [0] segments
    const int* pair_src;      // (source rank * n + row) * 32 + k of each pair
    int n, topk, H, I;
    int tiles;                // M-tiles (128 weight rows) per segment
    const uint8_t* bstage;    // this projection's staged operand: [columns][K] bf16 in group tiles
    uint8_t* hstage;          // gate/up: the down projection's staged operand
    EpView ep;                // down: expert outputs of each source rank
    CUtensorMap wmap;         // nibble rows of the pool: (row bytes, 16 rows, chunk, record)
    uint32_t* err;
};

DM_DEV int seg_cols(int tokens) { return (2 * tokens + 15) / 16 * 16; }

DM_DEV void tma_load_4d_tc(void* smem_dst, const CUtensorMap* map, int x, int y, int z, int w, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
        : "memory");
}

DM_DEV void sts128(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(smem_u32(p)), "r"(a), "r"(b), "r"(c), "r"(d)
                 : "memory");
}

// Four nibble pairs of one 32-bit word (bytes b0..b3, low nibble first) as bf16 pairs
// (q_lo - z, q_hi - z): the nibble becomes the low mantissa bits of 128.0 (exact), and the
// packed subtraction of 128 + z is exact.
DM_DEV void nib_word_minus_zero(uint32_t w, uint32_t zpair, uint32_t (&out)[4]) {
    const uint32_t lo4 = w & 0x0F0F0F0Fu, hi4 = (w >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t p = (__byte_perm(lo4, hi4, static_cast<uint32_t>(k | ((4 + k) << 8))) & 0x000F000Fu) | 0x43004300u;
        asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(out[k]) : "r"(p), "r"(zpair));
    }
}

template <int K, bool GATEUP>
__global__ void __launch_bounds__(kTcThreads, 1) b_expert_tc_kernel(const __grid_constant__ TcExpArgs a) {
    using G = TcGeom<K>;
    extern __shared__ __align__(1024) uint8_t tsm_raw[];
    uint8_t* sm = tsm_raw + ((1024u - (smem_u32(tsm_raw) & 1023u)) & 1023u);
    __shared__ __align__(8) uint64_t nib_full[kTcNKS], nib_empty[kTcNKS], a_full[kTcNAS], a_empty[kTcNAS],
        b_full[kTcNBS], b_empty[kTcNBS], acc_full[kTcNACC], acc_empty[kTcNACC], sz_full[2], sz_empty[2], done_bar;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    volatile int* abort_flag = &s_abort;
    if (tid == 0) {
        for (int i = 0; i < kTcNKS; ++i) {
            mbar_init(&nib_full[i], 1);
            mbar_init(&nib_empty[i], 128);
        }
        for (int i = 0; i < kTcNAS; ++i) {
            mbar_init(&a_full[i], 128);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < kTcNBS; ++i) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < kTcNACC; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 128);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sz_full[i], 1);
            mbar_init(&sz_empty[i], 128);
        }
        mbar_init(&done_bar, 1);
        mbar_fence_init();
        s_abort = 0;
    }
    if (warp == 5) tc_alloc(&s_tmem, kTcNACC * kTcAccCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    pdl_wait();  // segments, pairs and the staged operand come from the kernels before
    const int nitems = a.work[0] * a.tiles;
    pdl_launch_dependents();

    if (warp == 4) {
        // ---------------- producer: TMA nibble stages, B tiles, scales + zeros ----------------
        if (lane == 0) {
            uint32_t kbq = 0, q = 0, it = 0;
            for (int item = blockIdx.x; item < nitems; item += gridDim.x, ++it) {
                const int4 sg = a.segs[item / a.tiles];
                const int t = item % a.tiles;
                const int N = seg_cols(sg.z);
                const uint8_t* rec = a.experts + static_cast<int64_t>(sg.x) * a.expert_bytes + a.proj_off;
                const int sb = it & 1;
                if (!mbar_wait_bounded(&sz_empty[sb], ring_parity(it, 2) ^ 1u, a.err, abort_flag)) break;
                mbar_arrive_expect_tx(&sz_full[sb], G::SZ);
                for (int c = 0; c < 8; ++c)
                    bulk_g2s(sm + G::SZ_OFF + sb * G::SZ + c * G::SZC,
                             rec + static_cast<int64_t>(8 * t + c) * a.chunk_bytes + G::S_OFF, G::SZC, &sz_full[sb]);
                const uint8_t* bst = a.bstage + static_cast<size_t>(sg.w) * K * 2;
                bool ok = true;
                for (int g = 0; g < G::NG && ok; ++g, ++q) {
                    if (g % G::GPB == 0) {
                        const int s = kbq % kTcNKS;
                        if (!(ok = mbar_wait_bounded(&nib_empty[s], ring_parity(kbq, kTcNKS) ^ 1u, a.err, abort_flag)))
                            break;
                        fence_proxy_async_smem();
                        mbar_arrive_expect_tx(&nib_full[s], G::NIB);
                        for (int c = 0; c < 8; ++c)
                            tma_load_4d_tc(sm + G::N_OFF + s * G::NIB_AL + c * G::BOX, &a.wmap, G::RB * (g / G::GPB), 0,
                                           8 * t + c, sg.x, &nib_full[s]);
                        ++kbq;
                    }
                    const int bs = q % kTcNBS;
                    if (!(ok = mbar_wait_bounded(&b_empty[bs], ring_parity(q, kTcNBS) ^ 1u, a.err, abort_flag))) break;
                    mbar_arrive_expect_tx(&b_full[bs], static_cast<uint32_t>(N) * 128u);
                    bulk_g2s(sm + G::B_OFF + bs * kTcTile, bst + static_cast<size_t>(g) * N * 128,
                             static_cast<uint32_t>(N) * 128u, &b_full[bs]);
                }
                if (!ok) break;
            }
            // every copy this thread issued has landed before the CTA may leave (bounded)
            for (uint32_t u = kbq > kTcNKS ? kbq - kTcNKS : 0; u < kbq; ++u)
                mbar_wait_bounded(&nib_full[u % kTcNKS], ring_parity(u, kTcNKS), a.err, nullptr);
            for (uint32_t u = q > kTcNBS ? q - kTcNBS : 0; u < q; ++u)
                mbar_wait_bounded(&b_full[u % kTcNBS], ring_parity(u, kTcNBS), a.err, nullptr);
            for (uint32_t u = it > 2 ? it - 2 : 0; u < it; ++u)
                mbar_wait_bounded(&sz_full[u % 2], ring_parity(u, 2), a.err, nullptr);
        }
    } else if (warp == 5) {
        // ---------------- MMA issue (one thread) ----------------
        if (lane == 0) {
            uint32_t q = 0;
            bool ok = true;
            for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
                const int4 sg = a.segs[item / a.tiles];
                const uint32_t idesc = tc_idesc_bf16(128, seg_cols(sg.z));
                for (int g = 0; g < G::NG; ++g, ++q) {
                    const int as = q % kTcNAS, bs = q % kTcNBS, ab = q % kTcNACC;
                    ok = mbar_wait_bounded(&a_full[as], ring_parity(q, kTcNAS), a.err, abort_flag) &&
                         mbar_wait_bounded(&b_full[bs], ring_parity(q, kTcNBS), a.err, abort_flag) &&
                         mbar_wait_bounded(&acc_empty[ab], ring_parity(q, kTcNACC) ^ 1u, a.err, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    const uint64_t ad = tc_desc_sw128(smem_u32(sm + G::A_OFF + as * kTcTile));
                    const uint64_t bd = tc_desc_sw128(smem_u32(sm + G::B_OFF + bs * kTcTile));
                    const uint32_t d = tmem + static_cast<uint32_t>(ab * kTcAccCols);
#pragma unroll
                    for (int k = 0; k < 4; ++k) tc_mma_bf16(d, ad + 2 * k, bd + 2 * k, idesc, k > 0);
                    tc_commit(&acc_full[ab]);
                    tc_commit(&a_empty[as]);
                    tc_commit(&b_empty[bs]);
                }
            }
            tc_commit(&done_bar);  // every MMA issued above has completed once this arrives
            mbar_wait_bounded(&done_bar, 0, a.err, nullptr);
        }
    } else {
        // ---------------- math warps: dequantise, drain, epilogue ----------------
        const int r = tid;  // weight row of the tile = tensor-memory lane
        uint32_t kbq = 0, q = 0, it = 0;
        float acc[kTcAccCols];
        bool ok = true;
        // waits of the math warps are made warp-uniform: the tensor-memory loads after them
        // are .sync.aligned and need every lane
        auto wwait = [&](uint64_t* bar, uint32_t parity) -> bool {
            return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, a.err, abort_flag));
        };
        for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x, ++it) {
            const int4 sg = a.segs[item / a.tiles];
            const int t = item % a.tiles;
            const int T = sg.z;
            const int N = seg_cols(T);
            const int sb = it & 1;
            if (!(ok = wwait(&sz_full[sb], ring_parity(it, 2)))) break;
            const uint8_t* szc = sm + G::SZ_OFF + sb * G::SZ + (r >> 4) * G::SZC;
            const uint16_t* srow = reinterpret_cast<const uint16_t*>(szc + (r & 15) * G::NG * 2);
            const uint8_t* zrow = szc + 16 * G::NG * 2 + (r & 15) * (G::NG / 2);
#pragma unroll
            for (int j = 0; j < kTcAccCols; ++j) acc[j] = 0.0f;
            uint8_t* arow = sm + G::A_OFF + (r >> 3) * 1024 + (r & 7) * 128;
            const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * warp) << 16);

            auto drain = [&](uint32_t qq, int gg) -> bool {
                const int ab = qq % kTcNACC;
                if (!wwait(&acc_full[ab], ring_parity(qq, kTcNACC))) return false;
                tc_fence_after();
                const float sc = __half2float(__ushort_as_half(srow[gg]));
                const uint32_t ta = lane_base + static_cast<uint32_t>(ab * kTcAccCols);
#pragma unroll
                for (int c = 0; c < kTcAccCols / 16; ++c) {
                    if (c * 16 < N) {
                        float v[16];
                        tc_ld16(ta + 16 * c, v);
                        tc_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j) acc[16 * c + j] = fmaf(sc, v[j], acc[16 * c + j]);
                    }
                }
                tc_fence_before();
                mbar_arrive(&acc_empty[ab]);
                return true;
            };

            for (int g = 0; g < G::NG; ++g, ++q) {
                const int s = kbq % kTcNKS;
                const int gk = g % G::GPB;
                if (gk == 0 && !(ok = wwait(&nib_full[s], ring_parity(kbq, kTcNKS)))) break;
                const int as = q % kTcNAS;
                if (!(ok = wwait(&a_empty[as], ring_parity(q, kTcNAS) ^ 1u))) break;
                // row r, group g: 32 nibble bytes -> 64 bf16 (q - z)
                const uint8_t* nrow = sm + G::N_OFF + s * G::NIB_AL + (r >> 4) * G::BOX + (r & 15) * G::RB;
                uint4 w0, w1;
                if (G::SWZ) {
                    w0 = *reinterpret_cast<const uint4*>(nrow + (((2 * gk) ^ (r & 7)) << 4));
                    w1 = *reinterpret_cast<const uint4*>(nrow + (((2 * gk + 1) ^ (r & 7)) << 4));
                } else {
                    w0 = *reinterpret_cast<const uint4*>(nrow + 32 * gk);
                    w1 = *reinterpret_cast<const uint4*>(nrow + 32 * gk + 16);
                }
                const uint32_t z = (zrow[g >> 1] >> (4 * (g & 1))) & 15u;
                const uint32_t zpair = (0x4300u | z) * 0x10001u;
                const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                uint8_t* adst = arow + as * kTcTile;
#pragma unroll
                for (int v = 0; v < 8; ++v) {
                    uint32_t o[4];
                    nib_word_minus_zero(words[v], zpair, o);
                    sts128(adst + ((v ^ (r & 7)) << 4), o[0], o[1], o[2], o[3]);
                }
                fence_proxy_async_smem();  // generic writes before the tensor cores read the tile
                mbar_arrive(&a_full[as]);
                if (gk == G::GPB - 1) {
                    mbar_arrive(&nib_empty[s]);
                    ++kbq;
                }
                if (g > 0 && !(ok = drain(q - 1, g - 1))) break;
            }
            if (ok) ok = drain(q - 1, G::NG - 1);
            mbar_arrive(&sz_empty[sb]);
            if (!ok) break;

            // ---------------- epilogue: hi + lo columns of every token ----------------
            if (GATEUP) {
                const int j = r & 15;
                const int i_loc = 8 * (r >> 4) + (j & 7);  // intermediate index inside the tile's 64
                uint8_t* hst = a.hstage + static_cast<size_t>(sg.w) * a.I * 2 + static_cast<size_t>(t) * N * 128;
#pragma unroll
                for (int tok = 0; tok < kSegTok; ++tok) {
                    if (tok < T) {
                        const float y = acc[2 * tok] + acc[2 * tok + 1];
                        const float u = __shfl_down_sync(0xffffffffu, y, 8);
                        if (j < 8) {
                            const float h = silu_f(y) * u;
                            const uint16_t hi = f32_to_bf16(h);
                            const uint16_t lo = f32_to_bf16(h - bf16_to_f32(hi));
                            *reinterpret_cast<uint16_t*>(hst + sw128_off(2 * tok, i_loc)) = hi;
                            *reinterpret_cast<uint16_t*>(hst + sw128_off(2 * tok + 1, i_loc)) = lo;
                        }
                    }
                }
            } else {
                const int o = 128 * t + r;
#pragma unroll
                for (int tok = 0; tok < kSegTok; ++tok) {
                    if (tok < T) {
                        const int ps = a.pair_src[sg.y + tok];
                        const int src = ps >> 5, k = ps & 31;
                        float* dst = a.ep.eout[src / a.n] + (static_cast<size_t>(src % a.n) * (a.topk + 1) + k) * a.H;
                        dst[o] = acc[2 * tok] + acc[2 * tok + 1];
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tc_dealloc(tmem, kTcNACC * kTcAccCols);
    }
    if (!GATEUP && a.ep.world > 1) __threadfence_system();
}

// ---- staging of the gate/up operand: each segment's token rows as hi/lo bf16 tiles ----
struct XStageArgs {
    const int4* segs;
    const int* work;
    const int* pair_src;
    int n, K;
    EpView ep;          // the normalised MoE inputs of every source rank (peer memory: plain loads)
    uint8_t* stage;
};

__global__ void __launch_bounds__(256) b_xstage_kernel(const __grid_constant__ XStageArgs a) {
    pdl_wait();
    const int nseg = a.work[0];
    pdl_launch_dependents();
    const int units = a.K / 8;
    for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < nseg * units; f += gridDim.x * blockDim.x) {
        const int s = f / units, v = f % units;
        const int4 sg = a.segs[s];
        const int N = seg_cols(sg.z);
        uint8_t* tile = a.stage + static_cast<size_t>(sg.w) * a.K * 2 + static_cast<size_t>(v >> 3) * N * 128;
        const int u = v & 7;
        for (int tok = 0; tok < sg.z; ++tok) {
            const int src = a.pair_src[sg.y + tok] >> 5;
            const float4* row = reinterpret_cast<const float4*>(a.ep.xn[src / a.n] + static_cast<size_t>(src % a.n) * a.K + 8 * v);
            const float4 f0 = row[0], f1 = row[1];
            const float x[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint16_t h0 = f32_to_bf16(x[2 * i]), h1 = f32_to_bf16(x[2 * i + 1]);
                const uint16_t l0 = f32_to_bf16(x[2 * i] - bf16_to_f32(h0));
                const uint16_t l1 = f32_to_bf16(x[2 * i + 1] - bf16_to_f32(h1));
                hw[i] = static_cast<uint32_t>(h0) | (static_cast<uint32_t>(h1) << 16);
                lw[i] = static_cast<uint32_t>(l0) | (static_cast<uint32_t>(l1) << 16);
            }
            const int nh = 2 * tok, nl = 2 * tok + 1;
            *reinterpret_cast<uint4*>(tile + (nh >> 3) * 1024 + (nh & 7) * 128 + ((u ^ (nh & 7)) << 4)) =
                make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4*>(tile + (nl >> 3) * 1024 + (nl & 7) * 128 + ((u ^ (nl & 7)) << 4)) =
                make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
    }
}

#define DM_TC_INSTANCES(X) X(128) X(256) X(512) X(1024) X(2048) X(4096)

bool expert_tc_supported(int K) {
    return K == 128 || K == 256 || K == 512 || K == 1024 || K == 2048 || K == 4096;
}

cudaError_t b_experts_set_attrs() {
    cudaError_t e = cudaSuccess;
#define DM_TC_ATTR(KK)                                                                                     \
    if (e == cudaSuccess)                                                                                  \
        e = cudaFuncSetAttribute(b_expert_tc_kernel<KK, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 static_cast<int>(TcGeom<KK>::SMEM));                                      \
    if (e == cudaSuccess)                                                                                  \
        e = cudaFuncSetAttribute(b_expert_tc_kernel<KK, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 static_cast<int>(TcGeom<KK>::SMEM));
    DM_TC_INSTANCES(DM_TC_ATTR)
#undef DM_TC_ATTR
    return e;
}

static cudaError_t launch_tc_proj(const LaunchCfg& lc, int K, bool gateup, const TcExpArgs& a) {
    const dim3 grid(lc.num_sms), block(kTcThreads);
#define DM_TC_LAUNCH(KK)                                                                                        \
    if (K == KK)                                                                                                \
        return gateup ? launch_kernel(lc, b_expert_tc_kernel<KK, true>, grid, block, TcGeom<KK>::SMEM, a)      \
                      : launch_kernel(lc, b_expert_tc_kernel<KK, false>, grid, block, TcGeom<KK>::SMEM, a);
    DM_TC_INSTANCES(DM_TC_LAUNCH)
#undef DM_TC_LAUNCH
    return cudaErrorInvalidValue;
}

cudaError_t launch_b_experts(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& bb,
                             const Buffers& b, int n) {
    if (!w.tm_gu || !w.tm_dn || !expert_tc_supported(d.H) || !expert_tc_supported(d.I) || d.I % 64 || d.H % 128)
        return cudaErrorInvalidValue;
    XStageArgs xs{};
    xs.segs = bb.segs;
    xs.work = bb.work;
    xs.pair_src = bb.pair_src;
    xs.n = n;
    xs.K = d.H;
    xs.ep = bb.ep;
    xs.stage = bb.xgu;
    cudaError_t e = launch_kernel(lc, b_xstage_kernel, dim3(4 * lc.num_sms), dim3(256), 0, xs);
    if (e != cudaSuccess) return e;
    TcExpArgs a{};
    a.experts = w.experts;
    a.expert_bytes = d.expert_bytes;
    a.segs = bb.segs;
    a.work = bb.work;
    a.pair_src = bb.pair_src;
    a.n = n;
    a.topk = d.topk;
    a.H = d.H;
    a.I = d.I;
    a.ep = bb.ep;
    a.err = b.err;
    // gate/up: K = H, tiles of 8 chunks (64 gate + 64 up rows)
    a.proj_off = 0;
    a.chunk_bytes = d.gu_chunk_bytes;
    a.tiles = d.I / 64;
    a.bstage = bb.xgu;
    a.hstage = bb.xdn;
    a.wmap = *static_cast<const CUtensorMap*>(w.tm_gu);
    e = launch_tc_proj(lc, d.H, true, a);
    if (e != cudaSuccess) return e;
    // down: K = I, tiles of 128 output rows
    a.proj_off = static_cast<int64_t>(d.gu_chunks) * d.gu_chunk_bytes;
    a.chunk_bytes = d.d_chunk_bytes;
    a.tiles = d.H / 128;
    a.bstage = bb.xdn;
    a.hstage = nullptr;
    a.wmap = *static_cast<const CUtensorMap*>(w.tm_dn);
    return launch_tc_proj(lc, d.I, false, a);
}

}  // namespace dm
