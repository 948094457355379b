// dm_expert_tc.cu — routed + shared experts of the batched decode step on the 5th-generation
// tensor cores (tcgen05), fed by TMA, with the 4-bit weights expanded into tensor memory.
//
// Reference: parallel_moe_experts (src/core/worker_pool.mojo:383) running swiglu_forward
// (src/layers/swiglu.mojo:52) per expert over the tokens routed to it; weights in the
// asymmetric 4-bit format w = s * (q - z), one fp16 scale s and one 4-bit zero z per
// group of 64 along K, nibbles low first (quant_format.md:831-854).
//
// Work.  The (token, expert) pairs of a layer are grouped by expert into segments of at
// most kSegTok = 32 tokens.  A segment's activations are staged once, before the expert
// kernels, as an fp16 operand B of 2T rows (row 2t = hi(x_t), row 2t + 1 = lo(x_t) with
// x = hi + lo to about 2^-22), padded to N = a multiple of 16 rows, in 64-column group
// tiles laid out as the MMA reads them from shared memory (128-byte swizzle).  Inside each
// 8-column unit the columns are stored in the order [0,4,1,5,2,6,3,7]: the order in which
// one 32-bit word of 8 nibbles yields its pairs (below); A uses the same order, so every
// dot product is unchanged.  An item is one segment and one M-tile of 128 weight rows;
// CTAs take items c, c + grid, ... in order.
//
// Arithmetic.  A nibble pair becomes the fp16 pair (1024 + q_j, 1024 + q_{j+4}) by one
// shift and one LOP3 ((w >> 4j) & 0x000F000F | 0x64006400), the packed subtraction of
// 1024 + z gives q - z exactly, and one packed multiply by the group's fp16 scale gives
// w = fp16(s (q - z)): the exact product rounded once (relative error <= 2^-12; the
// reference's own 4-bit path rounds its dequantised weights to bf16, 2^-9).  The tensor
// cores then accumulate w x over the whole K of the item in fp32 in one chain: one
// accumulator per item, read once.
//
// Why this shape.  Measured on the way (tcgen05.mma probes and %globaltimer stamps of the
// pipeline): a chain of 4 MMAs (M = 128, N = 16) plus its commit costs ~435 SM cycles,
// whatever the operands' placement, while longer chains cost ~48 cycles per MMA; keeping
// the per-group scale outside the MMA (one chain per 64 columns, drained into registers)
// ran at ~0.5 us per group.  A lives in tensor memory (tcgen05.st from the expanding
// thread's registers into its own lane), so shared memory only carries the nibbles and B.
//
// Roles (704 threads; K is processed in K-blocks of 256 columns (4 groups), held in a ring
// of 3 slots: slot j has a nibble stage, 4 A buffers in tensor memory (columns 128 + 128 j
// ..) and 4 B tiles; D buffers are tensor-memory columns [0, 128)):
//   producer warp 20   per K-block: waits for the slot's previous MMAs, then TMA-loads the
//                      8 chunks' nibble boxes and, with one 1-D bulk copy, the 4 groups' B
//                      tiles (consecutive in the staged operand); per item the 8 chunks'
//                      scales and zeros;
//   expand warps 0-15  four sets of four (one warp per sub-partition); set s expands the
//                      groups q with q % 4 == s, warp 4 s + p rows 32 p .. 32 p + 31, a whole
//                      row per thread, into the group's A buffer.  Four groups are expanded
//                      at once: one group's chain (shared-memory loads -> ALU -> tensor-memory
//                      store -> arrive) is latency-bound (with three sets the MMA thread still
//                      waited ~450 cycles per K-block for its inputs);
//   MMA warp 21        one thread: per K-block one wait (A of the 4 groups expanded and B
//                      landed: one barrier), 16 tcgen05.mma (M = 128, N, K = 16; A from
//                      tensor memory, B from shared memory) accumulating into the item's D
//                      buffer, one commit that frees the slot; at the item's end a commit
//                      hands D to the drain;
//   drain warps 16-19  warp 16 + p owns rows 32 p .. 32 p + 31: reads the item's D buffer
//                      16 columns at a time, runs the epilogue on them, frees the buffer.
// Measured on the way (tcgen05.mma probes, SM-cycle stamps of the pipeline): a chain of 4
// MMAs (N = 16) with its commit costs ~435 cycles, long chains ~70 cycles per MMA; an
// mbarrier wait in the busy kernel costs the MMA thread 200-400 cycles even when the phase
// has long completed, so the single-thread roles wait once per K-block, not per group.
// A slot cannot be reused early: the producer refills slot j for K-block kb + 3 only after
// the MMAs of kb, which need every expander's arrival for kb, so the nibbles of kb have
// been read and its A buffers and B tiles consumed; each waiter's next phase needs its own
// progress first, so no wait can miss a phase.
// Each wait is bounded (1 s of %globaltimer): on a timeout the kernel raises the error bit,
// every role stops, the producer waits for its copies in flight, the MMA thread for its
// MMAs, and the tensor memory is freed.  An activation outside the fp16 range raises
// DM_DEVERR_RANGE (the host reports an error instead of an overflowed result).
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
#include "dm_q4mma.cuh"
#include "dm_tc.cuh"

namespace dm {

constexpr int kTcSets = 4;                    // expand sets: groups expanded at once
constexpr int kTcExpWarps = 4 * kTcSets;      // one warp per sub-partition and set
constexpr int kTcExp = kTcExpWarps * 32;
constexpr int kTcDrainWarp0 = kTcExpWarps;    // drain warps, one per sub-partition
constexpr int kTcDrain = 128;
constexpr int kTcProdWarp = kTcExpWarps + 4;
constexpr int kTcMmaWarp = kTcProdWarp + 1;
constexpr int kTcThreads = (kTcMmaWarp + 1) * 32;
constexpr int kTcNKS = 3;                     // K-block slots
constexpr int kTcNACC = 2;                    // D buffers (items in flight between MMA and drain)
constexpr int kTcDCols = 64;
constexpr int kTcACols = 32;                  // one group's A buffer
constexpr int kTcACol0 = kTcNACC * kTcDCols;  // first A column
constexpr int kTcBTile = 8192;                // <= 64 rows x 128 bytes
constexpr int kTcGPBMax = 4;                  // groups per K-block

static_assert(2 * kSegTok <= kTcDCols, "a segment's hi and lo rows fit one D buffer");
static_assert(kTcACol0 + kTcNKS * kTcGPBMax * kTcACols <= 512, "tensor memory columns");

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
    static constexpr int B_OFF = 0;                        // slot j: B tiles of its 4 groups
    static constexpr int B_SLOT = kTcGPBMax * kTcBTile;
    static constexpr int N_OFF = B_OFF + kTcNKS * B_SLOT;
    static constexpr int SZ_OFF = N_OFF + kTcNKS * NIB_AL;
    static constexpr size_t SMEM = SZ_OFF + 2 * SZ + 1024;  // + alignment slack
    static_assert(K % 128 == 0 && K >= 128, "whole zero bytes and 64-column groups");
    static_assert(SZC % 16 == 0, "bulk copies of scales and zeros");
    static_assert(SMEM <= 227 * 1024, "shared memory of the expert kernel");
};

struct TcExpArgs {
    const uint8_t* experts;   // record 0 of the layer's pool; the shared record follows the routed ones
    int64_t expert_bytes, proj_off, chunk_bytes;
    const int4* segs;         // (record, first pair, tokens, first staged row)
    const int* work;          // [0] segments
    const int* pair_src;      // (source rank * n + row) * 32 + k of each pair
    int n, topk, H, I;
    int tiles;                // M-tiles (128 weight rows) per segment
    const uint8_t* bstage;    // this projection's staged operand: [rows][K] fp16 in group tiles
    uint8_t* hstage;          // gate/up: the down projection's staged operand
    EpView ep;                // down: expert outputs of each source rank
    CUtensorMap wmap;         // nibble rows of the pool: (row bytes, 16 rows, chunk, record)
    uint64_t* trace;          // CTA 0's pipeline stamps of its first kTcTraceGroups groups, or null
    uint32_t* err;
};

// Pipeline trace (CTA 0, group q < kTcTraceGroups, SM cycles), stamps per group:
// 0 producer issues the group's K-block, 1 the MMA thread starts the group's MMAs, 2 the
// expanding warp of sub-partition 0 starts (nibbles landed), 3 its tensor-memory stores are
// done, 4 it has arrived; for the last group of an item: 5 the first drain warp starts
// waiting, 6 the accumulator is ready, 7 the epilogue is done; 8 the MMA thread has issued
// the K-block's commit, 9 its wait for the K-block's inputs returned.
constexpr int kTcTraceGroups = 32;
constexpr int kTcTraceSlots = 10;
// Stamps are SM clock cycles (clock64): all of them come from CTA 0's SM, and reading
// %globaltimer per group slowed the traced kernel down by half.
DM_DEV void tc_stamp(uint64_t* tr, uint32_t q, int k) {
    if (tr && blockIdx.x == 0 && q < kTcTraceGroups) tr[kTcTraceSlots * q + k] = static_cast<uint64_t>(clock64());
}

DM_DEV int seg_cols(int tokens) { return (2 * tokens + 15) / 16 * 16; }

// Position in an mbarrier ring of N stages: the stage index and the parity of its current
// use (a "full" barrier is waited with `ph`, an "empty" one with ph ^ 1).  Kept as counters
// so that the single-thread roles do no division per group.
template <int N>
struct RingPos {
    uint32_t i = 0, ph = 0;
    DM_DEV void next() {
        if (++i == N) {
            i = 0;
            ph ^= 1u;
        }
    }
};

// Item sequence of a CTA: items c, c + grid, ...; the segment record of the next item is
// loaded one item ahead.
struct ItemIter {
    int item, nitems, tiles, t;
    int4 sg, nx;
    DM_DEV ItemIter(const int4* segs, int n, int tiles_) : item(blockIdx.x), nitems(n), tiles(tiles_) {
        t = item % tiles;
        sg = make_int4(0, 0, 0, 0);
        nx = sg;
        if (item < nitems) sg = segs[item / tiles];
        const int n2 = item + static_cast<int>(gridDim.x);
        if (n2 < nitems) nx = segs[n2 / tiles];
    }
    DM_DEV bool valid() const { return item < nitems; }
    DM_DEV void next(const int4* segs) {
        item += gridDim.x;
        t = item % tiles;
        sg = nx;
        const int n2 = item + static_cast<int>(gridDim.x);
        if (n2 < nitems) nx = segs[n2 / tiles];
    }
};

// Staged position of element e (0..7) of an 8-column unit: [0,4,1,5,2,6,3,7] holds e.
DM_DEV int unit_pos(int e) { return e < 4 ? 2 * e : 2 * (e - 4) + 1; }

// Byte offset of element k (0..63) of row n of a staged group tile.
DM_DEV uint32_t stage_off(int n, int k) {
    return static_cast<uint32_t>((n >> 3) * 1024 + (n & 7) * 128 + ((((k >> 3) ^ (n & 7)) & 7) << 4) +
                                 unit_pos(k & 7) * 2);
}

// x as fp16 hi + lo (lo = fp16(x - hi)); raises DM_DEVERR_RANGE outside the fp16 range.
DM_DEV void split_f16(float x, uint16_t& hi, uint16_t& lo, uint32_t* err) {
    if (!(fabsf(x) <= 65504.0f)) raise_error(err, DM_DEVERR_RANGE);
    const __half h = __float2half_rn(x);
    hi = __half_as_ushort(h);
    lo = __half_as_ushort(__float2half_rn(x - __half2float(h)));
}

DM_DEV void tma_load_4d_tc(void* smem_dst, const CUtensorMap* map, int x, int y, int z, int w, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
        : "memory");
}

// Pair j of a word of 8 nibbles (after the word was shifted right by 4j): the fp16 pair
// fp16(s (q_j - z)), fp16(s (q_{j+4} - z)); (1024 + q) - (1024 + z) is exact, the
// multiply rounds once.
DM_DEV uint32_t nib_pair_w(uint32_t w, uint32_t zpair, uint32_t spair) {
    uint32_t p, d, m;
    asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(p) : "r"(w));  // (a & b) | c
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(p), "r"(zpair));
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(m) : "r"(d), "r"(spair));
    return m;
}

template <int K, bool GATEUP>
__global__ void __launch_bounds__(kTcThreads, 1) b_expert_tc_kernel(const __grid_constant__ TcExpArgs a) {
    using G = TcGeom<K>;
    extern __shared__ __align__(1024) uint8_t tsm_raw[];
    uint8_t* sm = tsm_raw + ((1024u - (smem_u32(tsm_raw) & 1023u)) & 1023u);
    __shared__ __align__(8) uint64_t nib_full[kTcNKS], in_full[kTcNKS], mma_done[kTcNKS], acc_full[kTcNACC],
        acc_empty[kTcNACC], sz_full[2], sz_empty[2], done_bar;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    volatile int* abort_flag = &s_abort;
    if (tid == 0) {
        for (int i = 0; i < kTcNKS; ++i) {
            mbar_init(&nib_full[i], 1);
            mbar_init(&in_full[i], 128 * G::GPB + 1);  // every group's expanding set + the B copy
            mbar_init(&mma_done[i], 1);
        }
        for (int i = 0; i < kTcNACC; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kTcDrain);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sz_full[i], 1);
            mbar_init(&sz_empty[i], kTcExp);  // every set, every item
        }
        mbar_init(&done_bar, 1);
        mbar_fence_init();
        s_abort = 0;
    }
    if (warp == kTcMmaWarp) tc_alloc(&s_tmem, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;

    pdl_wait();  // segments, pairs and the staged operand come from the kernels before
    const int nitems = a.work[0] * a.tiles;
    pdl_launch_dependents();

    if (warp == kTcProdWarp) {
        // ---------------- producer: per K-block the nibble stage and the 4 B tiles ----------------
        if (lane == 0) {
            RingPos<kTcNKS> kq;
            RingPos<2> zq;
            uint32_t n_kb = 0, n_sz = 0, q = 0;
            bool ok = true;
            for (ItemIter itr(a.segs, nitems, a.tiles); itr.valid() && ok; itr.next(a.segs)) {
                const int4 sg = itr.sg;
                const int t = itr.t;
                const uint32_t bbytes = static_cast<uint32_t>(seg_cols(sg.z)) * 128u;
                const uint8_t* rec = a.experts + static_cast<int64_t>(sg.x) * a.expert_bytes + a.proj_off;
                if (!(ok = mbar_wait_bounded(&sz_empty[zq.i], zq.ph ^ 1u, a.err, abort_flag))) break;
                mbar_arrive_expect_tx(&sz_full[zq.i], G::SZ);
                for (int c = 0; c < 8; ++c)
                    bulk_g2s(sm + G::SZ_OFF + zq.i * G::SZ + c * G::SZC,
                             rec + static_cast<int64_t>(8 * t + c) * a.chunk_bytes + G::S_OFF, G::SZC, &sz_full[zq.i]);
                zq.next();
                ++n_sz;
                const uint8_t* bsrc = a.bstage + static_cast<size_t>(sg.w) * K * 2;
                for (int kb = 0; kb < G::NG / G::GPB; ++kb, q += G::GPB) {
                    if (!(ok = mbar_wait_bounded(&mma_done[kq.i], kq.ph ^ 1u, a.err, abort_flag))) break;
                    tc_stamp(a.trace, q, 0);
                    fence_proxy_async_smem();
                    mbar_arrive_expect_tx(&nib_full[kq.i], G::NIB);
                    uint8_t* dst = sm + G::N_OFF + kq.i * G::NIB_AL;
                    for (int c = 0; c < 8; ++c)
                        tma_load_4d_tc(dst + c * G::BOX, &a.wmap, G::RB * kb, 0, 8 * t + c, sg.x, &nib_full[kq.i]);
                    mbar_arrive_expect_tx(&in_full[kq.i], G::GPB * bbytes);
                    bulk_g2s(sm + G::B_OFF + kq.i * G::B_SLOT, bsrc, G::GPB * bbytes, &in_full[kq.i]);
                    bsrc += G::GPB * bbytes;
                    kq.next();
                    ++n_kb;
                }
            }
            // every copy this thread issued has landed before the CTA may leave (bounded)
            for (uint32_t u = n_kb > kTcNKS ? n_kb - kTcNKS : 0; u < n_kb; ++u)
                mbar_wait_bounded(&nib_full[u % kTcNKS], (u / kTcNKS) & 1u, a.err, nullptr);
            for (uint32_t u = n_sz > 2 ? n_sz - 2 : 0; u < n_sz; ++u)
                mbar_wait_bounded(&sz_full[u % 2], (u / 2) & 1u, a.err, nullptr);
            // (the B copies of a K-block complete the slot's in_full phase together with the
            //  expanders; the MMA thread's final wait covers the last ones)
        }
    } else if (warp == kTcMmaWarp) {
        // ---------------- MMA issue (one thread): one accumulation chain per item ----------------
        if (lane == 0) {
            RingPos<kTcNKS> kq;      // K-block slot
            RingPos<kTcNACC> dq;     // D buffer of the item
            uint32_t q = 0;
            bool ok = true;
            const uint32_t b0 = smem_u32(sm + G::B_OFF);
            for (ItemIter itr(a.segs, nitems, a.tiles); itr.valid() && ok; itr.next(a.segs)) {
                const int N = seg_cols(itr.sg.z);
                const uint32_t idesc = tc_idesc_f16(128, N);
                if (!mbar_try_wait(&acc_empty[dq.i], dq.ph ^ 1u) &&
                    !(ok = mbar_wait_bounded(&acc_empty[dq.i], dq.ph ^ 1u, a.err, abort_flag)))
                    break;
                const uint32_t d = tmem + dq.i * kTcDCols;
                for (int kb = 0; kb < G::NG / G::GPB; ++kb) {
                    if (!mbar_try_wait(&in_full[kq.i], kq.ph) &&
                        !(ok = mbar_wait_bounded(&in_full[kq.i], kq.ph, a.err, abort_flag)))
                        break;
                    tc_stamp(a.trace, q, 9);
                    tc_fence_after();
                    const uint32_t bslot = b0 + kq.i * G::B_SLOT;
                    for (int gk = 0; gk < G::GPB; ++gk, ++q) {
                        tc_stamp(a.trace, q, 1);
                        const uint32_t at = tmem + static_cast<uint32_t>(kTcACol0 + (kq.i * kTcGPBMax + gk) * kTcACols);
                        const uint64_t bd = tc_desc_sw128(bslot + gk * N * 128);
                        tc_mma_bf16_ts(d, at, bd, idesc, kb > 0 || gk > 0);
                        tc_mma_bf16_ts(d, at + 8, bd + 2, idesc, true);
                        tc_mma_bf16_ts(d, at + 16, bd + 4, idesc, true);
                        tc_mma_bf16_ts(d, at + 24, bd + 6, idesc, true);
                    }
                    tc_commit(&mma_done[kq.i]);
                    tc_stamp(a.trace, q - 1, 8);
                    kq.next();
                }
                if (!ok) break;
                tc_commit(&acc_full[dq.i]);
                dq.next();
            }
            tc_commit(&done_bar);  // every MMA issued above has completed once this arrives
            mbar_wait_bounded(&done_bar, 0, a.err, nullptr);
        }
    } else {
        // waits are warp-uniform: the tensor-memory accesses after them are .sync.aligned
        auto wwait = [&](uint64_t* bar, uint32_t parity) -> bool {
            return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, a.err, abort_flag));
        };
        const int sp = warp & 3;
        const int r = 32 * sp + lane;  // weight row of the tile = tensor-memory lane
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * sp) << 16);
        bool ok = true;
        if (warp < kTcExpWarps) {
            // ---------------- expand warps: nibbles -> fp16 s (q - z) pairs in tensor memory ----------------
            const int set = warp >> 2;
            RingPos<kTcNKS> kq;
            RingPos<2> zq;
            RingPos<kTcSets> mine;  // mine.i == set: this set expands the group
            uint32_t q = 0;
            for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
                const int sb = zq.i;
                if (!(ok = wwait(&sz_full[sb], zq.ph))) break;
                const uint8_t* szc = sm + G::SZ_OFF + sb * G::SZ + (r >> 4) * G::SZC;
                const uint16_t* srow = reinterpret_cast<const uint16_t*>(szc + (r & 15) * G::NG * 2);
                const uint8_t* zrow = szc + 16 * G::NG * 2 + (r & 15) * (G::NG / 2);
                for (int g = 0; g < G::NG; ++g, ++q) {
                    const int gk = g % G::GPB;
                    if (static_cast<int>(mine.i) == set) {
                        const int s = kq.i;
                        if (!(ok = wwait(&nib_full[s], kq.ph))) break;  // also: the slot's A buffers are free
                        tc_fence_after();
                        if (tid == 32 * 4 * set) tc_stamp(a.trace, q, 2);
                        // row r, group g: 64 nibbles -> 32 columns of pairs
                        const uint8_t* nrow = sm + G::N_OFF + s * G::NIB_AL + (r >> 4) * G::BOX + (r & 15) * G::RB;
                        const int u0 = 2 * gk, u1 = 2 * gk + 1;  // 16-byte units of the row's group bytes
                        const uint4 w0 = *reinterpret_cast<const uint4*>(nrow + ((G::SWZ ? (u0 ^ (r & 7)) : u0) << 4));
                        const uint4 w1 = *reinterpret_cast<const uint4*>(nrow + ((G::SWZ ? (u1 ^ (r & 7)) : u1) << 4));
                        const uint32_t z = (zrow[g >> 1] >> (4 * (g & 1))) & 15u;
                        const uint32_t zpair = (0x6400u | z) * 0x10001u;
                        const uint32_t spair = static_cast<uint32_t>(srow[g]) * 0x10001u;
                        const uint32_t words[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                        uint32_t c0[16], c1[16];
#pragma unroll
                        for (int v = 0; v < 4; ++v) {
                            c0[4 * v] = nib_pair_w(words[v], zpair, spair);
                            c0[4 * v + 1] = nib_pair_w(words[v] >> 4, zpair, spair);
                            c0[4 * v + 2] = nib_pair_w(words[v] >> 8, zpair, spair);
                            c0[4 * v + 3] = nib_pair_w(words[v] >> 12, zpair, spair);
                            c1[4 * v] = nib_pair_w(words[4 + v], zpair, spair);
                            c1[4 * v + 1] = nib_pair_w(words[4 + v] >> 4, zpair, spair);
                            c1[4 * v + 2] = nib_pair_w(words[4 + v] >> 8, zpair, spair);
                            c1[4 * v + 3] = nib_pair_w(words[4 + v] >> 12, zpair, spair);
                        }
                        const uint32_t acol =
                            lane_base + static_cast<uint32_t>(kTcACol0 + (s * kTcGPBMax + gk) * kTcACols);
                        tc_st16(acol, c0);
                        tc_st16(acol + 16, c1);
                        tc_wait_st();
                        if (tid == 32 * 4 * set) tc_stamp(a.trace, q, 3);
                        tc_fence_before();
                        mbar_arrive(&in_full[s]);
                        if (tid == 32 * 4 * set) tc_stamp(a.trace, q, 4);
                    }
                    mine.next();
                    if (gk == G::GPB - 1) kq.next();
                }
                mbar_arrive(&sz_empty[sb]);
                zq.next();
            }
        } else {
            // ---------------- drain warps: the item's accumulator, 16 columns (8 tokens) at a time ----------------
            RingPos<kTcNACC> dq;
            uint32_t q_end = 0;
            for (ItemIter itr(a.segs, nitems, a.tiles); itr.valid() && ok; itr.next(a.segs)) {
                const int4 sg = itr.sg;
                const int t = itr.t;
                const int T = sg.z;
                const int N = seg_cols(T);
                q_end += G::NG;
                const bool stamp = tid == kTcDrainWarp0 * 32;
                if (stamp) tc_stamp(a.trace, q_end - 1, 5);
                if (!(ok = wwait(&acc_full[dq.i], dq.ph))) break;
                if (stamp) tc_stamp(a.trace, q_end - 1, 6);
                tc_fence_after();
                const uint32_t ta = lane_base + static_cast<uint32_t>(dq.i * kTcDCols);
                const int j = r & 15;
                const int i_loc = 8 * (r >> 4) + (j & 7);  // gate/up: intermediate index inside the tile's 64
                uint8_t* hst = GATEUP ? a.hstage + static_cast<size_t>(sg.w) * a.I * 2 + static_cast<size_t>(t) * N * 128
                                      : nullptr;
                for (int c = 0; c * 16 < N; ++c) {
                    float dv[16];
                    tc_ld16(ta + 16 * c, dv);
                    tc_wait_ld();
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const int tok = 8 * c + e;
                        if (tok < T) {
                            const float y = dv[2 * e] + dv[2 * e + 1];
                            if (GATEUP) {
                                const float up = __shfl_down_sync(0xffffffffu, y, 8);
                                if (j < 8) {
                                    uint16_t hi, lo;
                                    split_f16(silu_f(y) * up, hi, lo, a.err);
                                    *reinterpret_cast<uint16_t*>(hst + stage_off(2 * tok, i_loc)) = hi;
                                    *reinterpret_cast<uint16_t*>(hst + stage_off(2 * tok + 1, i_loc)) = lo;
                                }
                            } else {
                                const int ps = a.pair_src[sg.y + tok];
                                const int src = ps >> 5, k = ps & 31;
                                float* dst =
                                    a.ep.eout[src / a.n] + (static_cast<size_t>(src % a.n) * (a.topk + 1) + k) * a.H;
                                dst[128 * t + r] = y;
                            }
                        }
                    }
                }
                tc_fence_before();
                mbar_arrive(&acc_empty[dq.i]);
                dq.next();
                if (stamp) tc_stamp(a.trace, q_end - 1, 7);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kTcMmaWarp) {
        tc_fence_after();
        tc_dealloc(tmem, 512);
    }
    if (!GATEUP && a.ep.world > 1) __threadfence_system();
}

// ---- staging of the gate/up operands: each large segment's token rows as hi/lo fp16
// tiles; each small segment's token rows as digit records (one per pair) ----
struct XStageArgs {
    const int4* segs;
    const int* work;
    const int* pair_src;
    int n, K;
    EpView ep;          // the normalised MoE inputs of every source rank (peer memory: plain loads)
    uint8_t* stage;
    uint8_t* xrec;      // small segments: [pairs] records of vrec_bytes(K) bytes
    uint32_t* err;
};

__global__ void __launch_bounds__(256) b_xstage_kernel(const __grid_constant__ XStageArgs a) {
    pdl_wait();
    const int nseg = a.work[0], nall = a.work[3];
    pdl_launch_dependents();
    const int units = a.K / 8;
    // segments over grid.y, (token, 16-byte unit) over grid.x: every row unit is one thread
    for (int s = blockIdx.y; s < nseg; s += gridDim.y) {
        const int4 sg = a.segs[s];
        const int N = seg_cols(sg.z);
        for (int f = blockIdx.x * blockDim.x + threadIdx.x; f < sg.z * units; f += gridDim.x * blockDim.x) {
            const int tok = f / units, v = f % units;
            uint8_t* tile = a.stage + static_cast<size_t>(sg.w) * a.K * 2 + static_cast<size_t>(v >> 3) * N * 128;
            const int u = v & 7;
            const int src = a.pair_src[sg.y + tok] >> 5;
            const float4* row =
                reinterpret_cast<const float4*>(a.ep.xn[src / a.n] + static_cast<size_t>(src % a.n) * a.K + 8 * v);
            const float4 f0 = row[0], f1 = row[1];
            // the staged order inside a unit: elements [0,4,1,5,2,6,3,7]
            const float x[8] = {f0.x, f1.x, f0.y, f1.y, f0.z, f1.z, f0.w, f1.w};
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint16_t h0, l0, h1, l1;
                split_f16(x[2 * i], h0, l0, a.err);
                split_f16(x[2 * i + 1], h1, l1, a.err);
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
    // small segments: one warp per 32 elements of a token row (one half of a scale group,
    // which takes its own digit unit)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    const int halves = a.K / 32, rb = vrec_bytes(a.K), vfb = vfrag_bytes(a.K);
    for (int s = nseg + blockIdx.y; s < nall; s += gridDim.y) {
        const int4 sg = a.segs[s];
        for (int u = blockIdx.x * nw + warp; u < sg.z * halves; u += gridDim.x * nw) {
            const int tok = u / halves, k = (u % halves) * 32 + lane;
            const int src = a.pair_src[sg.y + tok] >> 5;
            const float* row = a.ep.xn[src / a.n] + static_cast<size_t>(src % a.n) * a.K;
            int8_t* vf = reinterpret_cast<int8_t*>(a.xrec + static_cast<size_t>(sg.y + tok) * rb);
            vgroup_build_half(vf, reinterpret_cast<VGroup*>(vf + vfb), k, row[k]);
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

// Whether a step of n rows per rank can hold a segment of more than kSmTok tokens (the
// tcgen05 kernels' work): a routed expert takes at most one pair per row of every rank of
// the group, the shared expert one per row of this rank.
static bool may_have_large(const Dims& d, const BatchBuffers& bb, int n) {
    if (!expert_q4_supported(d.H, d.I, d.G)) return true;
    return static_cast<int64_t>(n) * (bb.ep.world > 1 ? bb.ep.world : 1) > kSmTok;
}

int b_expert_launches(const Dims& d, const BatchBuffers& bb, int n) {
    return 1 + (expert_q4_supported(d.H, d.I, d.G) ? 2 : 0) + (may_have_large(d, bb, n) ? 2 : 0);
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
    xs.xrec = bb.xrec;
    xs.err = b.err;
    cudaError_t e = launch_kernel(lc, b_xstage_kernel, dim3(8, lc.num_sms), dim3(256), 0, xs);
    if (e != cudaSuccess) return e;
    // small segments (integer path), then the large ones (tcgen05), per projection
    const bool q4 = expert_q4_supported(d.H, d.I, d.G);
    if (q4 && (e = launch_b_experts_q4(lc, d, w, bb, b, n, true)) != cudaSuccess) return e;
    if (!may_have_large(d, bb, n)) return q4 ? launch_b_experts_q4(lc, d, w, bb, b, n, false) : cudaSuccess;
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
    a.trace = b.trace ? b.trace + kTrCta : nullptr;
    // gate/up: K = H, tiles of 8 chunks (64 gate + 64 up rows)
    a.proj_off = 0;
    a.chunk_bytes = d.gu_chunk_bytes;
    a.tiles = d.I / 64;
    a.bstage = bb.xgu;
    a.hstage = bb.xdn;
    a.wmap = *static_cast<const CUtensorMap*>(w.tm_gu);
    e = launch_tc_proj(lc, d.H, true, a);
    if (e != cudaSuccess) return e;
    if (q4 && (e = launch_b_experts_q4(lc, d, w, bb, b, n, false)) != cudaSuccess) return e;
    // down: K = I, tiles of 128 output rows
    a.proj_off = static_cast<int64_t>(d.gu_chunks) * d.gu_chunk_bytes;
    a.chunk_bytes = d.d_chunk_bytes;
    a.tiles = d.H / 128;
    a.bstage = bb.xdn;
    a.hstage = nullptr;
    a.trace = b.trace ? b.trace + kTrCta + kTcTraceSlots * kTcTraceGroups : nullptr;
    a.wmap = *static_cast<const CUtensorMap*>(w.tm_dn);
    return launch_tc_proj(lc, d.I, false, a);
}

}  // namespace dm
