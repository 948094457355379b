// dm_expert_q4.cu — routed experts of the batched decode step for small segments (at most
// kSqTok tokens of one expert), on the integer tensor-core path of the single-row MoE.
//
// Reference: parallel_moe_experts (src/core/worker_pool.mojo:383) running swiglu_forward
// (src/layers/swiglu.mojo:52) per expert over the tokens routed to it; weights in the
// asymmetric 4-bit format w = s * (q - z), group 64 along K, nibbles low first
// (quant_format.md:831-854).
//
// Why a second expert path.  A decode batch of a few rows spreads its (row, expert) pairs
// over many experts with one or two rows each.  The tcgen05 kernels expand every weight to
// fp16 in tensor memory, a cost per weight that does not shrink with the rows of a
// segment, so a one-row segment pays the full expansion for one row.  Here the nibbles go
// to mma.sync m16n8k32 (u8 x s8) as they are (one AND or shift-AND per four weights) and
// the activations as two signed 8-bit digits per element with a unit per scale group
// (q4_set_mma_tok): the work per weight is a fraction of an instruction, and each extra
// row of a segment adds only its own MMAs and group epilogue.  The kernels stream the
// expert records at the rate the copies allow.
//
// Work.  The grouping kernel lists the large segments first (segments [0, work[0]), the
// tcgen05 kernels) and the small ones after them ([work[0], work[3])) as pieces of at most
// kSqTok rows, pieces of 4 rows first, then 3, 2, 1.  The staging kernel writes each
// piece's input rows as digit records (vrec_bytes(H) bytes per pair, the pairs of a piece
// adjacent).  An item is (piece, tile):
//   gate/up  tile t = chunks 4t .. 4t + 3 (gate and up rows of intermediate indices
//            32t .. 32t + 31: one half group of the down projection's K).  Two warps per
//            chunk, each half of the chunk's sets; the partial rows meet in shared memory
//            (bounded mbarriers, no named barrier) and warp q of the group forms h =
//            SiLU(gate) * up of token q and writes the half group straight into the down
//            projection's digit record of the pair;
//   down     tile t = chunks 8t .. 8t + 7 (output rows 128t .. 128t + 127), one warp per
//            chunk; each token's rows go to the expert-output rows of its source rank
//            (peer memory in an expert-parallel group: plain stores).
// A CTA's first item is its own index; the later ones come from a counter per kernel
// (work[1], work[2], zeroed by the grouping kernel; item = grid size + count), so the CTAs
// that finish early take more.  A producer warp (one thread) takes the
// item indices two ahead and bulk-copies each item's input records (four buffers) and,
// with one more copy, its chunks (adjacent in the record) into an item slot, ahead of two
// groups of 8 consumer warps that take alternate items; every wait is bounded
// (DM_WAIT_NS, then the error bit, all roles stop, the producer waits for its copies in
// flight).
#include <cuda.h>

#include "dm_kernels.h"
#include "dm_q4mma.cuh"

namespace dm {

constexpr int kSqWarps = 16;                     // consumer warps: two groups of eight
constexpr int kSqGroups = 2;                     // consumer groups (alternate items)
constexpr int kSqGroupWarps = kSqWarps / kSqGroups;
constexpr int kSqXBufs = 2 * kSqGroups;          // input-record buffers: two per group
constexpr int kSqThreads = (kSqWarps + 1) * 32;  // + the producer warp
constexpr int kSqProdWarp = kSqWarps;
constexpr int kSqMaxSlots = 32;
constexpr int kSqSmemMax = 226 * 1024;  // dynamic + static shared memory of one CTA (1 KB spare)

template <int K, bool GATEUP>
struct SqGeom {
    using Q = Q4<K, kQ4G>;
    static constexpr int NG = K / kQ4G;
    static constexpr int CHUNK = Q::CHUNK;
    // gate/up: 4 chunks = 32 intermediate indices (one half group of the down input);
    // down: 8 chunks = 128 output rows
    static constexpr int CPI = GATEUP ? 4 : 8;
    static constexpr int WPC = kSqGroupWarps / CPI;  // warps per chunk
    static constexpr int NS = (NG + 3) / 4;          // sets of four groups per row
    static constexpr int RBY = vrec_bytes(K);        // one token's input record
    static constexpr int XB = kSqTok * RBY;          // an item's input records
    static constexpr int C_OFF = kSqXBufs * XB;      // chunk slots after the record buffers
    static constexpr int PART = GATEUP ? kSqWarps * kSqTok * 16 : 1;  // floats of the partial rows
    static constexpr int STATIC = PART * 4 + (2 * kSqMaxSlots + 2 * kSqXBufs + 2 * kSqGroups) * 8 + kSqXBufs * 32 + 256;
    static_assert(static_cast<size_t>(CPI) * CHUNK < (1u << 20), "one item's copy within an mbarrier's tx count");
    // chunk slots in item slots of CPI (an item's chunks are adjacent in its record: one bulk
    // copy), their number a multiple of kSqGroups: item slot ic % NIS then belongs to group
    // ic % 2 alone, so a warp waits for a slot's next use only after it has seen the
    // previous one complete (an mbarrier parity names phases two apart alike)
    static constexpr int NSLOT_FIT = (kSqSmemMax - STATIC - C_OFF) / CHUNK;
    static constexpr int NSLOT_CAP = NSLOT_FIT > kSqMaxSlots ? kSqMaxSlots : NSLOT_FIT;
    static constexpr int NSLOT = NSLOT_CAP / (kSqGroups * CPI) * (kSqGroups * CPI);
    static constexpr int NIS = NSLOT / CPI;           // item slots: an item's CPI chunks, one copy
    static constexpr size_t SMEM = static_cast<size_t>(C_OFF) + static_cast<size_t>(NSLOT) * CHUNK;
    static_assert(kSqGroupWarps % CPI == 0, "whole warps per chunk");
    static_assert(CHUNK % 16 == 0 && XB % 16 == 0 && RBY % 16 == 0, "bulk copy sizes");
    static_assert(NSLOT >= kSqGroups * CPI, "chunk ring: one item per group at least");
};

struct SqArgs {
    const uint8_t* experts;   // record 0 of the layer's pool
    int64_t expert_bytes, proj_off;
    const int4* segs;         // (record, first pair, tokens, -)
    int* work;                // [0] large segments, [3] all segments; [1] / [2] the gate/up and
                              // down item counters (zero at launch)
    const int* pair_src;      // (source rank * n + row) * 32 + k of each pair
    const uint8_t* xrec;      // this projection's input records, one per pair (vrec_bytes(K))
    uint8_t* hrec;            // gate/up: the down projection's input records (vrec_bytes(I))
    int n, topk, H, I;
    int tiles;                // items per segment
    EpView ep;                // down: expert outputs of each source rank
    uint64_t* trace;          // %globaltimer stamps or null: [2c] CTA c entry, [2c + 1] exit; at
                              // [2 kTrQ4MaxCtas] CTA 0: 0 after the wait, per item i < 8 of the CTA:
                              // 1 + 4i records issued, 2 + 4i chunks issued, 3 + 4i the first
                              // warp of its group has the chunks, 4 + 4i that warp is done with them
    uint32_t* err;
};

template <int N>
struct SqTok {
    static constexpr int value = N;
};

DM_DEV void sq_stamp(uint64_t* tr, int k) {
    if (tr) tr[k] = globaltimer_ns();
}

// One item as the producer hands it to a consumer group: the segment record and the tile
// (tokens 0: no more items for the group).
struct SqItem {
    int4 sg;
    int t, pad[3];
};

template <int K, bool GATEUP>
__global__ void __launch_bounds__(kSqThreads, 1) b_expert_q4_kernel(const __grid_constant__ SqArgs a) {
    using G = SqGeom<K, GATEUP>;
    extern __shared__ __align__(128) uint8_t sq_raw[];
    uint8_t* sm = sq_raw;
    __shared__ __align__(8) uint64_t cfull[G::NIS], cempty[G::NIS], xfull[kSqXBufs], xempty[kSqXBufs];
    // gate/up: a group's partial rows written (all 8 warps) / read by the h warps (all 8 arrive)
    __shared__ __align__(8) uint64_t pfull[kSqGroups], pfree[kSqGroups];
    __shared__ float s_part[G::PART];            // gate/up: [group][warp of group][token][row]
    __shared__ SqItem s_item[kSqXBufs];          // the item whose records buffer b holds
    __shared__ int s_abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int* abort_flag = &s_abort;
    uint64_t* tr = a.trace && blockIdx.x < kTrQ4MaxCtas ? a.trace : nullptr;
    uint64_t* td = a.trace && blockIdx.x == 0 ? a.trace + 2 * kTrQ4MaxCtas : nullptr;
    if (threadIdx.x == 0) {
        sq_stamp(tr, 2 * blockIdx.x);
        for (int i = 0; i < G::NIS; ++i) {
            mbar_init(&cfull[i], 1);
            mbar_init(&cempty[i], kSqGroupWarps);
        }
        for (int i = 0; i < kSqXBufs; ++i) {
            mbar_init(&xfull[i], 1);
            mbar_init(&xempty[i], kSqGroupWarps);
        }
        for (int i = 0; i < kSqGroups; ++i) {
            mbar_init(&pfull[i], kSqGroupWarps);
            mbar_init(&pfree[i], kSqGroupWarps);
        }
        mbar_fence_init();
        s_abort = 0;
    }
    __syncthreads();

    pdl_wait();  // segments, pairs and the input records come from the kernels before
    const int seg0 = a.work[0];
    const int nitems = (a.work[3] - seg0) * a.tiles;
    pdl_launch_dependents();

    if (warp == kSqProdWarp) {
        // ---- producer (one thread): items from the kernel's counter (the lowest first:
        // the grouping lists the heaviest pieces first), indices two ahead; per item its record
        // buffer (ic % 4: group ic % 2 alternates two), the item into shared memory, its
        // input records, then its chunks into the ring.  A slot is refilled once its
        // readers have arrived on its empty barrier: their generic reads are ordered before
        // the bulk copy's writes by that barrier, no proxy fence needed.  At the end each
        // group gets an item of 0 tokens ----
        if (lane == 0) {
            sq_stamp(td, 0);
            asm volatile("fence.proxy.async.global;" ::: "memory");  // records written by generic stores
            int* counter = a.work + (GATEUP ? 1 : 2);
            uint32_t ic = 0, nc = 0;  // items begun, items whose chunks were copied
            bool ok = true;
            // item indices two ahead, segment records one ahead: neither latency is waited for.
            // A CTA's first item is its own index; the counter hands out the items from the
            // grid size on (no atomic round trip before the first copy)
            const int grid = static_cast<int>(gridDim.x);
            int item = static_cast<int>(blockIdx.x);
            int nxt = grid + atomicAdd(counter, 1);
            int4 sg = item < nitems ? a.segs[seg0 + item / a.tiles] : make_int4(0, 0, 0, 0);
            while (item < nitems && ok) {
                const int nxt2 = nxt < nitems ? grid + atomicAdd(counter, 1) : nitems;
                const int4 sg_next = nxt < nitems ? a.segs[seg0 + nxt / a.tiles] : sg;
                const int t = item % a.tiles;
                const int T = max(1, min(sg.z, kSqTok));
                const uint32_t xb = ic % kSqXBufs, is = ic % G::NIS;
                if (!(ok = mbar_wait_bounded(&xempty[xb], ((ic / kSqXBufs) & 1u) ^ 1u, a.err, abort_flag))) break;
                s_item[xb].sg = make_int4(sg.x, sg.y, T, 0);
                s_item[xb].t = t;
                mbar_arrive_expect_tx(&xfull[xb], static_cast<uint32_t>(T * G::RBY));
                bulk_g2s(sm + xb * G::XB, a.xrec + static_cast<size_t>(sg.y) * G::RBY, static_cast<uint32_t>(T * G::RBY),
                         &xfull[xb]);
                if (ic < 8) sq_stamp(td, 1 + 4 * ic);
                if (!(ok = mbar_wait_bounded(&cempty[is], ((ic / G::NIS) & 1u) ^ 1u, a.err, abort_flag))) {
                    ++ic;  // the records' copy above is in flight: drained below
                    break;
                }
                ++nc;
                const uint8_t* rec = a.experts + static_cast<int64_t>(sg.x) * a.expert_bytes + a.proj_off +
                                     static_cast<int64_t>(t) * G::CPI * G::CHUNK;
                mbar_arrive_expect_tx(&cfull[is], static_cast<uint32_t>(G::CPI * G::CHUNK));
                bulk_g2s(sm + G::C_OFF + is * G::CPI * G::CHUNK, rec, static_cast<uint32_t>(G::CPI * G::CHUNK), &cfull[is]);
                if (ic < 8) sq_stamp(td, 2 + 4 * ic);
                ++ic;
                item = nxt;
                nxt = nxt2;
                sg = sg_next;
            }
            // the end marker of each group (after a failure the consumers' waits return at once)
            for (int g = 0; g < kSqGroups && ok; ++g, ++ic) {
                const uint32_t xb = ic % kSqXBufs;
                if (!(ok = mbar_wait_bounded(&xempty[xb], ((ic / kSqXBufs) & 1u) ^ 1u, a.err, abort_flag))) break;
                s_item[xb].sg = make_int4(0, 0, 0, 0);
                mbar_arrive(&xfull[xb]);
            }
            // every copy this thread issued has landed before the CTA may leave (bounded)
            for (uint32_t u = nc > G::NIS ? nc - G::NIS : 0; u < nc; ++u)
                mbar_wait_bounded(&cfull[u % G::NIS], (u / G::NIS) & 1u, a.err, nullptr);
            for (uint32_t u = ic > kSqXBufs ? ic - kSqXBufs : 0; u < ic; ++u)
                mbar_wait_bounded(&xfull[u % kSqXBufs], (u / kSqXBufs) & 1u, a.err, nullptr);
        }
    } else {
        // ---- consumer group cg = warp / 8 takes the CTA's items cg, cg + 2, ... until an
        // item of 0 tokens or a failed wait.  The warps of a group meet only at mbarriers
        // with bounded waits (no named barrier): a warp that leaves early makes the others'
        // waits run out, never hang ----
        auto wwait = [&](uint64_t* bar, uint32_t parity) -> bool {
            return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, a.err, abort_flag));
        };
        const int cg = warp / kSqGroupWarps, wl = warp % kSqGroupWarps;
        const int j = wl / G::WPC, sub = wl % G::WPC;  // chunk of the item, part of its sets
        const int r = lane >> 2;
        float* part = s_part + (GATEUP ? cg * kSqGroupWarps * kSqTok * 16 : 0);
        for (uint32_t ic = cg, kg = 0;; ic += kSqGroups, ++kg) {  // kg: the group's item count
            const uint32_t xb = ic % kSqXBufs;
            if (!wwait(&xfull[xb], (ic / kSqXBufs) & 1u)) break;
            const SqItem it = s_item[xb];
            const int4 sg = it.sg;
            const int T = sg.z;
            if (T == 0) break;
            const int t = it.t;
            const uint32_t is = ic % G::NIS;
            // down: lane q < T holds token q's pair source (loaded while the chunk lands)
            const int my_src = !GATEUP && lane < T ? a.pair_src[sg.y + lane] : 0;
            bool ok = wwait(&cfull[is], (ic / G::NIS) & 1u);
            // gate/up: the group's previous partial rows have been read (bounded)
            if (GATEUP && kg > 0) ok = wwait(&pfree[cg], (kg - 1) & 1u) && ok;
            const bool stamp = wl == 0 && lane == 0 && ic < 8;
            if (stamp) sq_stamp(td, 3 + 4 * ic);
            const uint8_t* chunk = sm + G::C_OFF + (is * G::CPI + j) * G::CHUNK;
            const uint8_t* xr = sm + xb * G::XB;
            const int row = 16 * (t * G::CPI + j) + r;  // down: output row of lanes r (and r + 8)
            // tokens q0 .. q0 + TT - 1 (those < T count): the chunk's sets of this warp, the
            // rows summed over the four lanes of each, then the gate/up partial rows into
            // shared memory or the down rows into the expert outputs
            auto tokens = [&](auto tt, int q0) {
                constexpr int TT = decltype(tt)::value;
                float ya[TT], yb[TT];
#pragma unroll
                for (int q = 0; q < TT; ++q) ya[q] = yb[q] = 0.0f;
                if (ok) {
#pragma unroll 1
                    for (int S = sub; S < G::NS; S += G::WPC)
                        q4_set_mma_tok<K, TT>(chunk, xr + q0 * G::RBY, S, G::NG - 4 * S < 4 ? G::NG - 4 * S : 4, lane,
                                              ya, yb);
                }
                int src[TT];
#pragma unroll
                for (int q = 0; q < TT; ++q) {
                    ya[q] += __shfl_xor_sync(0xffffffffu, ya[q], 1);
                    yb[q] += __shfl_xor_sync(0xffffffffu, yb[q], 1);
                    ya[q] += __shfl_xor_sync(0xffffffffu, ya[q], 2);
                    yb[q] += __shfl_xor_sync(0xffffffffu, yb[q], 2);
                    src[q] = __shfl_sync(0xffffffffu, my_src, (q0 + q) & 31);
                }
                if ((lane & 3) != 0) return;
#pragma unroll
                for (int q = 0; q < TT; ++q) {
                    if (q0 + q >= T) break;
                    if (GATEUP) {
                        part[(wl * kSqTok + q0 + q) * 16 + r] = ya[q];
                        part[(wl * kSqTok + q0 + q) * 16 + r + 8] = yb[q];
                    } else if (ok) {
                        const int src_row = src[q] >> 5, k = src[q] & 31;
                        float* dst = a.ep.eout[src_row / a.n] +
                                     (static_cast<size_t>(src_row % a.n) * (a.topk + 1) + k) * a.H;
                        dst[row] = ya[q];
                        dst[row + 8] = yb[q];
                    }
                }
            };
            if (T == 1) {
                tokens(SqTok<1>{}, 0);
            } else {
#pragma unroll 1
                for (int q0 = 0; q0 < T; q0 += 2) tokens(SqTok<2>{}, q0);
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&cempty[is]);
                mbar_arrive(&xempty[xb]);
                if (GATEUP) mbar_arrive(&pfull[cg]);  // this warp's partial rows are written
            }
            if (stamp) sq_stamp(td, 4 + 4 * ic);
            if (GATEUP) {
                // warp q of the group: token q's h over the tile's 32 intermediate indices
                // (one half group of the down input): lane l = index 32 t + l, chunk l / 8
                if (wl < T && wwait(&pfull[cg], kg & 1u)) {
                    const int q = wl, cj = lane >> 3, kr = lane & 7;
                    float gt = 0.0f, up = 0.0f;
#pragma unroll
                    for (int u = 0; u < G::WPC; ++u) {
                        gt += part[((cj * G::WPC + u) * kSqTok + q) * 16 + kr];
                        up += part[((cj * G::WPC + u) * kSqTok + q) * 16 + 8 + kr];
                    }
                    int8_t* vf = reinterpret_cast<int8_t*>(a.hrec + static_cast<size_t>(sg.y + q) * vrec_bytes(a.I));
                    vgroup_build_half(vf, reinterpret_cast<VGroup*>(vf + vfrag_bytes(a.I)), 32 * t + lane,
                                      silu_f(gt) * up);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&pfree[cg]);  // (warps q >= T read nothing)
            }
        }
    }
    if (!GATEUP && a.ep.world > 1) __threadfence_system();
    if (tr) {
        __syncthreads();
        if (threadIdx.x == 0) sq_stamp(tr, 2 * blockIdx.x + 1);
    }
}

// gate/up takes K = H, down K = I; one item slot per group must fit the shared memory
// (gate/up items of K = 4096 and down items of K = 2048 do not)
#define DM_SQ_GU_INSTANCES(X) X(256) X(512) X(1024) X(2048)
#define DM_SQ_DN_INSTANCES(X) X(128) X(256) X(512) X(1024)

size_t q4_vrec_bytes(int K) { return static_cast<size_t>(vrec_bytes(K)); }

bool expert_q4_supported(int H, int I, int G) {
    const bool h_ok = H == 256 || H == 512 || H == 1024 || H == 2048;
    const bool i_ok = I == 128 || I == 256 || I == 512 || I == 1024;
    return G == kQ4G && h_ok && i_ok;
}

cudaError_t b_experts_q4_set_attrs() {
    cudaError_t e = cudaSuccess;
#define DM_SQ_ATTR_GU(KK)                                                                                       \
    if (e == cudaSuccess)                                                                                       \
        e = cudaFuncSetAttribute(b_expert_q4_kernel<KK, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                 static_cast<int>(SqGeom<KK, true>::SMEM));
#define DM_SQ_ATTR_DN(KK)                                                                                       \
    if (e == cudaSuccess)                                                                                       \
        e = cudaFuncSetAttribute(b_expert_q4_kernel<KK, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,   \
                                 static_cast<int>(SqGeom<KK, false>::SMEM));
    DM_SQ_GU_INSTANCES(DM_SQ_ATTR_GU)
    DM_SQ_DN_INSTANCES(DM_SQ_ATTR_DN)
#undef DM_SQ_ATTR_GU
#undef DM_SQ_ATTR_DN
    return e;
}

cudaError_t launch_b_experts_q4(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& bb,
                                const Buffers& b, int n, bool gateup) {
    if (!expert_q4_supported(d.H, d.I, d.G)) return cudaErrorInvalidValue;
    SqArgs a{};
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
    a.trace = b.trace && lc.num_sms <= kTrQ4MaxCtas ? b.trace + kTrQ4 + (gateup ? 0 : kTrQ4Slots) : nullptr;
    const dim3 grid(lc.num_sms), block(kSqThreads);
    if (gateup) {
        a.proj_off = 0;
        a.xrec = bb.xrec;
        a.hrec = bb.hrec;
        a.tiles = d.I / 32;
#define DM_SQ_LAUNCH_GU(KK) \
    if (d.H == KK) return launch_kernel(lc, b_expert_q4_kernel<KK, true>, grid, block, SqGeom<KK, true>::SMEM, a);
        DM_SQ_GU_INSTANCES(DM_SQ_LAUNCH_GU)
#undef DM_SQ_LAUNCH_GU
    } else {
        a.proj_off = static_cast<int64_t>(d.gu_chunks) * d.gu_chunk_bytes;
        a.xrec = bb.hrec;
        a.hrec = nullptr;
        a.tiles = d.H / 128;
#define DM_SQ_LAUNCH_DN(KK) \
    if (d.I == KK) return launch_kernel(lc, b_expert_q4_kernel<KK, false>, grid, block, SqGeom<KK, false>::SMEM, a);
        DM_SQ_DN_INSTANCES(DM_SQ_LAUNCH_DN)
#undef DM_SQ_LAUNCH_DN
    }
    return cudaErrorInvalidValue;
}

}  // namespace dm
