// dm_attn.cu — gated-attention decode step over a paged bf16 KV cache (sm_100a).
//
// Semantics of reference forward_attention_qwen36 (src/layers/attention.mojo:219-435) for
// the token at position `pos`, with the KV cache of LayerKVCache (kv_cache.mojo:302-375):
//   q, gate = halves of q_proj (first Hq*D rows q, next Hq*D rows gate)
//   per-head RMSNorm of q and k with q_norm / k_norm            (attention.mojo:282-316)
//   partial RoPE on the first rotary_dim = int(D * factor) dims, rotate-half pairs
//   (i, i + rotary_dim/2), inv_freq_i = 1 / theta^(2i / rotary_dim)   (:318-354)
//   k, v rounded once to bf16 and appended at pos (pos == current length)
//   softmax(q k^T / sqrt(D)) over positions [0, pos] of the KV head (GQA: query head h
//   reads KV head h / (Hq / Hkv)), output * sigmoid(gate)          (:356-427)
//
// Grid (Hkv, nsplit): CTA (g, s) normalises and rotates the Hq/Hkv query heads of KV head
// g, scores its share of the positions (a whole number of 16-token pages) for all of them
// at once, and writes an unnormalised partial (max, sum, acc[D]) per head; the last CTA
// of KV head g (atomic counter) merges the partials and applies the output gate.  The
// current token's k/v come from shared memory, so the append by CTA (g, 0) never races
// with the reads of the other CTAs, which only touch positions < pos.
#include <cooperative_groups.h>
#include <cuda.h>

#include "dm_common.cuh"
#include "dm_kernels.h"

namespace dm {

constexpr int kAttnCluster = 4;  // splits merged on chip per cluster
constexpr int kAT = 512;          // threads of a decode-attention CTA
constexpr int kAW = kAT / 32;     // its warps

struct AttnArgs {
    const float* qg;          // [2*Hq*D]
    const float* kvnew;       // [2*Hkv*D] k then v (raw projections)
    const uint16_t* q_norm;   // [D]
    const uint16_t* k_norm;   // [D]
    uint16_t* kv;             // layer base [num_pages][2][Hkv][16][D]
    const int* page_table;    // [max_pages] for the slot
    const int* pos;
    int Hq, Hkv, rot_dim, max_pages, num_pages, nsplit, cap;
    float theta, eps;
    float* part;              // [Hq][kMaxSplits][D+2]
    float* out;               // [Hq*D]
    unsigned* counters;       // [Hkv]
    const float2* rope;       // [capacity][rot_dim/2] (cos, sin)
    uint64_t* trace;          // phase stamps (CTA (0, last split), thread 0) or null
    uint64_t* cta_trace;      // per-CTA stamps (kTrCtaSlots per CTA, thread 0) or null
    uint64_t* kt;             // launch timeline record or null
    uint32_t* err;
    // 2-D tiled view of the whole KV arena (all attention layers): columns D, rows
    // [att][page][K|V][Hkv][16]; boxes of 16 rows x 64 columns, 128-byte swizzle
    CUtensorMap kv_map;
    int kv_row0;              // first row of this layer
    // batched launch (grid.z = batch rows): row b attends for sequence slots[b]; page table
    // and pos advance by the slot, the q/k/v inputs, partials, outputs and counters by the
    // row.  slots == nullptr: one sequence.
    const int* slots;
    int pt_ss, cnt_bs;
    size_t qg_bs, kvn_bs, part_bs, out_bs;
};

// RoPE table [capacity][rot_dim / 2] of (cos, sin) of fp32(pos) * inv_freq_i with
// inv_freq_i = 1 / theta^(2i / rot_dim) (reference attention.mojo:318-354), filled once
// per context so the decode step never evaluates trigonometry of large arguments.
__global__ void rope_table_kernel(float2* tab, int capacity, int rot_dim, float theta) {
    const int half = rot_dim / 2;
    const int64_t n = static_cast<int64_t>(capacity) * half;
    for (int64_t k = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; k < n;
         k += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int p = static_cast<int>(k / half), i = static_cast<int>(k % half);
        const float inv_freq = 1.0f / powf(theta, static_cast<float>(2 * i) / static_cast<float>(rot_dim));
        const float ang = static_cast<float>(p) * inv_freq;
        tab[k] = make_float2(cosf(ang), sinf(ang));
    }
}

cudaError_t launch_rope_table(cudaStream_t st, float2* tab, int capacity, int rot_dim, float theta) {
    int blocks = (capacity * (rot_dim / 2) + 255) / 256;
    if (blocks > 4096) blocks = 4096;
    if (blocks < 1) blocks = 1;
    rope_table_kernel<<<blocks, 256, 0, st>>>(tab, capacity, rot_dim, theta);
    return cudaGetLastError();
}

constexpr int kAttnStages = 6;   // K+V page tiles in flight per CTA (one sequence)
constexpr int kMaxPagesPerSplit = 256;  // page ids staged in shared memory

// One KV page (16 tokens, one head) per ring stage: the K tile then the V tile, each as
// D/64 column chunks of [16 rows][128 bytes] written by the tensor-map copy with the
// 128-byte swizzle (16-byte unit u of row r lands at unit u ^ (r & 7)), so the 8 rows an
// ldmatrix reads at one column fall in 8 distinct bank groups.
template <int D>
struct AttnGeom {
    static constexpr int CHUNK = kPageTokens * 128;      // one 64-column chunk of a tile
    static constexpr int TILE = (D / 64) * CHUNK;        // K (or V) of one page
    static constexpr int STAGE = 2 * TILE;
    static_assert(D % 64 == 0, "whole 128-byte column chunks");
};
// Byte offset of (row, col) inside a staged tile.
template <int D>
DM_DEV uint32_t kv_tile_off(int row, int col) {
    return (col >> 6) * AttnGeom<D>::CHUNK + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4) + (col & 7) * 2;
}
// 2-D tiled tensor-map load (no multicast) completing on an mbarrier.
DM_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// mma.sync m16n8k16, bf16 inputs, fp32 accumulate (fragment layouts of the PTX ISA:
// g = lane / 4, t = lane % 4; A a0 = A[g][2t..2t+1], a1 = A[g+8][..], a2 = A[g][2t+8..],
// a3 = A[g+8][2t+8..]; B b0 = B[2t..2t+1][g], b1 = B[2t+8..2t+9][g];
// C c0 = C[g][2t], c1 = C[g][2t+1], c2 = C[g+8][2t], c3 = C[g+8][2t+1]).
DM_DEV void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
DM_DEV void ldsm_x2(uint32_t& r0, uint32_t& r1, const void* row_addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r0), "=r"(r1)
                 : "r"(smem_u32(row_addr)));
}
DM_DEV void ldsm_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* row_addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(row_addr)));
}
DM_DEV void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* row_addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(smem_u32(row_addr)));
}
// all four A registers (rows g and g + 8)
DM_DEV void mma_bf16_16816_full(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
DM_DEV uint32_t pack_bf16x2(uint16_t lo, uint16_t hi) { return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16); }

// ---- per-CTA preparation of the new token (shared by the decode kernels) ---------------
// q heads of KV group g, new k, new v: one parallel load, per-head RMSNorm (q_norm / k_norm)
// and partial RoPE in fp32 (norm weights and the RoPE row staged by the caller), then k, v
// rounded to bf16 (cache format) and q split into hi + lo bf16 terms for the tensor cores.
// All NT threads of the CTA take part; ends with a barrier.
template <int D, int GRP, int NT>
DM_DEV void attn_prepare(const float* qsrc, const float* ksrc, const float* vsrc, const float* qn_s, const float* kn_s,
                         const float2* cs_s, int rot_dim, float eps, float (*qsm)[D + 4], float* knew, float* vnew,
                         uint16_t* kbits, uint16_t* vbits, uint16_t (*qh)[D + 8], uint16_t (*ql)[D + 8]) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    {
        constexpr int QPT = (GRP * D + NT - 1) / NT, KPT = (D + NT - 1) / NT;
        float qv[QPT], kv[KPT], vv[KPT];
#pragma unroll
        for (int i = 0; i < QPT; ++i) qv[i] = tid + NT * i < GRP * D ? qsrc[tid + NT * i] : 0.0f;
#pragma unroll
        for (int i = 0; i < KPT; ++i) {
            const int d = tid + NT * i;
            kv[i] = d < D ? ksrc[d] : 0.0f;
            vv[i] = d < D ? vsrc[d] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < QPT; ++i)
            if (tid + NT * i < GRP * D) qsm[(tid + NT * i) / D][(tid + NT * i) % D] = qv[i];
#pragma unroll
        for (int i = 0; i < KPT; ++i) {
            const int d = tid + NT * i;
            if (d < D) {
                knew[d] = kv[i];
                vnew[d] = vv[i];
            }
        }
    }
    __syncthreads();
    for (int hh = warp; hh < GRP + 1; hh += NT / 32) {
        float* v = hh < GRP ? qsm[hh] : knew;
        const float* wn = hh < GRP ? qn_s : kn_s;
        float ss = 0.0f;
        for (int d = lane; d < D; d += 32) ss = fmaf(v[d], v[d], ss);
        ss = warp_sum(ss);
        const float rs = 1.0f / sqrtf(ss / static_cast<float>(D) + eps);
        for (int d = lane; d < D; d += 32) v[d] = v[d] * rs * wn[d];
        __syncwarp();
        const int half = rot_dim / 2;
        for (int i = lane; i < half; i += 32) {
            const float2 c = cs_s[i];
            const float x0 = v[i], x1 = v[i + half];
            v[i] = x0 * c.x - x1 * c.y;
            v[i + half] = x0 * c.y + x1 * c.x;
        }
        __syncwarp();
    }
    __syncthreads();
    for (int d = tid; d < D; d += NT) {
        kbits[d] = f32_to_bf16(knew[d]);
        vbits[d] = f32_to_bf16(vnew[d]);
    }
    for (int i = tid; i < GRP * D; i += NT) {
        const float q = qsm[i / D][i % D];
        const uint16_t hi = f32_to_bf16(q);
        qh[i / D][i % D] = hi;
        ql[i / D][i % D] = f32_to_bf16(q - bf16_to_f32(hi));
    }
    __syncthreads();
}

// Split-K ("flash-decoding") decode attention over the paged bf16 KV cache.
// Grid (Hkv, nsplit), clusters of kAttnCluster splits, kAT threads, one CTA per SM.
//   pre-wait  page ids of the split, every page of the split (up to kAttnStages) in
//             flight as per-row bulk copies into padded shared rows, norm weights and the
//             RoPE row staged
//   post-wait q heads of the group, new k, v: per-head RMSNorm + RoPE (fp32), k/v rounded
//             to bf16, appended at pos by split 0 and patched into the staged page
//   scores    tensor cores: S = Q K^T with q = q_hi + q_lo (two bf16 terms, fp32
//             accumulation; K is bf16), one warp per 8-token n-tile
//   softmax   per head over the batch, online across batches (max shift, expf)
//   P V       tensor cores: O += (p_hi + p_lo) V, each warp 16 output dims
//   merge     splits of a cluster through distributed shared memory, then the cluster
//             partials of a head by the CTAs of the last cluster to finish, with the
//             sigmoid output gate (reference attention.mojo:219-435 in decode form).
// NB = pages scored per batch, ST = ring stages: NB == ST (one sequence: every page of a
// split in flight at once) or NB < ST, so that ST - NB pages load while a batch is scored.
template <int D, int GRP, int NB, int ST>
__global__ void __launch_bounds__(kAT, 1) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
    static_assert(NB >= 1 && NB <= ST && ST % NB == 0, "batch of whole ring stages");
    constexpr int kAttnStages = ST;
    using AG = AttnGeom<D>;
    static_assert(GRP <= 8, "heads of a KV group are rows 0..7 of the m16 tile");
    extern __shared__ __align__(1024) uint8_t ring_raw[];
    // the swizzled tiles need 1024-byte aligned stages (the launch adds the slack)
    uint8_t* ring = ring_raw + ((1024u - (smem_u32(ring_raw) & 1023u)) & 1023u);
    __shared__ __align__(8) uint64_t bar[kAttnStages];
    constexpr int QST = D + 4;  // fp32 q rows (norm / RoPE)
    __shared__ __align__(16) float qsm[GRP][QST];
    constexpr int QBS = D + 8;  // bf16 q rows: 8 rows of an A fragment hit distinct banks
    __shared__ __align__(16) uint16_t qh[GRP][QBS], ql[GRP][QBS];
    constexpr int NT = NB * kPageTokens;  // tokens of a full batch
    constexpr int PBS = NT + 8;
    __shared__ __align__(16) uint16_t ph[GRP][PBS], pl[GRP][PBS];
    __shared__ __align__(16) float knew[D], vnew[D];
    __shared__ __align__(16) uint16_t kbits[D], vbits[D];
    __shared__ float sc[GRP][NT];
    __shared__ float m_run[GRP], l_run[GRP], scale[GRP];
    __shared__ int last_flag;
    const int g = blockIdx.x, s = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int bz = blockIdx.z;
    const int slot = a.slots ? a.slots[bz] : 0;  // host-written before the step
    const float* qg_in = a.qg + bz * a.qg_bs;
    const float* kvnew_in = a.kvnew + bz * a.kvn_bs;
    const int* page_table = a.page_table + slot * a.pt_ss;
    float* part_out = a.part + bz * a.part_bs;
    float* attn_out = a.out + bz * a.out_bs;
    unsigned* counters = a.counters + bz * a.cnt_bs;
    const int fg = lane >> 2, ft = lane & 3;  // fragment row / column-pair of this lane

    uint64_t* tr = (tid == 0 && g == 0 && s == gridDim.y - 1) ? a.trace : nullptr;
    uint64_t* ct = (tid == 0 && a.cta_trace) ? a.cta_trace + (s * gridDim.x + g) * kTrCtaSlots : nullptr;
    trace_stamp(tr, 0);
    trace_stamp(ct, 0);
    kt_start(a.kt);
    // positions < pos were written by earlier steps and the page table is fixed: the
    // range of this split and its page tiles do not depend on the previous kernel
    const int pos = a.pos[slot];
    const int n_tok = pos + 1;
    const int capacity = a.max_pages * kPageTokens;
    const bool in_range = pos >= 0 && pos < capacity;
    // pages spread evenly over the splits (every split gets floor or ceil of the mean)
    const int n_pg = in_range ? (n_tok + kPageTokens - 1) / kPageTokens : 0;
    const int pg0 = static_cast<int>(static_cast<long long>(s) * n_pg / a.nsplit);
    const int pg1 = static_cast<int>(static_cast<long long>(s + 1) * n_pg / a.nsplit);
    const int np = pg1 - pg0;
    const int t0 = pg0 * kPageTokens;
    const int t1 = min(n_tok, pg1 * kPageTokens);
    __shared__ int pages[kMaxPagesPerSplit];
    for (int i = tid; i < np && i < kMaxPagesPerSplit; i += kAT) pages[i] = page_table[pg0 + i];
    if (tid == 0) {
        for (int i = 0; i < kAttnStages; ++i) mbar_init(&bar[i], 1);
        mbar_fence_init();
    }
    __syncthreads();
    // page i of the split into its ring stage: K then V, D/64 tensor-map boxes each, all
    // issued by lane 0 of warp 0
    auto issue = [&](int i) {
        const int slot = i % kAttnStages;
        const int page = i < kMaxPagesPerSplit ? pages[i] : page_table[pg0 + i];
        const bool good = page >= 0 && page < a.num_pages;
        if (lane == 0) {
            if (good) {
                mbar_arrive_expect_tx(&bar[slot], 2 * kPageTokens * D * 2);
                uint8_t* st = ring + static_cast<size_t>(slot) * AG::STAGE;
#pragma unroll
                for (int kv = 0; kv < 2; ++kv) {
                    const int y = a.kv_row0 + ((page * 2 + kv) * a.Hkv + g) * kPageTokens;
#pragma unroll
                    for (int j = 0; j < D / 64; ++j) tma_load_2d(st + kv * AG::TILE + j * AG::CHUNK, &a.kv_map, 64 * j, y, &bar[slot]);
                }
            } else {
                raise_error(a.err, DM_DEVERR_PAGE);
                mbar_arrive(&bar[slot]);  // no copy: the tile is left as is and masked below
            }
        }
    };
    if (warp == 0)
        for (int i = 0; i < np && i < kAttnStages; ++i) issue(i);
    if (tid < GRP) {
        m_run[tid] = -INFINITY;
        l_run[tid] = 0.0f;
    }
    __shared__ float qn_s[D], kn_s[D];
    __shared__ float2 cs_s[D / 2];
    for (int i = tid; i < D; i += kAT) {
        qn_s[i] = bf16_to_f32(a.q_norm[i]);
        kn_s[i] = bf16_to_f32(a.k_norm[i]);
    }
    if (in_range)
        for (int i = tid; i < a.rot_dim / 2; i += kAT) cs_s[i] = a.rope[static_cast<size_t>(pos) * (a.rot_dim / 2) + i];
    trace_stamp(tr, 1);
    pdl_wait();
    kt_ready(a.kt);
    trace_stamp(tr, 2);
    trace_stamp(ct, 1);
    if (!in_range) {  // no room: report, touch nothing
        if (tid == 0 && s == 0) raise_error(a.err, DM_DEVERR_CAPACITY);
        kt_end(a.kt);
        return;
    }

    const float sm_scale = 1.0f / sqrtf(static_cast<float>(D));
    attn_prepare<D, GRP, kAT>(qg_in + static_cast<size_t>(g * GRP) * D, kvnew_in + static_cast<size_t>(g) * D,
                              kvnew_in + static_cast<size_t>(a.Hkv + g) * D, qn_s, kn_s, cs_s, a.rot_dim, a.eps, qsm,
                              knew, vnew, kbits, vbits, qh, ql);
    __syncthreads();
    pdl_launch_dependents();
    trace_stamp(tr, 3);

    // ---- append at pos (one CTA per KV head) ----
    if (s == 0) {
        const int page = page_table[pos / kPageTokens];
        if (page < 0 || page >= a.num_pages) {
            if (tid == 0) raise_error(a.err, DM_DEVERR_PAGE);
        } else {
            uint16_t* kd = a.kv + ((static_cast<size_t>(page) * 2 + 0) * a.Hkv + g) * kPageTokens * D +
                           static_cast<size_t>(pos % kPageTokens) * D;
            uint16_t* vd = a.kv + ((static_cast<size_t>(page) * 2 + 1) * a.Hkv + g) * kPageTokens * D +
                           static_cast<size_t>(pos % kPageTokens) * D;
            for (int d = tid; d < D; d += kAT) {
                kd[d] = kbits[d];
                vd[d] = vbits[d];
            }
        }
    }

    // output accumulators: warp w owns output dims [16w, 16w + 16) (two n8 tiles) while
    // 16w < D; c0, c1 of tile u are head fg, dims 16w + 8u + 2ft, +1
    const bool pv_on = 16 * warp < D;
    float oacc[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
    const int ip_new = pos / kPageTokens - pg0;  // page of the split holding pos, if any

    for (int b0 = 0; b0 < np; b0 += NB) {
        const int nb = min(NB, np - b0);
        unsigned okm = 0;
        for (int i = 0; i < nb; ++i)
            if (mbar_wait_bounded(&bar[(b0 + i) % kAttnStages], ((b0 + i) / kAttnStages) & 1, a.err, nullptr))
                okm |= 1u << i;
        uint64_t* trp = (tr && b0 == 0) ? tr + 40 : nullptr;
        trace_stamp(trp, 0);
        // the staged copy of the page holding pos predates the append: patch its row
        if (ip_new >= b0 && ip_new < b0 + nb) {
            uint8_t* st = ring + static_cast<size_t>(ip_new % kAttnStages) * AG::STAGE;
            const int r = pos % kPageTokens;
            for (int d = tid; d < D; d += kAT) {
                *reinterpret_cast<uint16_t*>(st + kv_tile_off<D>(r, d)) = kbits[d];
                *reinterpret_cast<uint16_t*>(st + AG::TILE + kv_tile_off<D>(r, d)) = vbits[d];
            }
        }
        __syncthreads();
        // scores: warp w < 2 nb takes n-tile w (tokens 8w..8w+7 of the batch)
        if (warp < 2 * nb) {
            const int pi = warp >> 1;  // page of the batch
            const uint8_t* kt = ring + static_cast<size_t>((b0 + pi) % kAttnStages) * AG::STAGE;
            // ldmatrix x2 row addresses: lanes 0-7 tokens of k-columns 0-7, lanes 8-15 of 8-15
            const int krow = 8 * (warp & 1) + (lane & 7), kcol = 8 * ((lane >> 3) & 1);
            float ch[4] = {0.0f, 0.0f, 0.0f, 0.0f}, cl[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const bool arow = fg < GRP;
#pragma unroll 4
            for (int ks = 0; ks < D / 16; ++ks) {
                uint32_t b0r, b1r;
                ldsm_x2(b0r, b1r, kt + kv_tile_off<D>(krow, 16 * ks + kcol));
                const int c0 = 16 * ks + 2 * ft;
                const uint32_t ah0 = arow ? *reinterpret_cast<const uint32_t*>(&qh[fg][c0]) : 0u;
                const uint32_t ah2 = arow ? *reinterpret_cast<const uint32_t*>(&qh[fg][c0 + 8]) : 0u;
                const uint32_t al0 = arow ? *reinterpret_cast<const uint32_t*>(&ql[fg][c0]) : 0u;
                const uint32_t al2 = arow ? *reinterpret_cast<const uint32_t*>(&ql[fg][c0 + 8]) : 0u;
                mma_bf16_16816(ch, ah0, ah2, b0r, b1r);
                mma_bf16_16816(cl, al0, al2, b0r, b1r);
            }
            if (arow) {
                const bool okp = (okm >> pi) & 1u;
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int tb = 8 * warp + 2 * ft + e;  // token of the batch
                    const int tpos = (pg0 + b0) * kPageTokens + tb;
                    const bool valid = okp && tpos >= t0 && tpos < t1;
                    sc[fg][tb] = valid ? (ch[e] + cl[e]) * sm_scale : -INFINITY;
                }
            }
        }
        __syncthreads();
        trace_stamp(trp, 1);
        // softmax over the batch, one warp per head, online across batches
        const int nt = nb * kPageTokens;
        for (int hh = warp; hh < GRP; hh += kAW) {
            float sv[(NT + 31) / 32];
            float mp = -INFINITY;
#pragma unroll
            for (int j = 0; j < (NT + 31) / 32; ++j) {
                const int tb = lane + 32 * j;
                sv[j] = tb < nt ? sc[hh][tb] : -INFINITY;
                mp = fmaxf(mp, sv[j]);
            }
            mp = warp_max(mp);
            const float mo = m_run[hh];
            const float mn = fmaxf(mo, mp);
            float ls = 0.0f;
#pragma unroll
            for (int j = 0; j < (NT + 31) / 32; ++j) {
                const int tb = lane + 32 * j;
                const float p = (sv[j] != -INFINITY) ? expf(sv[j] - mn) : 0.0f;
                ls += p;
                if (tb < NT) {
                    const uint16_t hi = f32_to_bf16(p);
                    ph[hh][tb] = hi;
                    pl[hh][tb] = f32_to_bf16(p - bf16_to_f32(hi));
                }
            }
            ls = warp_sum(ls);
            if (lane == 0) {
                const float f = (mo == -INFINITY) ? 0.0f : expf(mo - mn);
                scale[hh] = f;
                l_run[hh] = l_run[hh] * f + ls;
                m_run[hh] = mn;
            }
        }
        __syncthreads();
        trace_stamp(trp, 2);
        // P V: k-step = one page (16 tokens) of the batch
        if (pv_on) {
            const float f = fg < GRP ? scale[fg] : 0.0f;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                oacc[u][0] *= f;
                oacc[u][1] *= f;
            }
            const bool arow = fg < GRP;
            for (int pi = 0; pi < nb; ++pi) {
                const uint8_t* vt = ring + static_cast<size_t>((b0 + pi) % kAttnStages) * AG::STAGE + AG::TILE;
                // ldmatrix x4 .trans: matrix m = lane / 8: tokens 8(m & 1).., dims 16w + 8(m >> 1)
                const int m = lane >> 3;
                const uint8_t* vrow = vt + kv_tile_off<D>(8 * (m & 1) + (lane & 7), 16 * warp + 8 * (m >> 1));
                uint32_t v0, v1, v2, v3;
                ldsm_x4_trans(v0, v1, v2, v3, vrow);
                const int c0 = kPageTokens * pi + 2 * ft;
                const uint32_t ah0 = arow ? *reinterpret_cast<const uint32_t*>(&ph[fg][c0]) : 0u;
                const uint32_t ah2 = arow ? *reinterpret_cast<const uint32_t*>(&ph[fg][c0 + 8]) : 0u;
                const uint32_t al0 = arow ? *reinterpret_cast<const uint32_t*>(&pl[fg][c0]) : 0u;
                const uint32_t al2 = arow ? *reinterpret_cast<const uint32_t*>(&pl[fg][c0 + 8]) : 0u;
                mma_bf16_16816(oacc[0], ah0, ah2, v0, v1);
                mma_bf16_16816(oacc[0], al0, al2, v0, v1);
                mma_bf16_16816(oacc[1], ah0, ah2, v2, v3);
                mma_bf16_16816(oacc[1], al0, al2, v2, v3);
            }
        }
        __syncthreads();  // stages and scores free
        trace_stamp(trp, 3);
        if (warp == 0 && b0 + kAttnStages < np) {
            fence_proxy_async_smem();  // generic accesses of the stages before the next copies
            for (int i = b0 + kAttnStages; i < np && i < b0 + kAttnStages + nb; ++i) issue(i);
        }
    }

    trace_stamp(tr, 4);
    trace_stamp(ct, 2);
    // ---- merge 1: the kAttnCluster splits of this cluster through distributed shared
    // memory: every CTA pushes its partial into rank 0's (free) ring, rank 0 merges
    // locally and writes one partial (max, sum, acc) per head for the cluster ----
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int crank = static_cast<int>(cluster.block_rank());
    constexpr int PSZ = GRP * D + 2 * GRP;            // floats of one pushed partial
    static_assert(kAttnCluster * PSZ * 4 <= ST * AG::STAGE, "ring too small for the cluster merge");
    cluster.sync();                                    // every ring is free from here on
    float* dst0 = cluster.map_shared_rank(reinterpret_cast<float*>(ring), 0) + crank * PSZ;
    if (pv_on && fg < GRP) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int d = 16 * warp + 8 * u + 2 * ft;
            dst0[fg * D + d] = oacc[u][0];
            dst0[fg * D + d + 1] = oacc[u][1];
        }
    }
    if (tid < GRP) {
        dst0[GRP * D + tid] = np > 0 ? m_run[tid] : -INFINITY;
        dst0[GRP * D + GRP + tid] = np > 0 ? l_run[tid] : 0.0f;
    }
    const int ccount = gridDim.y / kAttnCluster;   // clusters per KV head
    const int cid = s / kAttnCluster;
    cluster.sync();                                    // all partials are in rank 0
    trace_stamp(tr, 5);
    trace_stamp(ct, 3);
    if (ct) {
        unsigned smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        ct[5] = smid;
    }
    if (crank == 0) {
        const float* P = reinterpret_cast<const float*>(ring);
        __shared__ float cw[GRP][kAttnCluster];
        __shared__ float cm[GRP], cl[GRP];
        if (tid < GRP) {
            float M = -INFINITY;
            for (int r = 0; r < kAttnCluster; ++r) {
                const float lr = P[r * PSZ + GRP * D + GRP + tid];
                if (lr > 0.0f) M = fmaxf(M, P[r * PSZ + GRP * D + tid]);
            }
            float L = 0.0f;
            for (int r = 0; r < kAttnCluster; ++r) {
                const float lr = P[r * PSZ + GRP * D + GRP + tid];
                const float w = lr > 0.0f ? expf(P[r * PSZ + GRP * D + tid] - M) : 0.0f;
                cw[tid][r] = w;
                L += w * lr;
            }
            cm[tid] = M;
            cl[tid] = L;
        }
        __syncthreads();
        for (int o = tid; o < GRP * D; o += kAT) {
            const int hh = o / D;
            float v = 0.0f;
#pragma unroll
            for (int r = 0; r < kAttnCluster; ++r) v = fmaf(cw[hh][r], P[r * PSZ + o], v);
            part_out[(static_cast<size_t>(g * GRP + hh) * kMaxSplits + cid) * (D + 2) + (o % D)] = v;
        }
        if (tid < GRP) {
            float* p = part_out + (static_cast<size_t>(g * GRP + tid) * kMaxSplits + cid) * (D + 2);
            p[D] = cm[tid];
            p[D + 1] = cl[tid];
        }
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            const unsigned prev = atomicAdd(counters + g, 1u);
            const int last = prev == static_cast<unsigned>(ccount) - 1;
            if (last) __threadfence();
            for (int r = 0; r < kAttnCluster; ++r) *cluster.map_shared_rank(&last_flag, r) = last;
        }
    }
    cluster.sync();  // last_flag of every rank is set
    trace_stamp(tr, 6);
    if (!last_flag) {
        trace_stamp(ct, 4);
        kt_end(a.kt);
        return;
    }

    // ---- merge 2 (the CTAs of the last cluster, each a slice of the outputs): the
    // cluster partials of every head of this KV group, output gate.  Each head's cluster
    // weights w_c = exp(m_c - M) and normaliser 1 / sum w_c l_c are formed once in shared
    // memory; every thread then loads only its outputs' partials, all in one batch ----
    constexpr int kMaxClusters = kMaxSplits / kAttnCluster;
    const int ns = ccount;
    __shared__ float mw[GRP][kMaxClusters];
    __shared__ float minv[GRP];
    if (tid < GRP) {
        const float* ph0 = part_out + static_cast<size_t>(g * GRP + tid) * kMaxSplits * (D + 2);
        float ml[kMaxClusters], ll[kMaxClusters];
#pragma unroll
        for (int c = 0; c < kMaxClusters; ++c) {
            const bool on = c < ns;
            ml[c] = on ? __ldcg(ph0 + static_cast<size_t>(c) * (D + 2) + D) : -INFINITY;
            ll[c] = on ? __ldcg(ph0 + static_cast<size_t>(c) * (D + 2) + D + 1) : 0.0f;
        }
        float M = -INFINITY;
#pragma unroll
        for (int c = 0; c < kMaxClusters; ++c)
            if (ll[c] > 0.0f) M = fmaxf(M, ml[c]);
        float L = 0.0f;
#pragma unroll
        for (int c = 0; c < kMaxClusters; ++c) {
            const float w = ll[c] > 0.0f ? expf(ml[c] - M) : 0.0f;
            mw[tid][c] = w;
            L = fmaf(w, ll[c], L);
        }
        minv[tid] = L > 0.0f ? 1.0f / L : 0.0f;
    }
    __syncthreads();
    for (int o = crank * kAT + tid; o < GRP * D; o += kAttnCluster * kAT) {
        const int hh = o / D, d = o % D;
        const int hq = g * GRP + hh;
        const float* ph0 = part_out + static_cast<size_t>(hq) * kMaxSplits * (D + 2);
        float pv[kMaxClusters];
#pragma unroll
        for (int c = 0; c < kMaxClusters; ++c) pv[c] = c < ns ? __ldcg(ph0 + static_cast<size_t>(c) * (D + 2) + d) : 0.0f;
        const float gate = qg_in[static_cast<size_t>(a.Hq) * D + static_cast<size_t>(hq) * D + d];
        float acc2 = 0.0f;
#pragma unroll
        for (int c = 0; c < kMaxClusters; ++c) acc2 = fmaf(mw[hh][c], pv[c], acc2);
        attn_out[static_cast<size_t>(hq) * D + d] = acc2 * minv[hh] * sigmoid_f(gate);
    }
    if (tid == 0 && crank == 0) counters[g] = 0u;
    if (tid == 0 && crank == 0 && a.trace) a.trace[7] = globaltimer_ns();
    trace_stamp(ct, 4);
    __syncthreads();
    kt_end(a.kt);
}

// ---------------------------------------------------------------------------------------
// Batched decode attention for long histories ("flash-decoding" per warp).
// Grid (Hkv, nsplit, rows), kWW warps per CTA, one CTA per SM.  The CTA prepares the new
// token as the one-sequence kernel does; then page i of the split goes to warp i % kWW
// through stage i % kWRing of a shared ring of tensor-map copies (the warp that consumes
// a stage refills it with page i + kWRing), and every warp keeps its own online softmax,
// so the main loop has no block barrier:
//   scores   S = Q K^T (8 query heads in rows 0..7 of the m16 tile, q = hi + lo bf16),
//            the lane holding head fg keeps the running max / partial sum of that head
//   P V      O^T += V^T P^T: A = V^T straight from the staged tile (ldmatrix .trans),
//            B = P from the score fragments of the same lane (p = hi + lo bf16), so P
//            never leaves registers; O^T is 16 x (D/16) fragments of (dims, heads)
// The warps' partials merge in shared memory into one partial per (row, head, split);
// attn_merge_kernel merges the splits.
constexpr int kWW = 8;        // warps per CTA (two per scheduler)
constexpr int kWRing = 12;    // ring stages (pages in flight) per CTA

template <int D>
constexpr size_t attn_warp_ring_bytes() {
    return static_cast<size_t>(kWRing) * AttnGeom<D>::STAGE + 1024;
}

template <int D, int GRP>
__global__ void __launch_bounds__(kWW * 32, 1) attn_decode_warp_kernel(const __grid_constant__ AttnArgs a) {
    using AG = AttnGeom<D>;
    constexpr int NT = kWW * 32;
    constexpr int KS = D / 16;  // k-steps of Q K^T, m-tiles of V^T P^T
    static_assert(GRP <= 8, "heads of a KV group are rows 0..7 of the m16 tile");
    extern __shared__ __align__(1024) uint8_t ring_raw[];
    uint8_t* ring = ring_raw + ((1024u - (smem_u32(ring_raw) & 1023u)) & 1023u);
    __shared__ __align__(8) uint64_t bar[kWRing];
    // fills issued per stage: the owner of page i waits for fill i / kWRing + 1 to be issued
    // before it waits on the stage's mbarrier, so a parity wait never runs a phase ahead
    __shared__ int filled[kWRing];
    __shared__ __align__(16) float qsm[GRP][D + 4];
    __shared__ __align__(16) uint16_t qh[GRP][D + 8], ql[GRP][D + 8];
    __shared__ __align__(16) float knew[D], vnew[D];
    __shared__ __align__(16) uint16_t kbits[D], vbits[D];
    __shared__ float qn_s[D], kn_s[D];
    __shared__ float2 cs_s[D / 2];
    __shared__ int pages[kMaxPagesPerSplit];
    __shared__ float wm[kWW][8], wl[kWW][8];
    const int g = blockIdx.x, s = blockIdx.y, bz = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int fg = lane >> 2, ft = lane & 3;
    const int slot = a.slots ? a.slots[bz] : 0;
    const float* qg_in = a.qg + bz * a.qg_bs;
    const float* kvnew_in = a.kvnew + bz * a.kvn_bs;
    const int* page_table = a.page_table + slot * a.pt_ss;
    float* part_out = a.part + bz * a.part_bs;

    kt_start(a.kt);
    const int pos = a.pos[slot];
    const int n_tok = pos + 1;
    const int capacity = a.max_pages * kPageTokens;
    const bool in_range = pos >= 0 && pos < capacity;
    const int n_pg = in_range ? (n_tok + kPageTokens - 1) / kPageTokens : 0;
    const int pg0 = static_cast<int>(static_cast<long long>(s) * n_pg / a.nsplit);
    const int pg1 = static_cast<int>(static_cast<long long>(s + 1) * n_pg / a.nsplit);
    const int np = pg1 - pg0;
    const int t0 = pg0 * kPageTokens;
    const int t1 = min(n_tok, pg1 * kPageTokens);
    for (int i = tid; i < np && i < kMaxPagesPerSplit; i += NT) pages[i] = page_table[pg0 + i];
    if (tid == 0) {
        for (int i = 0; i < kWRing; ++i) {
            mbar_init(&bar[i], 1);
            filled[i] = 0;
        }
        mbar_fence_init();
    }
    __syncthreads();
    // page i of the split into stage i % kWRing (a single thread issues)
    auto issue = [&](int i) {
        const int st = i % kWRing;
        const int page = i < kMaxPagesPerSplit ? pages[i] : page_table[pg0 + i];
        const bool good = page >= 0 && page < a.num_pages;
        if (good) {
            mbar_arrive_expect_tx(&bar[st], 2 * kPageTokens * D * 2);
            uint8_t* dst = ring + static_cast<size_t>(st) * AG::STAGE;
#pragma unroll
            for (int kv = 0; kv < 2; ++kv) {
                const int y = a.kv_row0 + ((page * 2 + kv) * a.Hkv + g) * kPageTokens;
#pragma unroll
                for (int c = 0; c < D / 64; ++c) tma_load_2d(dst + kv * AG::TILE + c * AG::CHUNK, &a.kv_map, 64 * c, y, &bar[st]);
            }
        } else {
            raise_error(a.err, DM_DEVERR_PAGE);
            mbar_arrive(&bar[st]);
        }
        __threadfence_block();
        *reinterpret_cast<volatile int*>(&filled[st]) = i / kWRing + 1;
    };
    const int my_np = np > warp ? (np - warp + kWW - 1) / kWW : 0;
    if (tid == 0)
        for (int i = 0; i < np && i < kWRing; ++i) issue(i);
    for (int i = tid; i < D; i += NT) {
        qn_s[i] = bf16_to_f32(a.q_norm[i]);
        kn_s[i] = bf16_to_f32(a.k_norm[i]);
    }
    if (in_range)
        for (int i = tid; i < a.rot_dim / 2; i += NT) cs_s[i] = a.rope[static_cast<size_t>(pos) * (a.rot_dim / 2) + i];
    pdl_wait();
    kt_ready(a.kt);
    if (!in_range) {  // no room: report, touch nothing (no copy was issued)
        if (tid == 0 && s == 0) raise_error(a.err, DM_DEVERR_CAPACITY);
        kt_end(a.kt);
        return;
    }
    attn_prepare<D, GRP, NT>(qg_in + static_cast<size_t>(g * GRP) * D, kvnew_in + static_cast<size_t>(g) * D,
                             kvnew_in + static_cast<size_t>(a.Hkv + g) * D, qn_s, kn_s, cs_s, a.rot_dim, a.eps, qsm, knew,
                             vnew, kbits, vbits, qh, ql);
    pdl_launch_dependents();
    if (s == 0) {  // append at pos (one CTA per row and KV head)
        const int page = page_table[pos / kPageTokens];
        if (page < 0 || page >= a.num_pages) {
            if (tid == 0) raise_error(a.err, DM_DEVERR_PAGE);
        } else {
            uint16_t* kd = a.kv + ((static_cast<size_t>(page) * 2 + 0) * a.Hkv + g) * kPageTokens * D +
                           static_cast<size_t>(pos % kPageTokens) * D;
            uint16_t* vd = a.kv + ((static_cast<size_t>(page) * 2 + 1) * a.Hkv + g) * kPageTokens * D +
                           static_cast<size_t>(pos % kPageTokens) * D;
            for (int d = tid; d < D; d += NT) {
                kd[d] = kbits[d];
                vd[d] = vbits[d];
            }
        }
    }

    // ---- per-warp streaming ----
    const float sm_scale = 1.0f / sqrtf(static_cast<float>(D));
    const bool hrow = fg < GRP;  // this lane's score row is a real head
    // A fragments of q (hi a0, hi a2, lo a0, lo a2 per k-step): held in registers up to
    // D = 128; at D = 256 they would crowd out the O^T accumulators, so they are re-read
    // from shared memory (padded rows: conflict-free) every page
    constexpr bool kQRegs = D <= 128;
    uint32_t qa[kQRegs ? KS : 1][4];
    auto qfrag = [&](int ks, int r) -> uint32_t {
        const int c0 = 16 * ks + 2 * ft + ((r & 1) ? 8 : 0);
        if (!hrow) return 0u;
        return (r < 2) ? *reinterpret_cast<const uint32_t*>(&qh[fg][c0]) : *reinterpret_cast<const uint32_t*>(&ql[fg][c0]);
    };
    if (kQRegs) {
#pragma unroll
        for (int ks = 0; ks < (kQRegs ? KS : 1); ++ks)
#pragma unroll
            for (int r = 0; r < 4; ++r) qa[ks][r] = qfrag(ks, r);
    }
    float o[KS][4];
#pragma unroll
    for (int t = 0; t < KS; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.0f;
    float m_run = -INFINITY, l_part = 0.0f;  // head fg: running max; this lane's share of the sum
    const int ip_new = pos / kPageTokens - pg0;
    for (int j = 0; j < my_np; ++j) {
        const int i = warp + kWW * j;
        const int st = i % kWRing;
        bool ok = true;
        {  // this page's fill issued (the previous owner of the stage is done with it)
            const volatile int* f = &filled[st];
            const int want = i / kWRing + 1;
            if (*f < want) {
                const uint64_t t0 = globaltimer_ns();
                uint32_t it = 0;
                while (*f < want) {
                    if ((++it & 255u) == 0 && globaltimer_ns() - t0 > DM_WAIT_NS) {
                        raise_error(a.err, DM_DEVERR_TIMEOUT);
                        ok = false;
                        break;
                    }
                }
            }
        }
        ok = ok && mbar_wait_bounded(&bar[st], (i / kWRing) & 1, a.err, nullptr);
        uint8_t* kt = ring + static_cast<size_t>(st) * AG::STAGE;
        uint8_t* vt = kt + AG::TILE;
        if (i == ip_new) {  // the staged copy of the page holding pos predates the append
            const int r = pos % kPageTokens;
            for (int d = lane; d < D; d += 32) {
                *reinterpret_cast<uint16_t*>(kt + kv_tile_off<D>(r, d)) = kbits[d];
                *reinterpret_cast<uint16_t*>(vt + kv_tile_off<D>(r, d)) = vbits[d];
            }
            __syncwarp();
        }
        // scores of the page's 16 tokens: n-tile 0 = tokens 0-7, n-tile 1 = tokens 8-15
        float sh0[4] = {0.f, 0.f, 0.f, 0.f}, sl0[4] = {0.f, 0.f, 0.f, 0.f};
        float sh1[4] = {0.f, 0.f, 0.f, 0.f}, sl1[4] = {0.f, 0.f, 0.f, 0.f};
        {
            // ldmatrix x4: matrix lane / 8 = (tokens 8 (m >> 1) .., columns 8 (m & 1) ..)
            const int mi = lane >> 3;
            const int krow = 8 * (mi >> 1) + (lane & 7), kcol = 8 * (mi & 1);
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                uint32_t k0, k1, k2, k3;
                ldsm_x4(k0, k1, k2, k3, kt + kv_tile_off<D>(krow, 16 * ks + kcol));
                uint32_t q0, q1, q2, q3;
                if (kQRegs) {
                    q0 = qa[kQRegs ? ks : 0][0];
                    q1 = qa[kQRegs ? ks : 0][1];
                    q2 = qa[kQRegs ? ks : 0][2];
                    q3 = qa[kQRegs ? ks : 0][3];
                } else {
                    q0 = qfrag(ks, 0);
                    q1 = qfrag(ks, 1);
                    q2 = qfrag(ks, 2);
                    q3 = qfrag(ks, 3);
                }
                mma_bf16_16816(sh0, q0, q1, k0, k1);
                mma_bf16_16816(sl0, q2, q3, k0, k1);
                mma_bf16_16816(sh1, q0, q1, k2, k3);
                mma_bf16_16816(sl1, q2, q3, k2, k3);
            }
        }
        // lane: head fg, tokens 2ft + e (n-tile 0) and 8 + 2ft + e (n-tile 1)
        const int tb = (pg0 + i) * kPageTokens;
        float sv[4];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int p0 = tb + 2 * ft + e, p1 = tb + 8 + 2 * ft + e;
            sv[e] = (ok && hrow && p0 >= t0 && p0 < t1) ? (sh0[e] + sl0[e]) * sm_scale : -INFINITY;
            sv[2 + e] = (ok && hrow && p1 >= t0 && p1 < t1) ? (sh1[e] + sl1[e]) * sm_scale : -INFINITY;
        }
        float mp = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
        mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 1));
        mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 2));
        const float mn = fmaxf(m_run, mp);
        const float alpha = (m_run == -INFINITY) ? (mn == -INFINITY ? 1.0f : 0.0f) : expf(m_run - mn);
        float p[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) p[e] = sv[e] == -INFINITY ? 0.0f : expf(sv[e] - mn);
        l_part = l_part * alpha + ((p[0] + p[1]) + (p[2] + p[3]));
        m_run = mn;
        // rescale O^T columns (heads 2ft, 2ft + 1) by their heads' alpha
        const float a_lo = __shfl_sync(0xffffffffu, alpha, 4 * (2 * ft));
        const float a_hi = __shfl_sync(0xffffffffu, alpha, 4 * (2 * ft + 1));
#pragma unroll
        for (int t = 0; t < KS; ++t) {
            o[t][0] *= a_lo;
            o[t][1] *= a_hi;
            o[t][2] *= a_lo;
            o[t][3] *= a_hi;
        }
        // B fragments of P^T (tokens x heads): b0 = tokens 2ft, 2ft+1 (n-tile 0), b1 = 8 + ...
        uint32_t bh0, bh1, bl0, bl1;
        {
            const uint16_t h00 = f32_to_bf16(p[0]), h01 = f32_to_bf16(p[1]);
            const uint16_t h10 = f32_to_bf16(p[2]), h11 = f32_to_bf16(p[3]);
            bh0 = pack_bf16x2(h00, h01);
            bh1 = pack_bf16x2(h10, h11);
            bl0 = pack_bf16x2(f32_to_bf16(p[0] - bf16_to_f32(h00)), f32_to_bf16(p[1] - bf16_to_f32(h01)));
            bl1 = pack_bf16x2(f32_to_bf16(p[2] - bf16_to_f32(h10)), f32_to_bf16(p[3] - bf16_to_f32(h11)));
        }
        {
            // ldmatrix x4 .trans: matrix lane / 8 = (tokens 8 (m >> 1) .., dims 16t + 8 (m & 1) ..)
            const int mi = lane >> 3;
            const int vrow = 8 * (mi >> 1) + (lane & 7), vcol = 8 * (mi & 1);
#pragma unroll
            for (int t = 0; t < KS; ++t) {
                uint32_t v0, v1, v2, v3;
                ldsm_x4_trans(v0, v1, v2, v3, vt + kv_tile_off<D>(vrow, 16 * t + vcol));
                mma_bf16_16816_full(o[t], v0, v1, v2, v3, bh0, bh1);
                mma_bf16_16816_full(o[t], v0, v1, v2, v3, bl0, bl1);
            }
        }
        __syncwarp();  // every lane is done with the stage
        if (lane == 0 && i + kWRing < np) {
            fence_proxy_async_smem();
            issue(i + kWRing);
        }
    }
    // sum of the head's lanes (ft = 0..3)
    float l_run = l_part;
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if (ft == 0 && fg < 8) {
        wm[warp][fg] = my_np > 0 ? m_run : -INFINITY;
        wl[warp][fg] = my_np > 0 ? l_run : 0.0f;
    }
    __syncthreads();  // every warp out of its loop: the rings are free
    // ---- merge the warps: weights w_w = exp(m_w - M) of each head ----
    float* ow = reinterpret_cast<float*>(ring);  // [kWW][GRP][D]
    const int h0 = 2 * ft, h1 = 2 * ft + 1;
#pragma unroll
    for (int t = 0; t < KS; ++t) {
        const int d0 = 16 * t + fg, d1 = d0 + 8;
        if (h0 < GRP) {
            ow[(warp * GRP + h0) * D + d0] = o[t][0];
            ow[(warp * GRP + h0) * D + d1] = o[t][2];
        }
        if (h1 < GRP) {
            ow[(warp * GRP + h1) * D + d0] = o[t][1];
            ow[(warp * GRP + h1) * D + d1] = o[t][3];
        }
    }
    __syncthreads();
    for (int idx = tid; idx < GRP * (D + 2); idx += NT) {
        const int hh = idx / (D + 2), d = idx % (D + 2);
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < kWW; ++w)
            if (wl[w][hh] > 0.0f) M = fmaxf(M, wm[w][hh]);
        float acc = 0.0f, L = 0.0f;
#pragma unroll
        for (int w = 0; w < kWW; ++w) {
            const float ww = wl[w][hh] > 0.0f ? expf(wm[w][hh] - M) : 0.0f;
            L = fmaf(ww, wl[w][hh], L);
            if (d < D) acc = fmaf(ww, ow[(w * GRP + hh) * D + d], acc);
        }
        float* pp = part_out + (static_cast<size_t>(g * GRP + hh) * kMaxSplits + s) * (D + 2);
        pp[d] = d < D ? acc : (d == D ? M : L);
    }
    __syncthreads();
    kt_end(a.kt);
}

// Dynamic shared memory of a CTA: the page ring of `stages` pages, and at least 120 KB so
// that one CTA runs per SM (two would share an SM's issue slots while other SMs idle).
size_t attn_ring_bytes(int D, int stages) {
    const size_t ring = static_cast<size_t>(stages) * 2 * kPageTokens * D * 2 + 1024;  // + alignment slack
    return ring > 120 * 1024 ? ring : 120 * 1024;
}

int attn_scores_cap(int max_pages, int nsplit) {
    const int max_tok = max_pages * kPageTokens;
    int chunk = (max_tok + nsplit - 1) / nsplit;
    return (chunk + kPageTokens - 1) / kPageTokens * kPageTokens;
}

int attn_nsplit(int num_sms, int Hkv) {
    int ns = num_sms / (Hkv > 0 ? Hkv : 1);
    if (ns > kMaxSplits) ns = kMaxSplits;
    ns = ns / kAttnCluster * kAttnCluster;  // whole clusters
    if (ns < kAttnCluster) ns = kAttnCluster;
    return ns;
}

bool attn_supported(int D, int grp) {
    return (D == 256 && (grp == 8 || grp == 4)) || (D == 128 && (grp == 8 || grp == 4)) ||
           (D == 64 && (grp == 4 || grp == 8));
}

#define DM_ATTN_INSTANCES(X) X(256, 8) X(256, 4) X(128, 8) X(128, 4) X(64, 4) X(64, 8)

template <int D, int GRP, int NB, int ST>
static cudaError_t attn_attr_one() {
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<D, GRP, NB, ST>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(attn_ring_bytes(D, ST)));
    if (e == cudaSuccess)  // largest shared-memory carve-out
        e = cudaFuncSetAttribute(attn_decode_kernel<D, GRP, NB, ST>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    return e;
}

// ---- split merge of the batched attention + the output projection's operand ------------
// One CTA of D threads per (row, query head): the weights w_s = exp(m_s - M) of the head's
// split partials once in shared memory, then every thread one output dimension:
// o = (sum_s w_s O_s[d]) / (sum_s w_s l_s) * sigmoid(gate), written as the hi / lo bf16
// rows of the out-projection GEMM operand (rows b and n + b, column hq * D + d).
template <int D>
__global__ void __launch_bounds__(D) attn_merge_kernel(const float* __restrict__ part, size_t part_bs, int nsplit,
                                                       int msplit, const float* __restrict__ qg, size_t qg_bs, int Hq,
                                                       uint16_t* xcat, int n) {
    const int hq = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    __shared__ float w[kMaxSplits];
    __shared__ float s_inv_l;
    pdl_wait();
    const float* ph = part + b * part_bs + static_cast<size_t>(hq) * msplit * (D + 2);
    if (d < 32) {  // one warp: the split weights and the normaliser
        float m[2], l[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int sp = d + 32 * i;
            const bool on = sp < nsplit;
            l[i] = on ? ph[static_cast<size_t>(sp) * (D + 2) + D + 1] : 0.0f;
            m[i] = (on && l[i] > 0.0f) ? ph[static_cast<size_t>(sp) * (D + 2) + D] : -INFINITY;
        }
        const float M = warp_max(fmaxf(m[0], m[1]));
        float L = 0.0f;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int sp = d + 32 * i;
            const float wi = l[i] > 0.0f ? expf(m[i] - M) : 0.0f;
            if (sp < kMaxSplits) w[sp] = wi;
            L = fmaf(wi, l[i], L);
        }
        L = warp_sum(L);
        if (d == 0) s_inv_l = L > 0.0f ? 1.0f / L : 0.0f;
    }
    __syncthreads();
    pdl_launch_dependents();
    float acc = 0.0f;
    for (int sp = 0; sp < nsplit; ++sp) acc = fmaf(w[sp], ph[static_cast<size_t>(sp) * (D + 2) + d], acc);
    const float gate = qg[b * qg_bs + static_cast<size_t>(Hq) * D + static_cast<size_t>(hq) * D + d];
    const float y = acc * s_inv_l * sigmoid_f(gate);
    const int K = Hq * D, col = hq * D + d;
    const uint16_t hi = f32_to_bf16(y);
    xcat[static_cast<size_t>(b) * K + col] = hi;
    xcat[static_cast<size_t>(n + b) * K + col] = f32_to_bf16(y - bf16_to_f32(hi));
}

cudaError_t launch_attn_merge_batch(const LaunchCfg& lc, const Dims& d, const BatchBuffers& bb, int n) {
    const int ns = attn_nsplit_batch(lc.num_sms, d.Hkv, n);
    const size_t part_bs = static_cast<size_t>(d.Hq) * kMaxSplits * (d.D + 2);
    const size_t qg_bs = static_cast<size_t>(2) * d.Hq * d.D;
    const dim3 grid(d.Hq, n);
    switch (d.D) {
        case 256: return launch_kernel(lc, attn_merge_kernel<256>, grid, dim3(256), 0, bb.attn_part, part_bs, ns, kMaxSplits, bb.qg, qg_bs, d.Hq, bb.xcat, n);
        case 128: return launch_kernel(lc, attn_merge_kernel<128>, grid, dim3(128), 0, bb.attn_part, part_bs, ns, kMaxSplits, bb.qg, qg_bs, d.Hq, bb.xcat, n);
        case 64: return launch_kernel(lc, attn_merge_kernel<64>, grid, dim3(64), 0, bb.attn_part, part_bs, ns, kMaxSplits, bb.qg, qg_bs, d.Hq, bb.xcat, n);
        default: return cudaErrorInvalidValue;
    }
}

template <int D, int GRP>
static cudaError_t attn_warp_attr_one() {
    return cudaFuncSetAttribute(attn_decode_warp_kernel<D, GRP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(attn_warp_ring_bytes<D>()));
}

cudaError_t attn_set_attrs(int max_scores_smem) {
    (void)max_scores_smem;
    cudaError_t e = cudaSuccess;
#define DM_ATTN_ATTR(DD, GG)                                                                 \
    if (e == cudaSuccess) e = attn_attr_one<DD, GG, kAttnStages, kAttnStages>();             \
    if (e == cudaSuccess) e = attn_warp_attr_one<DD, GG>();
    DM_ATTN_INSTANCES(DM_ATTN_ATTR)
#undef DM_ATTN_ATTR
    return e;
}

static cudaError_t attn_warp_launch(const LaunchCfg& lc, const Dims& d, const AttnArgs& a, dim3 grid) {
    const int grp = d.Hq / d.Hkv;
#define DM_ATTN_WLAUNCH(DD, GG)                                                                             \
    if (d.D == DD && grp == GG)                                                                             \
        return launch_kernel(lc, attn_decode_warp_kernel<DD, GG>, grid, dim3(kWW * 32), attn_warp_ring_bytes<DD>(), a);
    DM_ATTN_INSTANCES(DM_ATTN_WLAUNCH)
#undef DM_ATTN_WLAUNCH
    return cudaErrorInvalidValue;
}

static cudaError_t attn_launch(const LaunchCfg& lc, const Dims& d, const AttnArgs& a, dim3 grid) {
    const int grp = d.Hq / d.Hkv;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kAT);
    cfg.dynamicSmemBytes = attn_ring_bytes(d.D, kAttnStages);
    cfg.stream = lc.stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = lc.pdl ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = kAttnCluster;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
#define DM_ATTN_LAUNCH(DD, GG)                                                                              \
    if (d.D == DD && grp == GG)                                                                             \
        return cudaLaunchKernelEx(&cfg, attn_decode_kernel<DD, GG, kAttnStages, kAttnStages>, a);
    DM_ATTN_INSTANCES(DM_ATTN_LAUNCH)
#undef DM_ATTN_LAUNCH
    return cudaErrorInvalidValue;
}

static void attn_common_args(AttnArgs& a, const Dims& d, const LayerW& w, const Buffers& b) {
    a.kv_map = *static_cast<const CUtensorMap*>(b.kv_tmap);
    a.kv_row0 = w.sub * d.num_pages * 2 * d.Hkv * kPageTokens;
    a.q_norm = w.q_norm;
    a.k_norm = w.k_norm;
    a.kv = b.kv + static_cast<size_t>(w.sub) * d.num_pages * 2 * d.Hkv * kPageTokens * d.D;
    a.Hq = d.Hq;
    a.Hkv = d.Hkv;
    a.rot_dim = d.rot_dim;
    a.max_pages = d.max_pages;
    a.num_pages = d.num_pages;
    a.theta = d.theta;
    a.eps = d.eps;
    a.rope = b.rope;
    a.err = b.err;
}

cudaError_t launch_attn_decode(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                               const Buffers& b, int slot) {
    AttnArgs a{};
    attn_common_args(a, d, w, b);
    a.qg = b.qg;
    a.kvnew = b.kvnew;
    a.page_table = b.page_table + static_cast<size_t>(slot) * d.max_pages;
    a.pos = b.pos + slot;
    a.nsplit = attn_nsplit(lc.num_sms, d.Hkv);
    a.cap = attn_scores_cap(d.max_pages, a.nsplit);
    a.part = b.attn_part;
    a.out = b.attn_out;
    a.counters = b.counters + kCntAttnBase;
    a.trace = b.trace ? b.trace + kTrAttn : nullptr;
    a.cta_trace = b.trace ? b.trace + kTrCta : nullptr;
    a.kt = lc.kt;
    const dim3 grid(d.Hkv, a.nsplit);
    if (a.cta_trace && grid.x * grid.y * kTrCtaSlots > kTraceSlots - kTrCta) a.cta_trace = nullptr;
    return attn_launch(lc, d, a, grid);
}

// Splits per (row, KV head) of the batched launch (one CTA per SM): the count that
// minimises waves x (1 / ns + c), the time of a wave being the split's share of a row's
// pages plus a fixed per-CTA cost c (prologue, partial merge) taken as 1 % of a row.
int attn_nsplit_batch(int num_sms, int Hkv, int n) {
    const int units = (n > 0 ? n : 1) * (Hkv > 0 ? Hkv : 1);
    constexpr double kCtaCost = 0.01;
    int best = 1;
    double best_cost = 1e30;
    for (int ns = 1; ns <= kMaxSplits; ++ns) {
        const long long ctas = static_cast<long long>(units) * ns;
        const long long waves = (ctas + num_sms - 1) / num_sms;
        const double cost = static_cast<double>(waves) * (1.0 / ns + kCtaCost);
        if (cost < best_cost - 1e-12) {
            best_cost = cost;
            best = ns;
        }
    }
    return best;
}

cudaError_t launch_attn_decode_batch(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& bb,
                                     const Buffers& b, int n) {
    AttnArgs a{};
    attn_common_args(a, d, w, b);
    a.qg = bb.qg;
    a.kvnew = bb.kvnew;
    a.page_table = b.page_table;
    a.pos = b.pos;
    a.nsplit = attn_nsplit_batch(lc.num_sms, d.Hkv, n);
    a.cap = attn_scores_cap(d.max_pages, a.nsplit);
    a.part = bb.attn_part;
    a.out = bb.attn_out;
    a.counters = bb.attn_cnt;
    a.kt = lc.kt;
    a.slots = bb.slots;
    a.pt_ss = d.max_pages;
    a.cnt_bs = d.Hkv;
    a.qg_bs = static_cast<size_t>(2) * d.Hq * d.D;
    a.kvn_bs = static_cast<size_t>(2) * d.Hkv * d.D;
    a.part_bs = static_cast<size_t>(d.Hq) * kMaxSplits * (d.D + 2);
    a.out_bs = static_cast<size_t>(d.Hq) * d.D;
    return attn_warp_launch(lc, d, a, dim3(d.Hkv, a.nsplit, n));
}

// ---- prefill: a chunk of n prompt tokens of one sequence ---------------------------------
// Reference: forward_attention_qwen36 (src/layers/attention.mojo:219-435) over a prompt,
// causal softmax over every earlier position (:356-421), the prompt's K/V kept in the cache
// (LayerKVCache.store_prefill, kv_cache.mojo:245; appended at current_len, :302).  Row r of
// the chunk is position pos0 + r.
//   pf_attn_prep_kernel  per (row, KV group): the decode kernels' token preparation
//                        (q/k RMSNorm, partial RoPE, k/v to bf16), k/v appended to the
//                        paged cache, q stored as bf16 hi + lo
//   pf_attn_kernel       per (16-row query block, KV group, split of the causal key range):
//                        one warp per query head (rows = the block's 16 tokens), one
//                        producer warp streaming the key pages through a 4-stage ring of
//                        tensor-map copies shared by the group's warps; S = Q K^T and
//                        O += P V on the tensor cores (mma.sync m16n8k16, q and p as hi + lo
//                        bf16 terms), online softmax per row in registers; unnormalised
//                        partials (O, max, sum) per (row, head, split)
//   attn_merge_kernel    (above) merges the splits, applies sigmoid(gate), writes the
//                        out-projection operand rows.
struct PfAttnArgs {
    const float* qg;          // [n][2 Hq D] q | gate projections of the chunk's rows
    const float* kvnew;       // [n][2 Hkv D] k | v projections
    const uint16_t* q_norm;   // [D]
    const uint16_t* k_norm;   // [D]
    uint16_t* kv;             // layer base [num_pages][2][Hkv][16][D]
    const int* page_table;    // [max_pages] of the slot
    const float2* rope;       // [capacity][rot_dim / 2]
    int n, pos0, Hq, Hkv, rot_dim, max_pages, num_pages, nsplit, msplit;
    float eps;
    uint16_t* qhi;            // [n][Hq][D]
    uint16_t* qlo;
    float* part;              // [n][Hq][msplit][D + 2]
    CUtensorMap kv_map;
    int kv_row0;
    uint32_t* err;
};

constexpr int kPfStages = 4;

template <int D, int GRP>
__global__ void __launch_bounds__(256) pf_attn_prep_kernel(const __grid_constant__ PfAttnArgs a) {
    constexpr int NT = 256;
    __shared__ __align__(16) float qsm[GRP][D + 4];
    __shared__ __align__(16) uint16_t qh[GRP][D + 8], ql[GRP][D + 8];
    __shared__ __align__(16) float knew[D], vnew[D];
    __shared__ __align__(16) uint16_t kbits[D], vbits[D];
    __shared__ float qn_s[D], kn_s[D];
    __shared__ float2 cs_s[D / 2];
    const int r = blockIdx.x, g = blockIdx.y, tid = threadIdx.x;
    const int pos = a.pos0 + r;
    for (int i = tid; i < D; i += NT) {
        qn_s[i] = bf16_to_f32(a.q_norm[i]);
        kn_s[i] = bf16_to_f32(a.k_norm[i]);
    }
    for (int i = tid; i < a.rot_dim / 2; i += NT) cs_s[i] = a.rope[static_cast<size_t>(pos) * (a.rot_dim / 2) + i];
    pdl_wait();
    const float* qg = a.qg + static_cast<size_t>(r) * 2 * a.Hq * D;
    const float* kvn = a.kvnew + static_cast<size_t>(r) * 2 * a.Hkv * D;
    attn_prepare<D, GRP, NT>(qg + static_cast<size_t>(g * GRP) * D, kvn + static_cast<size_t>(g) * D,
                             kvn + static_cast<size_t>(a.Hkv + g) * D, qn_s, kn_s, cs_s, a.rot_dim, a.eps, qsm, knew,
                             vnew, kbits, vbits, qh, ql);
    pdl_launch_dependents();
    const int page = a.page_table[pos / kPageTokens];
    if (page < 0 || page >= a.num_pages) {
        if (tid == 0) raise_error(a.err, DM_DEVERR_PAGE);
    } else {
        uint16_t* kd = a.kv + ((static_cast<size_t>(page) * 2 + 0) * a.Hkv + g) * kPageTokens * D +
                       static_cast<size_t>(pos % kPageTokens) * D;
        uint16_t* vd = a.kv + ((static_cast<size_t>(page) * 2 + 1) * a.Hkv + g) * kPageTokens * D +
                       static_cast<size_t>(pos % kPageTokens) * D;
        for (int d = tid; d < D; d += NT) {
            kd[d] = kbits[d];
            vd[d] = vbits[d];
        }
    }
    for (int i = tid; i < GRP * D; i += NT) {
        const size_t o = (static_cast<size_t>(r) * a.Hq + g * GRP + i / D) * D + i % D;
        a.qhi[o] = qh[i / D][i % D];
        a.qlo[o] = ql[i / D][i % D];
    }
}

template <int D, int GRP>
constexpr size_t pf_attn_smem() {
    return static_cast<size_t>(kPfStages) * AttnGeom<D>::STAGE + 2ull * GRP * 16 * (D + 8) * 2 + 1024;
}

template <int D, int GRP>
__global__ void __launch_bounds__((GRP + 1) * 32, 1) pf_attn_kernel(const __grid_constant__ PfAttnArgs a) {
    using AG = AttnGeom<D>;
    constexpr int KS = D / 16;   // k-steps of Q K^T
    constexpr int NTL = D / 8;   // n-tiles of O
    constexpr int QP = D + 8;    // padded q row (bf16 elements): conflict-free ldmatrix rows
    extern __shared__ __align__(1024) uint8_t pf_smem[];
    uint8_t* ring = pf_smem + ((1024u - (smem_u32(pf_smem) & 1023u)) & 1023u);
    uint16_t* qhs = reinterpret_cast<uint16_t*>(ring + kPfStages * AG::STAGE);  // [GRP][16][QP]
    uint16_t* qls = qhs + GRP * 16 * QP;
    __shared__ __align__(8) uint64_t full[kPfStages], empty[kPfStages];
    __shared__ int s_abort;
    volatile int* abort_flag = &s_abort;
    const int qb = blockIdx.x, g = blockIdx.y, s = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = qb * 16;
    const int rmax = min(a.n, r0 + 16) - 1;
    const int n_pg = (a.pos0 + rmax) / kPageTokens + 1;  // pages of keys 0 .. pos0 + rmax
    const int pg0 = static_cast<int>(static_cast<long long>(s) * n_pg / a.nsplit);
    const int pg1 = static_cast<int>(static_cast<long long>(s + 1) * n_pg / a.nsplit);
    const int np = pg1 - pg0;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kPfStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], GRP);
        }
        mbar_fence_init();
        s_abort = 0;
    }
    __syncthreads();
    pdl_wait();  // q and the chunk's own keys come from the preparation kernel
    for (int i = threadIdx.x; i < GRP * 16 * (D / 8); i += (GRP + 1) * 32) {
        const int hh = i / (16 * (D / 8)), rr = (i / (D / 8)) % 16, c8 = i % (D / 8);
        uint4 vh = make_uint4(0u, 0u, 0u, 0u), vl = vh;
        if (r0 + rr < a.n) {
            const size_t o = (static_cast<size_t>(r0 + rr) * a.Hq + g * GRP + hh) * D + c8 * 8;
            vh = *reinterpret_cast<const uint4*>(a.qhi + o);
            vl = *reinterpret_cast<const uint4*>(a.qlo + o);
        }
        *reinterpret_cast<uint4*>(qhs + (hh * 16 + rr) * QP + c8 * 8) = vh;
        *reinterpret_cast<uint4*>(qls + (hh * 16 + rr) * QP + c8 * 8) = vl;
    }
    __syncthreads();
    pdl_launch_dependents();
    if (warp == GRP) {
        // ---- producer: page i of the split into stage i % kPfStages ----
        if (lane == 0) {
            bool ok = true;
            for (int i = 0; i < np && ok; ++i) {
                const int st = i % kPfStages;
                if (i >= kPfStages) {
                    ok = mbar_wait_bounded(&empty[st], ((i / kPfStages) - 1) & 1, a.err, abort_flag);
                    if (!ok) break;
                    fence_proxy_async_smem();
                }
                const int page = a.page_table[pg0 + i];
                if (page < 0 || page >= a.num_pages) {
                    raise_error(a.err, DM_DEVERR_PAGE);
                    mbar_arrive(&full[st]);
                    continue;
                }
                mbar_arrive_expect_tx(&full[st], 2 * kPageTokens * D * 2);
                uint8_t* dst = ring + static_cast<size_t>(st) * AG::STAGE;
#pragma unroll
                for (int kv = 0; kv < 2; ++kv) {
                    const int y = a.kv_row0 + ((page * 2 + kv) * a.Hkv + g) * kPageTokens;
#pragma unroll
                    for (int c = 0; c < D / 64; ++c) tma_load_2d(dst + kv * AG::TILE + c * AG::CHUNK, &a.kv_map, 64 * c, y, &full[st]);
                }
            }
            // the copies still in flight land before the CTA exits
            for (int u = np > kPfStages ? np - kPfStages : 0; u < np; ++u)
                mbar_wait_bounded(&full[u % kPfStages], (u / kPfStages) & 1, a.err, nullptr);
        }
        return;
    }
    // ---- consumer warp: query head g GRP + warp, rows = the block's 16 tokens ----
    const int fg = lane >> 2, ft = lane & 3;
    const uint16_t* qh_w = qhs + warp * 16 * QP;
    const uint16_t* ql_w = qls + warp * 16 * QP;
    const int qp0 = a.pos0 + r0 + fg, qp1 = qp0 + 8;  // positions of this lane's two rows
    const bool rv0 = r0 + fg < a.n, rv1 = r0 + fg + 8 < a.n;
    const float sm_scale = 1.0f / sqrtf(static_cast<float>(D));
    float o[NTL][4];
#pragma unroll
    for (int t = 0; t < NTL; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.0f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_part[2] = {0.0f, 0.0f};
    const int mi = lane >> 3;
    const int krow = 8 * (mi >> 1) + (lane & 7), kcol = 8 * (mi & 1);       // K fragments (B)
    const int arow = (lane & 7) + 8 * (mi & 1), acol = 8 * (mi >> 1);       // Q fragments (A)
    bool ok = true;
    for (int i = 0; i < np; ++i) {
        const int st = i % kPfStages;
        ok = ok && mbar_wait_bounded(&full[st], (i / kPfStages) & 1, a.err, abort_flag);
        const uint8_t* kt = ring + static_cast<size_t>(st) * AG::STAGE;
        const uint8_t* vt = kt + AG::TILE;
        float sh0[4] = {0.f, 0.f, 0.f, 0.f}, sl0[4] = {0.f, 0.f, 0.f, 0.f};
        float sh1[4] = {0.f, 0.f, 0.f, 0.f}, sl1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            uint32_t k0, k1, k2, k3, h0, h1, h2, h3, l0, l1, l2, l3;
            ldsm_x4(k0, k1, k2, k3, kt + kv_tile_off<D>(krow, 16 * ks + kcol));
            ldsm_x4(h0, h1, h2, h3, qh_w + arow * QP + 16 * ks + acol);
            ldsm_x4(l0, l1, l2, l3, ql_w + arow * QP + 16 * ks + acol);
            mma_bf16_16816_full(sh0, h0, h1, h2, h3, k0, k1);
            mma_bf16_16816_full(sl0, l0, l1, l2, l3, k0, k1);
            mma_bf16_16816_full(sh1, h0, h1, h2, h3, k2, k3);
            mma_bf16_16816_full(sl1, l0, l1, l2, l3, k2, k3);
        }
        // sv[4 hf + j]: row fg + 8 hf, keys 2ft, 2ft + 1, 8 + 2ft, 9 + 2ft of the page
        const int kb = (pg0 + i) * kPageTokens;
        float sv[8];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int key0 = kb + 2 * ft + e, key1 = kb + 8 + 2 * ft + e;
            sv[e] = (ok && rv0 && key0 <= qp0) ? (sh0[e] + sl0[e]) * sm_scale : -INFINITY;
            sv[2 + e] = (ok && rv0 && key1 <= qp0) ? (sh1[e] + sl1[e]) * sm_scale : -INFINITY;
            sv[4 + e] = (ok && rv1 && key0 <= qp1) ? (sh0[2 + e] + sl0[2 + e]) * sm_scale : -INFINITY;
            sv[6 + e] = (ok && rv1 && key1 <= qp1) ? (sh1[2 + e] + sl1[2 + e]) * sm_scale : -INFINITY;
        }
        float p[8], alpha[2];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            float mp = fmaxf(fmaxf(sv[4 * hf], sv[4 * hf + 1]), fmaxf(sv[4 * hf + 2], sv[4 * hf + 3]));
            mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 1));
            mp = fmaxf(mp, __shfl_xor_sync(0xffffffffu, mp, 2));
            const float mn = fmaxf(m_run[hf], mp);
            alpha[hf] = (m_run[hf] == -INFINITY) ? (mn == -INFINITY ? 1.0f : 0.0f) : expf(m_run[hf] - mn);
#pragma unroll
            for (int e = 0; e < 4; ++e) p[4 * hf + e] = sv[4 * hf + e] == -INFINITY ? 0.0f : expf(sv[4 * hf + e] - mn);
            l_part[hf] = l_part[hf] * alpha[hf] + ((p[4 * hf] + p[4 * hf + 1]) + (p[4 * hf + 2] + p[4 * hf + 3]));
            m_run[hf] = mn;
        }
#pragma unroll
        for (int t = 0; t < NTL; ++t) {
            o[t][0] *= alpha[0];
            o[t][1] *= alpha[0];
            o[t][2] *= alpha[1];
            o[t][3] *= alpha[1];
        }
        // P as A fragments: a0 = row fg keys 2ft.., a1 = row fg + 8, a2 / a3 = keys 8 + 2ft..
        uint32_t ah[4], al[4];
        {
            const int idx[4][2] = {{0, 1}, {4, 5}, {2, 3}, {6, 7}};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint16_t x0 = f32_to_bf16(p[idx[q][0]]), x1 = f32_to_bf16(p[idx[q][1]]);
                ah[q] = pack_bf16x2(x0, x1);
                al[q] = pack_bf16x2(f32_to_bf16(p[idx[q][0]] - bf16_to_f32(x0)), f32_to_bf16(p[idx[q][1]] - bf16_to_f32(x1)));
            }
        }
        // V as B fragments (.trans): matrices (keys 0-7 | 8-15) x (dims 16 j .. | 16 j + 8 ..)
        const int vrow = (lane & 7) + 8 * (mi & 1), vcol = 8 * (mi >> 1);
#pragma unroll
        for (int j = 0; j < NTL / 2; ++j) {
            uint32_t v0, v1, v2, v3;
            ldsm_x4_trans(v0, v1, v2, v3, vt + kv_tile_off<D>(vrow, 16 * j + vcol));
            mma_bf16_16816_full(o[2 * j], ah[0], ah[1], ah[2], ah[3], v0, v1);
            mma_bf16_16816_full(o[2 * j], al[0], al[1], al[2], al[3], v0, v1);
            mma_bf16_16816_full(o[2 * j + 1], ah[0], ah[1], ah[2], ah[3], v2, v3);
            mma_bf16_16816_full(o[2 * j + 1], al[0], al[1], al[2], al[3], v2, v3);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
    }
    const int hq = g * GRP + warp;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        float l = l_part[hf];
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        const int r = r0 + fg + 8 * hf;
        if (r < a.n) {
            float* pp = a.part + ((static_cast<size_t>(r) * a.Hq + hq) * a.msplit + s) * (D + 2);
#pragma unroll
            for (int t = 0; t < NTL; ++t) {
                pp[8 * t + 2 * ft] = o[t][2 * hf];
                pp[8 * t + 2 * ft + 1] = o[t][2 * hf + 1];
            }
            if (ft == 0) {
                pp[D] = m_run[hf];
                pp[D + 1] = l;
            }
        }
    }
}

template <int D, int GRP>
static cudaError_t pf_attn_attr_one() {
    return cudaFuncSetAttribute(pf_attn_kernel<D, GRP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(pf_attn_smem<D, GRP>()));
}

cudaError_t pf_attn_set_attrs() {
    cudaError_t e = cudaSuccess;
#define DM_PF_ATTR(DD, GG) \
    if (e == cudaSuccess) e = pf_attn_attr_one<DD, GG>();
    DM_ATTN_INSTANCES(DM_PF_ATTR)
#undef DM_PF_ATTR
    return e;
}

// Splits of the causal key range per (query block, KV group): about two CTAs per SM.
int pf_attn_nsplit(int num_sms, int Hkv, int n) {
    const int units = ((n + 15) / 16) * (Hkv > 0 ? Hkv : 1);
    int ns = (2 * num_sms + units - 1) / units;
    if (ns > kPfMaxSplits) ns = kPfMaxSplits;
    return ns < 1 ? 1 : ns;
}

cudaError_t launch_pf_attn(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& pb,
                           const Buffers& b, int slot, int pos0, int n) {
    PfAttnArgs a{};
    a.qg = pb.qg;
    a.kvnew = pb.kvnew;
    a.q_norm = w.q_norm;
    a.k_norm = w.k_norm;
    a.kv = b.kv + static_cast<size_t>(w.sub) * d.num_pages * 2 * d.Hkv * kPageTokens * d.D;
    a.page_table = b.page_table + static_cast<size_t>(slot) * d.max_pages;
    a.rope = b.rope;
    a.n = n;
    a.pos0 = pos0;
    a.Hq = d.Hq;
    a.Hkv = d.Hkv;
    a.rot_dim = d.rot_dim;
    a.max_pages = d.max_pages;
    a.num_pages = d.num_pages;
    a.nsplit = pf_attn_nsplit(lc.num_sms, d.Hkv, n);
    a.msplit = kPfMaxSplits;
    a.eps = d.eps;
    a.qhi = pb.pf_qhi;
    a.qlo = pb.pf_qlo;
    a.part = pb.attn_part;
    a.kv_map = *static_cast<const CUtensorMap*>(b.kv_tmap);
    a.kv_row0 = w.sub * d.num_pages * 2 * d.Hkv * kPageTokens;
    a.err = b.err;
    const int grp = d.Hq / d.Hkv;
    cudaError_t e = cudaErrorInvalidValue;
#define DM_PF_LAUNCH(DD, GG)                                                                                         \
    if (d.D == DD && grp == GG) {                                                                                    \
        e = launch_kernel(lc, pf_attn_prep_kernel<DD, GG>, dim3(n, d.Hkv), dim3(256), 0, a);                         \
        if (e == cudaSuccess)                                                                                        \
            e = launch_kernel(lc, pf_attn_kernel<DD, GG>, dim3((n + 15) / 16, d.Hkv, a.nsplit), dim3((GG + 1) * 32),  \
                              pf_attn_smem<DD, GG>(), a);                                                            \
    }
    DM_ATTN_INSTANCES(DM_PF_LAUNCH)
#undef DM_PF_LAUNCH
    if (e != cudaSuccess) return e;
    const size_t part_bs = static_cast<size_t>(d.Hq) * kPfMaxSplits * (d.D + 2);
    const size_t qg_bs = static_cast<size_t>(2) * d.Hq * d.D;
    const dim3 grid(d.Hq, n);
    switch (d.D) {
        case 256: return launch_kernel(lc, attn_merge_kernel<256>, grid, dim3(256), 0, pb.attn_part, part_bs, a.nsplit, kPfMaxSplits, pb.qg, qg_bs, d.Hq, pb.xcat, n);
        case 128: return launch_kernel(lc, attn_merge_kernel<128>, grid, dim3(128), 0, pb.attn_part, part_bs, a.nsplit, kPfMaxSplits, pb.qg, qg_bs, d.Hq, pb.xcat, n);
        case 64: return launch_kernel(lc, attn_merge_kernel<64>, grid, dim3(64), 0, pb.attn_part, part_bs, a.nsplit, kPfMaxSplits, pb.qg, qg_bs, d.Hq, pb.xcat, n);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace dm
