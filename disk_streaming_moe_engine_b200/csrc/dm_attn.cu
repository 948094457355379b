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
    const void* next_w;       // o_proj weights, prefetched into L2
    size_t next_bytes;
    uint32_t* err;
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

constexpr int kAttnStages = 6;   // K+V page tiles in flight per CTA
constexpr int kMaxPagesPerSplit = 256;  // page ids staged in shared memory

// One KV page tile (16 tokens x D, K then V) per ring stage.
// One KV page (16 tokens, one head) per ring stage: K rows then V rows, each row padded
// to RS bytes so that the 8 rows an ldmatrix reads fall in distinct bank groups.
template <int D>
struct AttnGeom {
    static constexpr int RS = (D + 8) * 2;               // bytes of one staged row
    static constexpr int TILE = kPageTokens * RS;        // K (or V) of one page
    static constexpr int STAGE = 2 * TILE;
    static constexpr int RING = kAttnStages * STAGE;
};

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
DM_DEV uint32_t pack_bf16x2(uint16_t lo, uint16_t hi) { return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16); }
DM_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

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
// NB = pages scored per batch: kAttnStages (one sequence: every page of a split in flight at
// once) or fewer, so that the next batch's pages load while this one is scored.
template <int D, int GRP, int NB>
__global__ void __launch_bounds__(kAT, 1) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
    static_assert(NB >= 1 && NB <= kAttnStages && kAttnStages % NB == 0, "batch of whole ring stages");
    using AG = AttnGeom<D>;
    static_assert(GRP <= 8, "heads of a KV group are rows 0..7 of the m16 tile");
    extern __shared__ __align__(128) uint8_t ring[];
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
    // page i of the split into its ring stage: 16 K rows and 16 V rows, one bulk copy
    // each, by the 32 lanes of warp 0 (row r < 16: K row r; r >= 16: V row r - 16)
    auto issue = [&](int i) {
        const int slot = i % kAttnStages;
        const int page = i < kMaxPagesPerSplit ? pages[i] : page_table[pg0 + i];
        const bool good = page >= 0 && page < a.num_pages;
        if (lane == 0) {
            if (good) {
                mbar_arrive_expect_tx(&bar[slot], 2 * kPageTokens * D * 2);
            } else {
                raise_error(a.err, DM_DEVERR_PAGE);
                mbar_arrive(&bar[slot]);  // no copy: the tile is left as is and masked below
            }
        }
        __syncwarp();
        if (good) {
            const int kv = lane >> 4, r = lane & 15;
            const uint16_t* src =
                a.kv + ((static_cast<size_t>(page) * 2 + kv) * a.Hkv + g) * kPageTokens * D + static_cast<size_t>(r) * D;
            bulk_g2s(ring + static_cast<size_t>(slot) * AG::STAGE + kv * AG::TILE + r * AG::RS, src, D * 2, &bar[slot]);
        }
    };
    if (warp == 0)
        for (int i = 0; i < np && i < kAttnStages; ++i) issue(i);
    prefetch_l2_share(a.next_w, a.next_bytes, s * gridDim.x + g, gridDim.x * gridDim.y, tid);
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

    // ---- q heads of this KV group, new k, new v: one parallel load, then per-head
    // RMSNorm + RoPE in shared memory (norm weights and the RoPE row were staged before
    // the wait) ----
    {
        constexpr int QPT = (GRP * D + kAT - 1) / kAT, KPT = (D + kAT - 1) / kAT;
        float qv[QPT], kv[KPT], vv[KPT];
        const float* qsrc = qg_in + static_cast<size_t>(g * GRP) * D;
#pragma unroll
        for (int i = 0; i < QPT; ++i) qv[i] = tid + kAT * i < GRP * D ? qsrc[tid + kAT * i] : 0.0f;
#pragma unroll
        for (int i = 0; i < KPT; ++i) {
            const int d = tid + kAT * i;
            kv[i] = d < D ? kvnew_in[static_cast<size_t>(g) * D + d] : 0.0f;
            vv[i] = d < D ? kvnew_in[static_cast<size_t>(a.Hkv + g) * D + d] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < QPT; ++i)
            if (tid + kAT * i < GRP * D) qsm[(tid + kAT * i) / D][(tid + kAT * i) % D] = qv[i];
#pragma unroll
        for (int i = 0; i < KPT; ++i) {
            const int d = tid + kAT * i;
            if (d < D) {
                knew[d] = kv[i];
                vnew[d] = vv[i];
            }
        }
    }
    __syncthreads();
    trace_stamp(tr, 8);
    for (int hh = warp; hh < GRP + 1; hh += kAW) {
        float* v = hh < GRP ? qsm[hh] : knew;
        const float* wn = hh < GRP ? qn_s : kn_s;
        float ss = 0.0f;
        for (int d = lane; d < D; d += 32) ss = fmaf(v[d], v[d], ss);
        ss = warp_sum(ss);
        const float rs = 1.0f / sqrtf(ss / static_cast<float>(D) + a.eps);
        for (int d = lane; d < D; d += 32) v[d] = v[d] * rs * wn[d];
        __syncwarp();
        const int half = a.rot_dim / 2;
        for (int i = lane; i < half; i += 32) {
            const float2 c = cs_s[i];
            const float x0 = v[i], x1 = v[i + half];
            v[i] = x0 * c.x - x1 * c.y;
            v[i + half] = x0 * c.y + x1 * c.x;
        }
        __syncwarp();
    }
    __syncthreads();
    trace_stamp(tr, 9);
    // k, v rounded to bf16 (cache format); q as hi + lo bf16 terms for the tensor cores
    const float sm_scale = 1.0f / sqrtf(static_cast<float>(D));
    for (int d = tid; d < D; d += kAT) {
        const uint16_t kb = f32_to_bf16(knew[d]);
        kbits[d] = kb;
        const uint16_t vb = f32_to_bf16(vnew[d]);
        vbits[d] = vb;
    }
    for (int i = tid; i < GRP * D; i += kAT) {
        const float q = qsm[i / D][i % D];
        const uint16_t hi = f32_to_bf16(q);
        qh[i / D][i % D] = hi;
        ql[i / D][i % D] = f32_to_bf16(q - bf16_to_f32(hi));
    }
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
            uint16_t* kr = reinterpret_cast<uint16_t*>(st + (pos % kPageTokens) * AG::RS);
            uint16_t* vr = reinterpret_cast<uint16_t*>(st + AG::TILE + (pos % kPageTokens) * AG::RS);
            for (int d = tid; d < D; d += kAT) {
                kr[d] = kbits[d];
                vr[d] = vbits[d];
            }
        }
        __syncthreads();
        // scores: warp w < 2 nb takes n-tile w (tokens 8w..8w+7 of the batch)
        if (warp < 2 * nb) {
            const int pi = warp >> 1;  // page of the batch
            const uint8_t* kt = ring + static_cast<size_t>((b0 + pi) % kAttnStages) * AG::STAGE;
            // ldmatrix x2 row addresses: lanes 0-7 tokens of k-columns 0-7, lanes 8-15 of 8-15
            const uint8_t* krow = kt + (8 * (warp & 1) + (lane & 7)) * AG::RS + ((lane >> 3) & 1) * 16;
            float ch[4] = {0.0f, 0.0f, 0.0f, 0.0f}, cl[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const bool arow = fg < GRP;
#pragma unroll 4
            for (int ks = 0; ks < D / 16; ++ks) {
                uint32_t b0r, b1r;
                ldsm_x2(b0r, b1r, krow + ks * 32);
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
                const uint8_t* vrow = vt + (8 * (m & 1) + (lane & 7)) * AG::RS + (16 * warp + 8 * (m >> 1)) * 2;
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
    static_assert(kAttnCluster * PSZ * 4 <= AG::RING, "ring too small for the cluster merge");
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
    // cluster partials of every head of this KV group, output gate; every load of an
    // output (its partials and their max / sum) is issued in one batch ----
    constexpr int kMaxClusters = kMaxSplits / kAttnCluster;
    const int ns = ccount;
    for (int o = crank * kAT + tid; o < GRP * D; o += kAttnCluster * kAT) {
        const int hh = o / D, d = o % D;
        const int hq = g * GRP + hh;
        const float* ph0 = part_out + static_cast<size_t>(hq) * kMaxSplits * (D + 2);
        float pv[kMaxClusters], ml[kMaxClusters], ll[kMaxClusters];
#pragma unroll
        for (int c = 0; c < kMaxClusters; ++c) {
            const bool on = c < ns;
            pv[c] = on ? __ldcg(ph0 + static_cast<size_t>(c) * (D + 2) + d) : 0.0f;
            ml[c] = on ? __ldcg(ph0 + static_cast<size_t>(c) * (D + 2) + D) : -INFINITY;
            ll[c] = on ? __ldcg(ph0 + static_cast<size_t>(c) * (D + 2) + D + 1) : 0.0f;
        }
        const float gate = qg_in[static_cast<size_t>(a.Hq) * D + static_cast<size_t>(hq) * D + d];
        float M = -INFINITY;
#pragma unroll
        for (int c = 0; c < kMaxClusters; ++c)
            if (ll[c] > 0.0f) M = fmaxf(M, ml[c]);
        float L = 0.0f, acc2 = 0.0f;
#pragma unroll
        for (int c = 0; c < kMaxClusters; ++c) {
            const float w = ll[c] > 0.0f ? expf(ml[c] - M) : 0.0f;
            L = fmaf(w, ll[c], L);
            acc2 = fmaf(w, pv[c], acc2);
        }
        attn_out[static_cast<size_t>(hq) * D + d] = (L > 0.0f ? acc2 / L : 0.0f) * sigmoid_f(gate);
    }
    if (tid == 0 && crank == 0) counters[g] = 0u;
    if (tid == 0 && crank == 0 && a.trace) a.trace[7] = globaltimer_ns();
    trace_stamp(ct, 4);
    __syncthreads();
    kt_end(a.kt);
}

// Dynamic shared memory of a CTA: the page ring, and at least 120 KB so that one CTA
// runs per SM (two would share an SM's issue slots while other SMs stay idle).
size_t attn_ring_bytes(int D) {
    const size_t ring = static_cast<size_t>(kAttnStages) * 2 * kPageTokens * (D + 8) * 2;
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
constexpr int kAttnBatchNB = 3;  // pages per scored batch of the batched launch (two batches in flight)

template <int D, int GRP, int NB>
static cudaError_t attn_attr_one(int max_scores_smem) {
    cudaError_t e = cudaFuncSetAttribute(attn_decode_kernel<D, GRP, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         max_scores_smem);
    if (e == cudaSuccess)  // largest shared-memory carve-out
        e = cudaFuncSetAttribute(attn_decode_kernel<D, GRP, NB>, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    return e;
}

cudaError_t attn_set_attrs(int max_scores_smem) {
    cudaError_t e = cudaSuccess;
#define DM_ATTN_ATTR(DD, GG)                                                    \
    if (e == cudaSuccess) e = attn_attr_one<DD, GG, kAttnStages>(max_scores_smem); \
    if (e == cudaSuccess) e = attn_attr_one<DD, GG, kAttnBatchNB>(max_scores_smem);
    DM_ATTN_INSTANCES(DM_ATTN_ATTR)
#undef DM_ATTN_ATTR
    return e;
}

static cudaError_t attn_launch(const LaunchCfg& lc, const Dims& d, const AttnArgs& a, dim3 grid, bool batched) {
    const int grp = d.Hq / d.Hkv;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kAT);
    cfg.dynamicSmemBytes = attn_ring_bytes(d.D);
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
        return batched ? cudaLaunchKernelEx(&cfg, attn_decode_kernel<DD, GG, kAttnBatchNB>, a)              \
                       : cudaLaunchKernelEx(&cfg, attn_decode_kernel<DD, GG, kAttnStages>, a);
    DM_ATTN_INSTANCES(DM_ATTN_LAUNCH)
#undef DM_ATTN_LAUNCH
    return cudaErrorInvalidValue;
}

static void attn_common_args(AttnArgs& a, const Dims& d, const LayerW& w, const Buffers& b) {
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
    a.next_w = lc.l2_prefetch ? w.w_out : nullptr;
    a.next_bytes = static_cast<size_t>(d.H) * d.Hq * d.D * 2;
    const dim3 grid(d.Hkv, a.nsplit);
    if (a.cta_trace && grid.x * grid.y * kTrCtaSlots > kTraceSlots - kTrCta) a.cta_trace = nullptr;
    return attn_launch(lc, d, a, grid, false);
}

// Splits per (row, KV head) of the batched launch: about two CTAs per SM over the whole
// grid, in whole clusters.
int attn_nsplit_batch(int num_sms, int Hkv, int n) {
    const int units = (n > 0 ? n : 1) * (Hkv > 0 ? Hkv : 1);
    int ns = (2 * num_sms + units - 1) / units;
    ns = (ns + kAttnCluster - 1) / kAttnCluster * kAttnCluster;
    if (ns > kMaxSplits) ns = kMaxSplits;
    if (ns < kAttnCluster) ns = kAttnCluster;
    return ns;
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
    return attn_launch(lc, d, a, dim3(d.Hkv, a.nsplit, n), true);
}

}  // namespace dm
