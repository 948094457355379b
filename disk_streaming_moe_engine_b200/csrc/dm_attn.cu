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
template <int D>
struct AttnGeom {
    static constexpr int TILE = kPageTokens * D * 2;     // bytes of K (or V) of one page, one head
    static constexpr int STAGE = 2 * TILE;
    static constexpr int RING = kAttnStages * STAGE;
};

template <int D, int GRP>
__global__ void __launch_bounds__(kAT, 1) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
    using AG = AttnGeom<D>;
    extern __shared__ __align__(128) uint8_t ring[];
    __shared__ __align__(8) uint64_t bar[kAttnStages];
    constexpr int QST = D + 4;  // padded q row: the 8 heads of a score step hit 8 bank groups
    __shared__ __align__(16) float qsm[GRP][QST];
    __shared__ __align__(16) float knew[D], vnew[D];
    __shared__ uint16_t kbits[D], vbits[D];
    __shared__ float sc[GRP][kPageTokens];
    __shared__ float m_run[GRP], l_run[GRP], scale[GRP];
    __shared__ float wsp[GRP][kMaxSplits];
    __shared__ int is_last;
    const int g = blockIdx.x, s = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;

    uint64_t* tr = (tid == 0 && g == 0 && s == gridDim.y - 1) ? a.trace : nullptr;
    uint64_t* ct = (tid == 0 && a.cta_trace) ? a.cta_trace + (s * gridDim.x + g) * kTrCtaSlots : nullptr;
    trace_stamp(tr, 0);
    trace_stamp(ct, 0);
    kt_start(a.kt);
    // positions < pos were written by earlier steps and the page table is fixed: the
    // range of this split and its first page tiles do not depend on the previous kernel
    const int pos = *a.pos;
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
    for (int i = tid; i < np && i < kMaxPagesPerSplit; i += kAT) pages[i] = a.page_table[pg0 + i];
    __syncthreads();
    auto issue = [&](int i) {  // page i of this split into its ring stage (thread 0 only)
        const int slot = i % kAttnStages;
        uint8_t* dst = ring + static_cast<size_t>(slot) * AG::STAGE;
        const int page = i < kMaxPagesPerSplit ? pages[i] : a.page_table[pg0 + i];
        if (page < 0 || page >= a.num_pages) {
            raise_error(a.err, DM_DEVERR_PAGE);
            mbar_arrive(&bar[slot]);  // no copy: the tile is left as is and masked below
            return;
        }
        mbar_arrive_expect_tx(&bar[slot], AG::STAGE);
        const uint16_t* kt = a.kv + ((static_cast<size_t>(page) * 2 + 0) * a.Hkv + g) * kPageTokens * D;
        const uint16_t* vt = a.kv + ((static_cast<size_t>(page) * 2 + 1) * a.Hkv + g) * kPageTokens * D;
        bulk_g2s(dst, kt, AG::TILE, &bar[slot]);
        bulk_g2s(dst + AG::TILE, vt, AG::TILE, &bar[slot]);
    };
    prefetch_l2_share(a.next_w, a.next_bytes, s * gridDim.x + g, gridDim.x * gridDim.y, tid);
    if (tid == 0) {
        for (int i = 0; i < kAttnStages; ++i) mbar_init(&bar[i], 1);
        mbar_fence_init();
        for (int i = 0; i < np && i < kAttnStages; ++i) issue(i);
    }
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
    {   // all loads issued together (one round trip), then stored
        constexpr int QPT = (GRP * D + kAT - 1) / kAT, KPT = (D + kAT - 1) / kAT;
        float qv[QPT], kv[KPT], vv[KPT];
        const float* qsrc = a.qg + static_cast<size_t>(g * GRP) * D;
#pragma unroll
        for (int i = 0; i < QPT; ++i) qv[i] = tid + kAT * i < GRP * D ? qsrc[tid + kAT * i] : 0.0f;
#pragma unroll
        for (int i = 0; i < KPT; ++i) {
            const int d = tid + kAT * i;
            kv[i] = d < D ? a.kvnew[static_cast<size_t>(g) * D + d] : 0.0f;
            vv[i] = d < D ? a.kvnew[static_cast<size_t>(a.Hkv + g) * D + d] : 0.0f;
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
    for (int d = tid; d < D; d += kAT) {
        const uint16_t kb = f32_to_bf16(knew[d]);
        kbits[d] = kb;
        knew[d] = bf16_to_f32(kb);
        const uint16_t vb = f32_to_bf16(vnew[d]);
        vbits[d] = vb;
        vnew[d] = bf16_to_f32(vb);
    }
    __syncthreads();
    pdl_launch_dependents();
    trace_stamp(tr, 3);

    // ---- append at pos (one CTA per KV head) ----
    if (s == 0) {
        const int page = a.page_table[pos / kPageTokens];
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

    const float sm_scale = 1.0f / sqrtf(static_cast<float>(D));
    // V mapping: accumulator element idx = tid + kAT * k (k < NA) is head idx / D, dim
    // idx % D; D divides kAT, so a thread's elements share the dim v_d = tid % D
    static_assert(kAT % D == 0, "D must divide the CTA size");
    constexpr int NA = (GRP * D + kAT - 1) / kAT;
    const int v_d = tid % D, v_h0 = tid / D;
    constexpr int VHS = kAT / D;  // head stride between a thread's elements
    const bool v_on = v_h0 < GRP;
    float acc[NA];
#pragma unroll
    for (int k = 0; k < NA; ++k) acc[k] = 0.0f;
    // score mapping: TPP threads per (token, head) pair, thread part p takes the 8-dim
    // blocks p, p + TPP, ... (adjacent parts read adjacent 16-byte words)
    constexpr int TPP = kAT / (kPageTokens * GRP);
    static_assert(TPP >= 1 && kAT % (kPageTokens * GRP) == 0 && (D / 8) % TPP == 0,
                  "the CTA must cover 16 tokens x GRP heads");
    const int pair = tid / TPP, part = tid % TPP;
    const int s_tt = pair / GRP, s_hh = pair % GRP;
    const float4* q4 = reinterpret_cast<const float4*>(qsm[s_hh]);

    for (int i = 0; i < np; ++i) {
        const int slot = i % kAttnStages;
        const bool ok = mbar_wait_bounded(&bar[slot], (i / kAttnStages) & 1, a.err, nullptr);
        uint64_t* trp = (tr && i < 4) ? tr + 40 + 4 * i : nullptr;  // per-page stamps, pages 0-3
        trace_stamp(trp, 0);
        const uint16_t* kt = reinterpret_cast<const uint16_t*>(ring + static_cast<size_t>(slot) * AG::STAGE);
        const uint16_t* vt = kt + kPageTokens * D;
        const int tp = (pg0 + i) * kPageTokens;  // position of the page's first token
        {   // score of token s_tt for head s_hh: eight independent partial sums
            const int t = tp + s_tt;
            float pa[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) pa[e] = 0.0f;
            if (t == pos) {
                const float4* k4 = reinterpret_cast<const float4*>(knew);
#pragma unroll 4
                for (int j = part; j < D / 8; j += TPP) {
                    const float4 k0 = k4[2 * j], k1 = k4[2 * j + 1];
                    const float4 q0 = q4[2 * j], q1 = q4[2 * j + 1];
                    pa[0] = fmaf(q0.x, k0.x, pa[0]); pa[1] = fmaf(q0.y, k0.y, pa[1]);
                    pa[2] = fmaf(q0.z, k0.z, pa[2]); pa[3] = fmaf(q0.w, k0.w, pa[3]);
                    pa[4] = fmaf(q1.x, k1.x, pa[4]); pa[5] = fmaf(q1.y, k1.y, pa[5]);
                    pa[6] = fmaf(q1.z, k1.z, pa[6]); pa[7] = fmaf(q1.w, k1.w, pa[7]);
                }
            } else {
                const uint4* kr = reinterpret_cast<const uint4*>(kt + s_tt * D);
#pragma unroll 4
                for (int j = part; j < D / 8; j += TPP) {
                    const uint4 u = kr[j];
                    const float4 q0 = q4[2 * j], q1 = q4[2 * j + 1];
                    pa[0] = fmaf(q0.x, bf16lo(u.x), pa[0]); pa[1] = fmaf(q0.y, bf16hi(u.x), pa[1]);
                    pa[2] = fmaf(q0.z, bf16lo(u.y), pa[2]); pa[3] = fmaf(q0.w, bf16hi(u.y), pa[3]);
                    pa[4] = fmaf(q1.x, bf16lo(u.z), pa[4]); pa[5] = fmaf(q1.y, bf16hi(u.z), pa[5]);
                    pa[6] = fmaf(q1.z, bf16lo(u.w), pa[6]); pa[7] = fmaf(q1.w, bf16hi(u.w), pa[7]);
                }
            }
            float p = ((pa[0] + pa[1]) + (pa[2] + pa[3])) + ((pa[4] + pa[5]) + (pa[6] + pa[7]));
#pragma unroll
            for (int m = 1; m < TPP; m <<= 1) p += __shfl_xor_sync(0xffffffffu, p, m);
            const bool valid = ok && t >= t0 && t < t1;
            if (part == 0) sc[s_hh][s_tt] = valid ? p * sm_scale : -INFINITY;
        }
        __syncthreads();
        trace_stamp(trp, 1);
        // online softmax update, one warp per head: lanes 0..15 hold the page's scores
        for (int hh = warp; hh < GRP; hh += kAW) {
            const float sv = lane < kPageTokens ? sc[hh][lane] : -INFINITY;
            const float mp = warp_max(sv);
            const float mo = m_run[hh];
            const float mn = fmaxf(mo, mp);
            const float pv = (lane < kPageTokens && sv != -INFINITY) ? expf(sv - mn) : 0.0f;
            const float ls = warp_sum(pv);
            if (lane < kPageTokens) sc[hh][lane] = pv;
            if (lane == 0) {
                const float f = (mo == -INFINITY) ? 0.0f : expf(mo - mn);
                scale[hh] = f;
                l_run[hh] = l_run[hh] * f + ls;
                m_run[hh] = mn;
            }
        }
        __syncthreads();
        trace_stamp(trp, 2);
        // V: the thread's NA accumulators (one dim, heads v_h0, v_h0 + VHS, ...)
        if (v_on) {
#pragma unroll
            for (int k = 0; k < NA; ++k) acc[k] *= scale[v_h0 + VHS * k];
#pragma unroll 4
            for (int tt = 0; tt < kPageTokens; ++tt) {
                const int t = tp + tt;
                const float v = (t == pos) ? vnew[v_d] : bf16_to_f32(vt[tt * D + v_d]);
#pragma unroll
                for (int k = 0; k < NA; ++k) acc[k] = fmaf(sc[v_h0 + VHS * k][tt], v, acc[k]);
            }
        }
        __syncthreads();  // stage free and sc reusable
        trace_stamp(trp, 3);
        if (tid == 0 && i + kAttnStages < np) issue(i + kAttnStages);
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
    if (v_on)
#pragma unroll
        for (int k = 0; k < NA; ++k) dst0[(v_h0 + VHS * k) * D + v_d] = acc[k];
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
    if (crank != 0) {
        trace_stamp(ct, 4);
        kt_end(a.kt);
        return;
    }
    {
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
            a.part[(static_cast<size_t>(g * GRP + hh) * kMaxSplits + cid) * (D + 2) + (o % D)] = v;
        }
        if (tid < GRP) {
            float* p = a.part + (static_cast<size_t>(g * GRP + tid) * kMaxSplits + cid) * (D + 2);
            p[D] = cm[tid];
            p[D + 1] = cl[tid];
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(a.counters + g, 1u);
        is_last = (prev == static_cast<unsigned>(ccount) - 1);
    }
    __syncthreads();
    trace_stamp(tr, 6);
    if (!is_last) {
        trace_stamp(ct, 4);
        kt_end(a.kt);
        return;
    }
    __threadfence();

    // ---- merge 2: the cluster partials of every head of this KV group, output gate ----
    const int ns = ccount;
    for (int hh = warp; hh < GRP; hh += kAW) {
        const float* ph = a.part + static_cast<size_t>(g * GRP + hh) * kMaxSplits * (D + 2);
        const float ml = lane < ns ? __ldcg(ph + lane * (D + 2) + D) : -INFINITY;
        const float ll = lane < ns ? __ldcg(ph + lane * (D + 2) + D + 1) : 0.0f;
        const float M = warp_max(ll > 0.0f ? ml : -INFINITY);
        const float wk = ll > 0.0f ? expf(ml - M) : 0.0f;
        const float L = warp_sum(wk * ll);
        if (lane < kMaxSplits) wsp[hh][lane] = wk / L;
    }
    __syncthreads();
    // every cluster partial of an output is loaded in one batch (fixed bound, unrolled)
    constexpr int kMaxClusters = kMaxSplits / kAttnCluster;
#pragma unroll 2
    for (int o = tid; o < GRP * D; o += kAT) {
        const int hh = o / D, d = o % D;
        const int hq = g * GRP + hh;
        const float* ph = a.part + static_cast<size_t>(hq) * kMaxSplits * (D + 2) + d;
        float pv[kMaxClusters];
#pragma unroll
        for (int c = 0; c < kMaxClusters; ++c) pv[c] = c < ns ? __ldcg(ph + static_cast<size_t>(c) * (D + 2)) : 0.0f;
        const float gate = a.qg[static_cast<size_t>(a.Hq) * D + static_cast<size_t>(hq) * D + d];
        float acc2 = 0.0f;
#pragma unroll
        for (int c = 0; c < kMaxClusters; ++c) acc2 = fmaf(wsp[hh][c], pv[c], acc2);
        a.out[static_cast<size_t>(hq) * D + d] = acc2 * sigmoid_f(gate);
    }
    if (tid == 0) a.counters[g] = 0u;
    if (tid == 0 && a.trace) a.trace[7] = globaltimer_ns();
    trace_stamp(ct, 4);
    __syncthreads();
    kt_end(a.kt);
}

// Dynamic shared memory of a CTA: the page ring, and at least 120 KB so that one CTA
// runs per SM (two would share an SM's issue slots while other SMs stay idle).
size_t attn_ring_bytes(int D) {
    const size_t ring = static_cast<size_t>(kAttnStages) * 2 * 2 * kPageTokens * D;
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

cudaError_t attn_set_attrs(int max_scores_smem) {
    cudaError_t e = cudaSuccess;
#define DM_ATTN_ATTR(DD, GG)                                                                      \
    if (e == cudaSuccess)                                                                         \
        e = cudaFuncSetAttribute(attn_decode_kernel<DD, GG>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 max_scores_smem);                                                \
    if (e == cudaSuccess) /* largest shared-memory carve-out: two CTAs per SM */                    \
        e = cudaFuncSetAttribute(attn_decode_kernel<DD, GG>,                                      \
                                 cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    DM_ATTN_INSTANCES(DM_ATTN_ATTR)
#undef DM_ATTN_ATTR
    return e;
}

cudaError_t launch_attn_decode(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                               const Buffers& b, int slot) {
    AttnArgs a{};
    a.qg = b.qg;
    a.kvnew = b.kvnew;
    a.q_norm = w.q_norm;
    a.k_norm = w.k_norm;
    a.kv = b.kv + static_cast<size_t>(w.sub) * d.num_pages * 2 * d.Hkv * kPageTokens * d.D;
    a.page_table = b.page_table + static_cast<size_t>(slot) * d.max_pages;
    a.pos = b.pos + slot;
    a.Hq = d.Hq;
    a.Hkv = d.Hkv;
    a.rot_dim = d.rot_dim;
    a.max_pages = d.max_pages;
    a.num_pages = d.num_pages;
    a.nsplit = attn_nsplit(lc.num_sms, d.Hkv);
    a.cap = attn_scores_cap(d.max_pages, a.nsplit);
    a.theta = d.theta;
    a.eps = d.eps;
    a.part = b.attn_part;
    a.out = b.attn_out;
    a.counters = b.counters + kCntAttnBase;
    a.rope = b.rope;
    a.trace = b.trace ? b.trace + kTrAttn : nullptr;
    a.cta_trace = b.trace ? b.trace + kTrCta : nullptr;
    a.kt = lc.kt;
    a.next_w = lc.l2_prefetch ? w.w_out : nullptr;
    a.next_bytes = static_cast<size_t>(d.H) * d.Hq * d.D * 2;
    a.err = b.err;
    const int grp = d.Hq / d.Hkv;
    const dim3 grid(d.Hkv, a.nsplit);
    if (a.cta_trace && grid.x * grid.y * kTrCtaSlots > kTraceSlots - kTrCta) a.cta_trace = nullptr;
    const size_t smem = attn_ring_bytes(d.D);
#define DM_ATTN_LAUNCH(DD, GG)                                                                 \
    if (d.D == DD && grp == GG) return cudaLaunchKernelEx(&cfg, attn_decode_kernel<DD, GG>, a);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kAT);
    cfg.dynamicSmemBytes = smem;
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
    DM_ATTN_INSTANCES(DM_ATTN_LAUNCH)
#undef DM_ATTN_LAUNCH
    return cudaErrorInvalidValue;
}

}  // namespace dm
