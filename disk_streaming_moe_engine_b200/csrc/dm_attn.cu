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

constexpr int kAttnCluster = 8;  // splits merged on chip per cluster

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
__global__ void __launch_bounds__(128) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
    using AG = AttnGeom<D>;
    constexpr int EPL = D / 32;  // q/k elements per lane in the score loop
    extern __shared__ __align__(128) uint8_t ring[];
    __shared__ __align__(8) uint64_t bar[kAttnStages];
    __shared__ __align__(16) float qsm[GRP][D];
    __shared__ __align__(16) float knew[D], vnew[D];
    __shared__ uint16_t kbits[D], vbits[D];
    __shared__ float sc[GRP][kPageTokens];
    __shared__ float m_run[GRP], l_run[GRP], scale[GRP];
    __shared__ float wsp[GRP][kMaxSplits];
    __shared__ int is_last;
    const int g = blockIdx.x, s = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;

    uint64_t* tr = (tid == 0 && g == 0 && s == gridDim.y - 1) ? a.trace : nullptr;
    trace_stamp(tr, 0);
    kt_start(a.kt);
    // positions < pos were written by earlier steps and the page table is fixed: the
    // range of this split and its first page tiles do not depend on the previous kernel
    const int pos = *a.pos;
    const int n_tok = pos + 1;
    const int capacity = a.max_pages * kPageTokens;
    const bool in_range = pos >= 0 && pos < capacity;
    int chunk = (n_tok + a.nsplit - 1) / a.nsplit;
    chunk = (chunk + kPageTokens - 1) / kPageTokens * kPageTokens;
    const int t0 = in_range ? s * chunk : 0;
    const int t1 = in_range ? min(n_tok, t0 + chunk) : 0;
    const int np = t1 > t0 ? (t1 - 1) / kPageTokens - t0 / kPageTokens + 1 : 0;
    const int pg0 = t0 / kPageTokens;
    __shared__ int pages[kMaxPagesPerSplit];
    for (int i = tid; i < np && i < kMaxPagesPerSplit; i += 128) pages[i] = a.page_table[pg0 + i];
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
    for (int i = tid; i < D; i += 128) {
        qn_s[i] = bf16_to_f32(a.q_norm[i]);
        kn_s[i] = bf16_to_f32(a.k_norm[i]);
    }
    if (in_range)
        for (int i = tid; i < a.rot_dim / 2; i += 128) cs_s[i] = a.rope[static_cast<size_t>(pos) * (a.rot_dim / 2) + i];
    trace_stamp(tr, 1);
    pdl_wait();
    kt_ready(a.kt);
    trace_stamp(tr, 2);
    if (!in_range) {  // no room: report, touch nothing
        if (tid == 0 && s == 0) raise_error(a.err, DM_DEVERR_CAPACITY);
        kt_end(a.kt);
        return;
    }

    // ---- q heads of this KV group, new k, new v: one parallel load, then per-head
    // RMSNorm + RoPE in shared memory (norm weights and the RoPE row were staged before
    // the wait) ----
    {   // all loads issued together (one round trip), then stored
        constexpr int QPT = GRP * D / 128, KPT = (D + 127) / 128;
        float qv[QPT], kv[KPT], vv[KPT];
        const float* qsrc = a.qg + static_cast<size_t>(g * GRP) * D;
#pragma unroll
        for (int i = 0; i < QPT; ++i) qv[i] = qsrc[tid + 128 * i];
#pragma unroll
        for (int i = 0; i < KPT; ++i) {
            const int d = tid + 128 * i;
            kv[i] = d < D ? a.kvnew[static_cast<size_t>(g) * D + d] : 0.0f;
            vv[i] = d < D ? a.kvnew[static_cast<size_t>(a.Hkv + g) * D + d] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < QPT; ++i) (&qsm[0][0])[tid + 128 * i] = qv[i];
#pragma unroll
        for (int i = 0; i < KPT; ++i) {
            const int d = tid + 128 * i;
            if (d < D) {
                knew[d] = kv[i];
                vnew[d] = vv[i];
            }
        }
    }
    __syncthreads();
    trace_stamp(tr, 8);
    for (int hh = warp; hh < GRP + 1; hh += 4) {
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
    for (int d = tid; d < D; d += 128) {
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
            for (int d = tid; d < D; d += 128) {
                kd[d] = kbits[d];
                vd[d] = vbits[d];
            }
        }
    }

    // q of this warp's lanes in registers: element e of head hh = q[hh][lane*EPL + e]
    float qr[GRP][EPL];
#pragma unroll
    for (int hh = 0; hh < GRP; ++hh)
#pragma unroll
        for (int e = 0; e < EPL; ++e) qr[hh][e] = qsm[hh][lane * EPL + e];
    const float sm_scale = 1.0f / sqrtf(static_cast<float>(D));
    constexpr int DPT = (D + 127) / 128;  // V dims per thread
    float acc[GRP][DPT];
#pragma unroll
    for (int hh = 0; hh < GRP; ++hh)
#pragma unroll
        for (int j = 0; j < DPT; ++j) acc[hh][j] = 0.0f;

    for (int i = 0; i < np; ++i) {
        const int slot = i % kAttnStages;
        const bool ok = mbar_wait_bounded(&bar[slot], (i / kAttnStages) & 1, a.err, nullptr);
        const uint16_t* kt = reinterpret_cast<const uint16_t*>(ring + static_cast<size_t>(slot) * AG::STAGE);
        const uint16_t* vt = kt + kPageTokens * D;
        const int tp = (pg0 + i) * kPageTokens;  // position of the page's first token
        // scores: warp w -> tokens w, w+4, w+8, w+12 of the page
        for (int tt = warp; tt < kPageTokens; tt += 4) {
            const int t = tp + tt;
            float kf[EPL];
            if (t == pos) {
#pragma unroll
                for (int e = 0; e < EPL; ++e) kf[e] = knew[lane * EPL + e];
            } else if (EPL == 8) {
                const uint4 u = *reinterpret_cast<const uint4*>(kt + tt * D + lane * 8);
                kf[0] = bf16lo(u.x); kf[1] = bf16hi(u.x); kf[2] = bf16lo(u.y); kf[3] = bf16hi(u.y);
                kf[4] = bf16lo(u.z); kf[5] = bf16hi(u.z); kf[6] = bf16lo(u.w); kf[7] = bf16hi(u.w);
            } else {
#pragma unroll
                for (int e = 0; e < EPL; ++e) kf[e] = bf16_to_f32(kt[tt * D + lane * EPL + e]);
            }
            const bool valid = ok && t >= t0 && t < t1;
#pragma unroll
            for (int hh = 0; hh < GRP; ++hh) {
                float p = 0.0f;
#pragma unroll
                for (int e = 0; e < EPL; ++e) p = fmaf(qr[hh][e], kf[e], p);
                p = warp_sum(p);
                if (lane == 0) sc[hh][tt] = valid ? p * sm_scale : -INFINITY;
            }
        }
        __syncthreads();
        // online softmax update, one warp per head: lanes 0..15 hold the page's scores
        for (int hh = warp; hh < GRP; hh += 4) {
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
        // V: thread owns dims tid, tid + 128, ...
#pragma unroll
        for (int j = 0; j < DPT; ++j) {
            const int d = tid + 128 * j;
            if (d < D) {
#pragma unroll
                for (int hh = 0; hh < GRP; ++hh) acc[hh][j] *= scale[hh];
                for (int tt = 0; tt < kPageTokens; ++tt) {
                    const int t = tp + tt;
                    const float v = (t == pos) ? vnew[d] : bf16_to_f32(vt[tt * D + d]);
#pragma unroll
                    for (int hh = 0; hh < GRP; ++hh) acc[hh][j] = fmaf(sc[hh][tt], v, acc[hh][j]);
                }
            }
        }
        __syncthreads();  // stage free and sc reusable
        if (tid == 0 && i + kAttnStages < np) issue(i + kAttnStages);
    }

    trace_stamp(tr, 4);
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
#pragma unroll
    for (int j = 0; j < DPT; ++j) {
        const int d = tid + 128 * j;
        if (d < D)
#pragma unroll
            for (int hh = 0; hh < GRP; ++hh) dst0[hh * D + d] = acc[hh][j];
    }
    if (tid < GRP) {
        dst0[GRP * D + tid] = np > 0 ? m_run[tid] : -INFINITY;
        dst0[GRP * D + GRP + tid] = np > 0 ? l_run[tid] : 0.0f;
    }
    const int ccount = gridDim.y / kAttnCluster;   // clusters per KV head
    const int cid = s / kAttnCluster;
    cluster.sync();                                    // all partials are in rank 0
    trace_stamp(tr, 5);
    if (crank != 0) {
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
        for (int o = tid; o < GRP * D; o += 128) {
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
        kt_end(a.kt);
        return;
    }
    __threadfence();

    // ---- merge 2: the cluster partials of every head of this KV group, output gate ----
    const int ns = ccount;
    for (int hh = warp; hh < GRP; hh += 4) {
        const float* ph = a.part + static_cast<size_t>(g * GRP + hh) * kMaxSplits * (D + 2);
        const float ml = lane < ns ? __ldcg(ph + lane * (D + 2) + D) : -INFINITY;
        const float ll = lane < ns ? __ldcg(ph + lane * (D + 2) + D + 1) : 0.0f;
        const float M = warp_max(ll > 0.0f ? ml : -INFINITY);
        const float wk = ll > 0.0f ? expf(ml - M) : 0.0f;
        const float L = warp_sum(wk * ll);
        if (lane < kMaxSplits) wsp[hh][lane] = wk / L;
    }
    __syncthreads();
    for (int o = tid; o < GRP * D; o += 128) {
        const int hh = o / D, d = o % D;
        const int hq = g * GRP + hh;
        const float* ph = a.part + static_cast<size_t>(hq) * kMaxSplits * (D + 2) + d;
        float acc2 = 0.0f;
        for (int c = 0; c < ns; ++c) acc2 = fmaf(wsp[hh][c], __ldcg(ph + static_cast<size_t>(c) * (D + 2)), acc2);
        const float gate = a.qg[static_cast<size_t>(a.Hq) * D + static_cast<size_t>(hq) * D + d];
        a.out[static_cast<size_t>(hq) * D + d] = acc2 * sigmoid_f(gate);
    }
    if (tid == 0) a.counters[g] = 0u;
    if (tid == 0 && a.trace) a.trace[7] = globaltimer_ns();
    __syncthreads();
    kt_end(a.kt);
}

size_t attn_ring_bytes(int D) {
    return static_cast<size_t>(kAttnStages) * 2 * 2 * kPageTokens * D;
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
                                 max_scores_smem);
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
    a.kt = lc.kt;
    a.next_w = lc.l2_prefetch ? w.w_out : nullptr;
    a.next_bytes = static_cast<size_t>(d.H) * d.Hq * d.D * 2;
    a.err = b.err;
    const int grp = d.Hq / d.Hkv;
    const dim3 grid(d.Hkv, a.nsplit);
    const size_t smem = attn_ring_bytes(d.D);
#define DM_ATTN_LAUNCH(DD, GG)                                                                 \
    if (d.D == DD && grp == GG) return cudaLaunchKernelEx(&cfg, attn_decode_kernel<DD, GG>, a);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(128);
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
