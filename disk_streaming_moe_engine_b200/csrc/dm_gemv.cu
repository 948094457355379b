// dm_gemv.cu — bf16-weight GEMV for the decode step (batch 1), HBM-bound.
//
// y[r] = sum_k W[r, k] * xs[k]   for r in [0, N),  W bf16 row-major, xs fp32 in smem.
//
// One 512-thread CTA per SM; warp gw of the grid reduces rows gw, gw + W, ... with
// 128-bit non-allocating loads (8 per lane in flight per row chunk).  At the 17-50 MB
// per-launch sizes of this path, many warps issuing 128-bit loads reach HBM bandwidth
// sooner than a single-issuer bulk-copy ring (measured on B200: 50 MB in 9.7 us vs 14.1 us
// for a 16 KB x 6 cp.async.bulk ring, 17 MB in 4.0 us vs 8.4 us).  The first row's
// weights are requested before griddepcontrol.wait (weights are read-only), so under
// programmatic dependent launch they stream while the previous kernel finishes; the next
// row's loads are issued before the current row's warp reduction.
//
// Prologues build xs from the previous kernel's output:
//   PRO_RMSNORM   xs = (x / sqrt(mean(x^2) + eps)) * gamma         (reference rmsnorm.mojo:10)
//   PRO_HEADNORM  xs[h*dv+d] = o*rsqrt(mean_h(o^2)+eps)*w[d]*z     (reference gdn.mojo:1134-1153)
//   PRO_COPY      xs = x
// Epilogues are per row segment: store, SiLU, residual add, ring-slot store (GDN conv
// window) or logits + argmax (first maximum wins, reference cmd_decode.mojo:115).
#include "dm_common.cuh"
#include <cstdlib>

#include "dm_kernels.h"

namespace dm {

// 16 warps per CTA, one CTA per SM; warp gw of the grid reduces rows gw, gw + W, ...
// (W = all warps), so consecutive warps read consecutive rows and every SM streams.
constexpr int kGemvThreads = 512;
constexpr int kGemvWarps = kGemvThreads / 32;

template <int K>
struct GemvGeom {
    static constexpr int VPL = K / 256;                 // 16-byte weight vectors per lane per row
    static constexpr int CH = VPL > 8 ? 8 : VPL;        // vectors held in registers at once
    static constexpr int NCH = VPL / CH;                // register chunks per row
};

// xs split layout: float4 lo[K/8] holds x[8j..8j+3], hi[K/8] holds x[8j+4..8j+7], so a
// lane reading its 8 elements touches consecutive 16-byte words (no bank conflicts).
__device__ __forceinline__ void xs_store(float* xs, int K, int k, float v) {
    int j = k >> 3, e = k & 7;
    xs[(e < 4 ? 0 : K / 2) + j * 4 + (e & 3)] = v;
}

template <int CH>
__device__ __forceinline__ void load_chunk(uint4 (&w)[CH], const uint16_t* rowp, int c, int lane) {
    const uint4* p = reinterpret_cast<const uint4*>(rowp) + c * CH * 32 + lane;
#pragma unroll
    for (int i = 0; i < CH; ++i) w[i] = ldg_nc_v4(p + 32 * i);
}

template <int CH>
__device__ __forceinline__ void fma_chunk(const uint4 (&w)[CH], const float4* xlo, const float4* xhi, int c,
                                          int lane, float& acc0, float& acc1) {
#pragma unroll
    for (int i = 0; i < CH; ++i) {
        const int j = c * CH * 32 + lane + 32 * i;
        const float4 x0 = xlo[j], x1 = xhi[j];
        acc0 = fmaf(bf16lo(w[i].x), x0.x, acc0);
        acc1 = fmaf(bf16hi(w[i].x), x0.y, acc1);
        acc0 = fmaf(bf16lo(w[i].y), x0.z, acc0);
        acc1 = fmaf(bf16hi(w[i].y), x0.w, acc1);
        acc0 = fmaf(bf16lo(w[i].z), x1.x, acc0);
        acc1 = fmaf(bf16hi(w[i].z), x1.y, acc1);
        acc0 = fmaf(bf16lo(w[i].w), x1.z, acc0);
        acc1 = fmaf(bf16hi(w[i].w), x1.w, acc1);
    }
}

template <int K, int PRO>
__global__ void __launch_bounds__(kGemvThreads, 2) gemv_bf16_kernel(const __grid_constant__ GemvArgs a) {
    using G = GemvGeom<K>;
    __shared__ __align__(16) float xs[K];
    __shared__ float red[kGemvWarps];
    __shared__ float cand_v[kGemvWarps];
    __shared__ int cand_i[kGemvWarps];
    __shared__ int is_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int nw = gridDim.x * kGemvWarps;
    int row = blockIdx.x * kGemvWarps + warp;
    kt_start(a.kt);

    // weights do not depend on the previous kernel: first chunk in flight before the wait
    uint4 w[G::CH];
    if (row < a.N) load_chunk<G::CH>(w, a.W + static_cast<size_t>(row) * K, 0, lane);
    // L2 look-ahead: lane 0 keeps the rows pf strides ahead of the one in registers
    // requested from HBM (no register or shared-memory cost)
    if (lane == 0)
        for (int q = 1; q <= a.pf; ++q)
            if (row + q * nw < a.N) bulk_prefetch_l2(a.W + static_cast<size_t>(row + q * nw) * K, K * 2);
    constexpr int XPT = K / kGemvThreads;  // activations per thread (K >= 512) or 1
    constexpr int XN = XPT > 0 ? XPT : 1;
    float gv[XN];  // norm gains are weights: fetched before the wait
    if (PRO == PRO_RMSNORM) {
#pragma unroll
        for (int i = 0; i < XN; ++i) {
            const int k = tid + kGemvThreads * i;
            gv[i] = k < K ? bf16_to_f32(a.gamma[k]) : 0.0f;
        }
    }
    pdl_wait();
    kt_ready(a.kt);

    if (PRO == PRO_RMSNORM) {
        float xv[XN];
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < XN; ++i) {
            const int k = tid + kGemvThreads * i;
            xv[i] = k < K ? a.x[k] : 0.0f;
            acc = fmaf(xv[i], xv[i], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) red[warp] = acc;
        __syncthreads();
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < kGemvWarps; ++i) ss += red[i];
        const float denom = sqrtf(ss / static_cast<float>(K) + a.eps);
#pragma unroll
        for (int i = 0; i < XN; ++i) {
            const int k = tid + kGemvThreads * i;
            if (k < K) xs_store(xs, K, k, (xv[i] / denom) * gv[i]);
        }
    } else if (PRO == PRO_HEADNORM) {
        // warp h handles heads h, h + 16, ...; the o and z values of a head (dv <= 128)
        // are loaded in one batch per lane
        const int dv = a.hn_dim, nh = K / dv;
        for (int h = warp; h < nh; h += kGemvWarps) {
            const float* oh = a.hn_o + h * dv;
            const float* zh = a.hn_z + h * dv;
            float ov[4], zv[4], wv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int d = lane + 32 * i;
                ov[i] = d < dv ? oh[d] : 0.0f;
                zv[i] = d < dv ? zh[d] : 0.0f;
                wv[i] = d < dv ? bf16_to_f32(a.hn_w[d]) : 0.0f;
            }
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) acc = fmaf(ov[i], ov[i], acc);
            acc = warp_sum(acc);
            const float rs = 1.0f / sqrtf(acc / static_cast<float>(dv) + a.eps);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int d = lane + 32 * i;
                if (d < dv) xs_store(xs, K, h * dv + d, ov[i] * rs * wv[i] * zv[i]);
            }
        }
    } else {
        float xv[XN];
#pragma unroll
        for (int i = 0; i < XN; ++i) {
            const int k = tid + kGemvThreads * i;
            xv[i] = k < K ? a.x[k] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < XN; ++i) {
            const int k = tid + kGemvThreads * i;
            if (k < K) xs_store(xs, K, k, xv[i]);
        }
    }
    __syncthreads();
    pdl_launch_dependents();

    const int ring_slot = a.pos ? (*a.pos & (kConvRing - 1)) : 0;
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    const float4* xlo = reinterpret_cast<const float4*>(xs);
    const float4* xhi = reinterpret_cast<const float4*>(xs + K / 2);

    while (row < a.N) {
        const uint16_t* rowp = a.W + static_cast<size_t>(row) * K;
        float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
        for (int c = 0; c < G::NCH; ++c) {
            if (c > 0) load_chunk<G::CH>(w, rowp, c, lane);
            fma_chunk<G::CH>(w, xlo, xhi, c, lane, acc0, acc1);
        }
        const int next = row + nw;
        if (next < a.N) load_chunk<G::CH>(w, a.W + static_cast<size_t>(next) * K, 0, lane);  // overlap the reduction
        if (lane == 0 && a.pf > 0 && row + (a.pf + 1) * nw < a.N)
            bulk_prefetch_l2(a.W + static_cast<size_t>(row + (a.pf + 1) * nw) * K, K * 2);
        const float acc = warp_sum(acc0 + acc1);
        if (lane == 0) {
            int s = 0, rstart = 0;
            while (s < a.nseg - 1 && row >= a.seg[s].row_end) {
                rstart = a.seg[s].row_end;
                ++s;
            }
            const GemvSeg& g = a.seg[s];
            const int lr = row - rstart;
            float* out = g.out + (g.ring_stride ? static_cast<size_t>(ring_slot) * g.ring_stride : 0);
            switch (g.act) {
                case ACT_SILU: out[lr] = silu_f(acc); break;
                case ACT_RESID: out[lr] = g.res[lr] + acc; break;
                case ACT_ARGMAX:
                    out[lr] = acc;
                    if (acc != acc || isinf(acc)) raise_error(a.err, DM_DEVERR_NONFINITE);
                    else if (acc > best_v) { best_v = acc; best_i = row; }
                    break;
                default: out[lr] = acc; break;
            }
        }
        row = next;
    }

    if (a.kt) {
        __syncthreads();
        kt_end(a.kt);
    }
    if (a.counter == nullptr) return;
    // ---- argmax across the grid: per-CTA candidate, last CTA reduces ----
    if (lane == 0) {
        cand_v[warp] = best_v;
        cand_i[warp] = best_i;
    }
    __syncthreads();
    if (tid == 0) {
        float bv = cand_v[0];
        int bi = cand_i[0];
        for (int q = 1; q < kGemvWarps; ++q)
            if (cand_v[q] > bv || (cand_v[q] == bv && cand_i[q] < bi)) { bv = cand_v[q]; bi = cand_i[q]; }
        a.cand_val[blockIdx.x] = bv;
        a.cand_idx[blockIdx.x] = bi;
        __threadfence();
        const unsigned prev = atomicAdd(a.counter, 1u);
        is_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    if (warp == 0) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int c = lane; c < static_cast<int>(gridDim.x); c += 32) {
            const float v = __ldcg(a.cand_val + c);
            const int i = __ldcg(a.cand_idx + c);
            if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
        }
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) {
            if (bi == 0x7fffffff) bi = 0;  // every logit non-finite: error already raised
            *a.token_out = bi;
            if (a.pos_inc) *a.pos_inc += 1;
            if (a.gen_out) {
                const int gi = *a.gen_idx;
                if (gi < a.gen_cap) a.gen_out[gi] = bi;
                *a.gen_idx = gi + 1;
            }
            *a.counter = 0u;
        }
    }
}

template <int K, int PRO>
static cudaError_t launch_gemv_t(const LaunchCfg& lc, GemvArgs a) {
    a.kt = lc.kt;
    // L2 look-ahead (lane 0 of every warp prefetching rows pf grid strides ahead, before the
    // wait too): off.  The fused MoE kernel before an input projection already prefetches
    // that projection's weights into L2 while its top-k leaves HBM idle; on top of that the
    // look-ahead only competes with the MoE's routed-expert copies.  Measured in the decode
    // step (two repetitions): 0 rows 624.8, 1 row 615.1, 2 rows 614.1 tok/s.  (Before the
    // MoE prefetched, one row was the best setting: 0 rows 558.4, 1 row 566.6, 2 rows 558.7.)
    a.pf = 0;
    const int want = (a.N + kGemvWarps - 1) / kGemvWarps;
    // two CTAs per SM: measured faster in the decode step than one, although one CTA per
    // SM leaves room for the next kernel's prologue (588.0 vs 588.0 tok/s for the attention
    // out-projection alone at one CTA per SM, slower for the input projections)
    const int cap = lc.num_sms * 2;
    int grid = want < cap ? want : cap;
    if (a.counter && grid > kMaxCtas) grid = kMaxCtas;
    return launch_kernel(lc, gemv_bf16_kernel<K, PRO>, dim3(grid), dim3(kGemvThreads), 0, a);
}

cudaError_t launch_gemv(const LaunchCfg& lc, int K, int pro, const GemvArgs& a) {
#define DM_GEMV_CASE(KK)                                                        \
    case KK:                                                                    \
        if (pro == PRO_RMSNORM) return launch_gemv_t<KK, PRO_RMSNORM>(lc, a);   \
        if (pro == PRO_HEADNORM) return launch_gemv_t<KK, PRO_HEADNORM>(lc, a); \
        return launch_gemv_t<KK, PRO_COPY>(lc, a);
    switch (K) {
        DM_GEMV_CASE(256)
        DM_GEMV_CASE(512)
        DM_GEMV_CASE(1024)
        DM_GEMV_CASE(2048)
        DM_GEMV_CASE(4096)
        default: return cudaErrorInvalidValue;
    }
#undef DM_GEMV_CASE
}

// Static shared memory only (<= 16 KB of activations): nothing to configure.
cudaError_t gemv_set_attrs() { return cudaSuccess; }

bool gemv_supported_k(int K) {
    return K == 256 || K == 512 || K == 1024 || K == 2048 || K == 4096;
}

// ---------------------------------------------------------------------------------------
// Embedding gather: xres[slot] = fp32(embed[token])  (reference gguf_embed_tokens,
// gguf_port_loader.mojo:274).  Token outside [0, V) raises DM_DEVERR_TOKEN and embeds 0.
__global__ void __launch_bounds__(256) embed_kernel(const uint16_t* __restrict__ embed, int H, int V,
                                                    const int* token, float* x, uint32_t* err, uint64_t* kt) {
    kt_start(kt);
    pdl_wait();
    kt_ready(kt);
    int t = *token;
    if (t < 0 || t >= V) {
        if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(err, DM_DEVERR_TOKEN);
        t = 0;
    }
    pdl_launch_dependents();
    const uint16_t* row = embed + static_cast<size_t>(t) * H;
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < H; k += gridDim.x * blockDim.x)
        x[k] = bf16_to_f32(row[k]);
    kt_end(kt);
}

cudaError_t launch_embed(const LaunchCfg& lc, const Dims& d, const uint16_t* embed,
                         const Buffers& b, int slot) {
    const int blocks = (d.H + 255) / 256;
    return launch_kernel(lc, embed_kernel, dim3(blocks), dim3(256), 0, embed, d.H, d.V,
                         b.token + slot, b.xres + static_cast<size_t>(slot) * d.H, b.err, lc.kt);
}

// ---------------------------------------------------------------------------------------
// Layer-level GEMV launches.
cudaError_t launch_gdn_in(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                          const Buffers& b, int slot) {
    GemvArgs a{};
    a.W = w.w_in;
    a.N = d.gdn_in_rows;
    a.x = b.xres + static_cast<size_t>(slot) * d.H;
    a.gamma = w.in_norm;
    a.eps = d.eps;
    float* ring = b.ring + (static_cast<size_t>(w.sub) * d.max_seqs + slot) * kConvRing * d.qkv_dim;
    a.seg[0] = GemvSeg{ring, nullptr, d.qkv_dim, ACT_STORE, d.qkv_dim};
    a.seg[1] = GemvSeg{b.z, nullptr, d.qkv_dim + d.z_dim, ACT_SILU, 0};
    a.seg[2] = GemvSeg{b.ab, nullptr, d.gdn_in_rows, ACT_STORE, 0};
    a.nseg = 3;
    a.pos = b.pos + slot;
    a.err = b.err;
    return launch_gemv(lc, d.H, PRO_RMSNORM, a);
}

cudaError_t launch_gdn_out(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                           const Buffers& b, int slot) {
    GemvArgs a{};
    a.W = w.w_out;
    a.N = d.H;
    a.hn_o = b.o;
    a.hn_z = b.z;
    a.hn_w = w.gdn_norm;
    a.hn_dim = d.dv;
    a.eps = d.eps;
    a.seg[0] = GemvSeg{b.xmid + static_cast<size_t>(slot) * d.H,
                       b.xres + static_cast<size_t>(slot) * d.H, d.H, ACT_RESID, 0};
    a.nseg = 1;
    a.err = b.err;
    return launch_gemv(lc, d.z_dim, PRO_HEADNORM, a);
}

cudaError_t launch_attn_in(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                           const Buffers& b, int slot) {
    GemvArgs a{};
    a.W = w.w_in;
    a.N = d.attn_in_rows;
    a.x = b.xres + static_cast<size_t>(slot) * d.H;
    a.gamma = w.in_norm;
    a.eps = d.eps;
    const int qg_rows = 2 * d.Hq * d.D;
    a.seg[0] = GemvSeg{b.qg, nullptr, qg_rows, ACT_STORE, 0};
    a.seg[1] = GemvSeg{b.kvnew, nullptr, d.attn_in_rows, ACT_STORE, 0};
    a.nseg = 2;
    a.err = b.err;
    return launch_gemv(lc, d.H, PRO_RMSNORM, a);
}

cudaError_t launch_attn_out(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                            const Buffers& b, int slot) {
    GemvArgs a{};
    a.W = w.w_out;
    a.N = d.H;
    a.x = b.attn_out;
    a.seg[0] = GemvSeg{b.xmid + static_cast<size_t>(slot) * d.H,
                       b.xres + static_cast<size_t>(slot) * d.H, d.H, ACT_RESID, 0};
    a.nseg = 1;
    a.err = b.err;
    return launch_gemv(lc, d.Hq * d.D, PRO_COPY, a);
}

cudaError_t launch_head(const LaunchCfg& lc, const Dims& d, const uint16_t* final_norm,
                        const uint16_t* lm_head, const Buffers& b, int slot, int advance,
                        int record_gen) {
    GemvArgs a{};
    a.W = lm_head;
    a.N = d.V;
    a.x = b.xres + static_cast<size_t>(slot) * d.H;
    a.gamma = final_norm;
    a.eps = d.eps;
    a.seg[0] = GemvSeg{b.logits, nullptr, d.V, ACT_ARGMAX, 0};
    a.nseg = 1;
    a.cand_val = b.cand_val;
    a.cand_idx = b.cand_idx;
    a.counter = b.counters + kCntHead;
    a.token_out = b.token + slot;
    a.pos_inc = advance ? b.pos + slot : nullptr;
    a.gen_out = record_gen ? b.gen_out : nullptr;
    a.gen_idx = b.gen_idx;
    a.gen_cap = b.gen_capacity;
    a.err = b.err;
    return launch_gemv(lc, d.H, PRO_RMSNORM, a);
}

}  // namespace dm
