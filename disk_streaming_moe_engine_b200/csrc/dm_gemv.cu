// dm_gemv.cu — bf16-weight GEMV for the decode step (batch 1), HBM-bound.
//
// y[r] = sum_k W[r, k] * xs[k]   for r in [0, N),  W bf16 row-major, xs fp32 in smem.
//
// One CTA per SM (grid = min(#SMs, N/4)), each owning a contiguous row range so that its
// weights are one contiguous byte range.  A producer warp streams that range through a
// ring of shared-memory stages with 1-D bulk copies (cp.async.bulk -> mbarrier
// complete_tx); four consumer warps each reduce one row of every stage.  The producer
// does not wait for the previous kernel (weights are read-only), so under programmatic
// dependent launch the first NSTAGE stages are in flight while the previous kernel of the
// decode step is still finishing.  Consumers wait (griddepcontrol.wait) before reading
// activations.
//
// Prologues build xs from the previous kernel's output:
//   PRO_RMSNORM   xs = (x / sqrt(mean(x^2) + eps)) * gamma         (reference rmsnorm.mojo:10)
//   PRO_HEADNORM  xs[h*dv+d] = o*rsqrt(mean_h(o^2)+eps)*w[d]*z     (reference gdn.mojo:1134-1153)
//   PRO_COPY      xs = x
// Epilogues are per row segment: store, SiLU, residual add, ring-slot store (GDN conv
// window) or logits + argmax (first maximum wins, reference cmd_decode.mojo:115).
#include "dm_common.cuh"
#include "dm_kernels.h"

namespace dm {

template <int K>
struct GemvGeom {
    static constexpr int ROW_BYTES = K * 2;
    static constexpr int STAGE_BYTES = kGemvRowsPerStage * ROW_BYTES;
    static constexpr int RING_BUDGET = 96 * 1024;
    static constexpr int NSTAGE_RAW = RING_BUDGET / STAGE_BYTES;
    static constexpr int NSTAGE = NSTAGE_RAW < 2 ? 2 : (NSTAGE_RAW > 8 ? 8 : NSTAGE_RAW);
    static constexpr int RING_BYTES = NSTAGE * STAGE_BYTES;
    static constexpr int XS_BYTES = K * 4;
    static constexpr int BAR_BYTES = 2 * NSTAGE * 8;
    static constexpr int SMEM = RING_BYTES + XS_BYTES + BAR_BYTES;
};

// Canonical RMSNorm reduction order (also restated by the CPU oracle): 128 virtual
// threads, thread t accumulates x[k]^2 for k = t, t+128, ... with fma; four butterfly
// warp sums; ((w0 + w1) + w2) + w3; denom = sqrt(ss / n + eps); y = (x / denom) * gamma.
// `tid` in [0, 128) and the 128 threads must be the four consumer warps.
__device__ __forceinline__ float rms_denominator(const float* x, int n, float eps, int tid,
                                                 float* red4) {
    float acc = 0.0f;
    for (int k = tid; k < n; k += 128) acc = __fmaf_rn(x[k], x[k], acc);
    acc = warp_sum(acc);
    if ((tid & 31) == 0) red4[tid >> 5] = acc;
    named_bar_sync(1, 128);
    float ss = __fadd_rn(__fadd_rn(__fadd_rn(red4[0], red4[1]), red4[2]), red4[3]);
    return __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(n)), eps));
}

// xs split layout: float4 lo[K/8] holds x[8j..8j+3], hi[K/8] holds x[8j+4..8j+7], so a
// lane reading its 8 elements touches consecutive 16-byte words (no bank conflicts).
__device__ __forceinline__ void xs_store(float* xs, int K, int k, float v) {
    int j = k >> 3, e = k & 7;
    xs[(e < 4 ? 0 : K / 2) + j * 4 + (e & 3)] = v;
}

template <int K, int PRO>
__global__ void __launch_bounds__(160, 1) gemv_bf16_kernel(const __grid_constant__ GemvArgs a) {
    using G = GemvGeom<K>;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;
    float* xs = reinterpret_cast<float*>(smem + G::RING_BYTES);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::RING_BYTES + G::XS_BYTES);
    uint64_t* empty = full + G::NSTAGE;
    __shared__ float red4[4];
    __shared__ int abort_flag;
    __shared__ float cand_v[4];
    __shared__ int cand_i[4];
    __shared__ int is_last;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = static_cast<int>(static_cast<int64_t>(blockIdx.x) * a.N / gridDim.x);
    const int r1 = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * a.N / gridDim.x);
    const int nst = (r1 - r0 + kGemvRowsPerStage - 1) / kGemvRowsPerStage;

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::NSTAGE; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 4);
        }
        abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == 4) {  // ---------------- producer ----------------
        if (lane == 0) {
            int issued = 0;
            for (int st = 0; st < nst; ++st) {
                const int slot = st % G::NSTAGE;
                if (st >= G::NSTAGE &&
                    !mbar_wait_bounded(&empty[slot], ((st / G::NSTAGE) - 1) & 1, a.err, &abort_flag))
                    break;
                const int row = r0 + st * kGemvRowsPerStage;
                const int rows = min(kGemvRowsPerStage, r1 - row);
                const uint32_t bytes = static_cast<uint32_t>(rows) * G::ROW_BYTES;
                mbar_arrive_expect_tx(&full[slot], bytes);
                bulk_g2s(ring + slot * G::STAGE_BYTES, a.W + static_cast<size_t>(row) * K, bytes,
                         &full[slot]);
                issued = st + 1;
            }
            if (abort_flag) {  // drain copies that may still be in flight, bounded
                for (int st = max(0, issued - G::NSTAGE); st < issued; ++st)
                    mbar_wait_bounded(&full[st % G::NSTAGE], (st / G::NSTAGE) & 1, a.err, nullptr);
            }
        }
        return;
    }

    // ---------------- consumers (threads 0..127) ----------------
    pdl_wait();
    const int tid = threadIdx.x;
    if (PRO == PRO_RMSNORM) {
        const float denom = rms_denominator(a.x, K, a.eps, tid, red4);
        for (int k = tid; k < K; k += 128) {
            const float y = __fmul_rn(__fdiv_rn(a.x[k], denom), bf16_to_f32(a.gamma[k]));
            xs_store(xs, K, k, y);
            if (a.xnorm_out && blockIdx.x == 0) a.xnorm_out[k] = y;
        }
    } else if (PRO == PRO_HEADNORM) {
        const int dv = a.hn_dim, nh = K / dv;
        for (int h = warp; h < nh; h += 4) {
            const float* oh = a.hn_o + h * dv;
            float acc = 0.0f;
            for (int d = lane; d < dv; d += 32) acc = __fmaf_rn(oh[d], oh[d], acc);
            acc = warp_sum(acc);
            const float rs = 1.0f / sqrtf(acc / static_cast<float>(dv) + a.eps);
            for (int d = lane; d < dv; d += 32) {
                const float nrm = oh[d] * rs * bf16_to_f32(a.hn_w[d]);
                xs_store(xs, K, h * dv + d, nrm * a.hn_z[h * dv + d]);
            }
        }
    } else {
        for (int k = tid; k < K; k += 128) xs_store(xs, K, k, a.x[k]);
    }
    named_bar_sync(1, 128);
    pdl_launch_dependents();

    const int ring_slot = a.pos ? (*a.pos & (kConvRing - 1)) : 0;
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    const float4* xlo = reinterpret_cast<const float4*>(xs);
    const float4* xhi = reinterpret_cast<const float4*>(xs + K / 2);

    for (int st = 0; st < nst; ++st) {
        const int slot = st % G::NSTAGE;
        if (!mbar_wait_bounded(&full[slot], (st / G::NSTAGE) & 1, a.err, &abort_flag)) break;
        const int row = r0 + st * kGemvRowsPerStage + warp;
        if (row < r1) {
            const uint4* wrow =
                reinterpret_cast<const uint4*>(ring + slot * G::STAGE_BYTES + warp * G::ROW_BYTES);
            float acc0 = 0.0f, acc1 = 0.0f;
#pragma unroll
            for (int i = 0; i < K / 256; ++i) {
                const int j = lane + 32 * i;
                const uint4 w = wrow[j];
                const float4 x0 = xlo[j], x1 = xhi[j];
                acc0 = fmaf(bf16lo(w.x), x0.x, acc0);
                acc1 = fmaf(bf16hi(w.x), x0.y, acc1);
                acc0 = fmaf(bf16lo(w.y), x0.z, acc0);
                acc1 = fmaf(bf16hi(w.y), x0.w, acc1);
                acc0 = fmaf(bf16lo(w.z), x1.x, acc0);
                acc1 = fmaf(bf16hi(w.z), x1.y, acc1);
                acc0 = fmaf(bf16lo(w.w), x1.z, acc0);
                acc1 = fmaf(bf16hi(w.w), x1.w, acc1);
            }
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
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }

    if (a.counter == nullptr) return;
    // ---- argmax across the grid: per-CTA candidate, last CTA reduces ----
    if (lane == 0) {
        cand_v[warp] = best_v;
        cand_i[warp] = best_i;
    }
    named_bar_sync(1, 128);
    if (tid == 0) {
        float bv = cand_v[0];
        int bi = cand_i[0];
        for (int w = 1; w < 4; ++w)
            if (cand_v[w] > bv || (cand_v[w] == bv && cand_i[w] < bi)) { bv = cand_v[w]; bi = cand_i[w]; }
        a.cand_val[blockIdx.x] = bv;
        a.cand_idx[blockIdx.x] = bi;
        __threadfence();
        const unsigned prev = atomicAdd(a.counter, 1u);
        is_last = (prev == gridDim.x - 1);
    }
    named_bar_sync(1, 128);
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
static cudaError_t launch_gemv_t(const LaunchCfg& lc, const GemvArgs& a) {
    using G = GemvGeom<K>;
    const int want = (a.N + kGemvRowsPerStage - 1) / kGemvRowsPerStage;
    int grid = want < lc.num_sms ? want : lc.num_sms;
    if (a.counter && grid > kMaxCtas) grid = kMaxCtas;
    return launch_kernel(lc, gemv_bf16_kernel<K, PRO>, dim3(grid), dim3(160), G::SMEM, a);
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

template <int K>
static cudaError_t set_attrs_k() {
    using G = GemvGeom<K>;
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(gemv_bf16_kernel<K, PRO_RMSNORM>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM)) != cudaSuccess)
        return e;
    if ((e = cudaFuncSetAttribute(gemv_bf16_kernel<K, PRO_HEADNORM>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM)) != cudaSuccess)
        return e;
    return cudaFuncSetAttribute(gemv_bf16_kernel<K, PRO_COPY>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM);
}

// Called once per device before any launch (outside stream capture).
cudaError_t gemv_set_attrs() {
    cudaError_t e;
    if ((e = set_attrs_k<256>()) != cudaSuccess) return e;
    if ((e = set_attrs_k<512>()) != cudaSuccess) return e;
    if ((e = set_attrs_k<1024>()) != cudaSuccess) return e;
    if ((e = set_attrs_k<2048>()) != cudaSuccess) return e;
    return set_attrs_k<4096>();
}

bool gemv_supported_k(int K) {
    return K == 256 || K == 512 || K == 1024 || K == 2048 || K == 4096;
}

// ---------------------------------------------------------------------------------------
// Embedding gather: xres[slot] = fp32(embed[token])  (reference gguf_embed_tokens,
// gguf_port_loader.mojo:274).  Token outside [0, V) raises DM_DEVERR_TOKEN and embeds 0.
__global__ void __launch_bounds__(256) embed_kernel(const uint16_t* __restrict__ embed, int H, int V,
                                                    const int* token, float* x, uint32_t* err) {
    pdl_wait();
    int t = *token;
    if (t < 0 || t >= V) {
        if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(err, DM_DEVERR_TOKEN);
        t = 0;
    }
    pdl_launch_dependents();
    const uint16_t* row = embed + static_cast<size_t>(t) * H;
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < H; k += gridDim.x * blockDim.x)
        x[k] = bf16_to_f32(row[k]);
}

cudaError_t launch_embed(const LaunchCfg& lc, const Dims& d, const uint16_t* embed,
                         const Buffers& b, int slot) {
    const int blocks = (d.H + 255) / 256;
    return launch_kernel(lc, embed_kernel, dim3(blocks), dim3(256), 0, embed, d.H, d.V,
                         b.token + slot, b.xres + static_cast<size_t>(slot) * d.H, b.err);
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
