// dm_gdn.cu — fused Gated DeltaNet decode step (one token) on sm_100a.
//
// Semantics of reference forward_gdn_block (src/layers/gdn.mojo:897-1183, steps 3 and 5)
// carried across tokens:
//   conv:  u[c] = SiLU( sum_{j<4} w[c][j] * p[t-3+j][c] )   p = pre-conv projection,
//          p[t'] = 0 for t' < 0 (the conv window is a 4-slot ring indexed by position % 4)
//   gate:  g = exp(-exp(A_log[h]) * softplus(a[h] + dt_bias[h]))   softplus thresholds
//          +-20 as reference _gdn_softplus (gdn.mojo:889-894);  beta = sigmoid(b[h])
//   heads: V head h reads q, k of QK head h / (nv / nk) (gdn.mojo:1054-1070)
//          k <- k / (||k|| + eps), q unnormalised
//   state: sk = S k;  S <- g * (S - beta * sk k^T) + beta * v k^T;  o = S q
//          (S row = dv index, column = dk index; gdn.mojo:1084-1132)
//
// Grid (nv, dv / 16): each CTA owns 16 rows of one head's state, so the update and the
// row-dot for o are CTA-local and the state makes exactly one HBM round trip per token.
// The rows are loaded before griddepcontrol.wait (the state was written by an earlier
// step), overlapping the previous kernel.
#include "dm_common.cuh"
#include "dm_kernels.h"

namespace dm {

struct GdnRecArgs {
    const float* ring;      // [4][qkv_dim] for (layer, slot)
    const uint16_t* conv_w; // [qkv_dim][conv_k]
    float* S;               // [nv][dv][dk] for (layer, slot)
    const float* a_log;
    const float* dt_bias;
    const float* ab;        // a[nv] then b[nv]
    float* o;               // [nv*dv]
    const int* pos;
    int nk, nv, qkv_dim;
    float eps;
    const void* next_w;     // out_proj weights, prefetched into L2
    size_t next_bytes;
    uint64_t* kt;
};

__device__ __forceinline__ float softplus_ref(float v) {
    if (v > 20.0f) return v;
    if (v < -20.0f) return expf(v);
    return logf(1.0f + expf(v));
}

template <int DK>
__global__ void __launch_bounds__(128) gdn_rec_kernel(const __grid_constant__ GdnRecArgs a) {
    constexpr int DV = DK;
    constexpr int RB = 16;          // state rows per CTA
    constexpr int CPL = DK / 32;    // columns per lane
    __shared__ float qs[DK], ks[DK], vs[RB];
    const int h = blockIdx.x, rb = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g_qk = h / (a.nv / a.nk);

    kt_start(a.kt);
    prefetch_l2_share(a.next_w, a.next_bytes, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y,
                      threadIdx.x);
    // ---- prologue: this CTA's state rows (4 per warp) into registers ----
    float* Sh = a.S + static_cast<size_t>(h) * DV * DK;
    float srow[4][CPL];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = rb * RB + warp * 4 + i;
        const float* src = Sh + static_cast<size_t>(r) * DK + lane * CPL;
        if (CPL == 4) {
            const float4 t = *reinterpret_cast<const float4*>(src);
            srow[i][0] = t.x; srow[i][1] = t.y; srow[i][2] = t.z; srow[i][3] = t.w;
        } else {
#pragma unroll
            for (int c = 0; c < CPL; ++c) srow[i][c] = src[c];
        }
    }
    const float alog = a.a_log[h], dtb = a.dt_bias[h];  // weights: before the wait
    pdl_wait();
    kt_ready(a.kt);
    const int pos = *a.pos;
    const float av = a.ab[h], bv = a.ab[a.nv + h];

    // ---- causal conv + SiLU for q (DK), k (DK) and this CTA's 16 v channels ----
    const int q0 = g_qk * DK, k0 = a.nk * DK + g_qk * DK, v0 = 2 * a.nk * DK + h * DV + rb * RB;
    for (int t = threadIdx.x; t < 2 * DK + RB; t += 128) {
        const int ch = t < DK ? q0 + t : (t < 2 * DK ? k0 + (t - DK) : v0 + (t - 2 * DK));
        const uint16_t* w = a.conv_w + static_cast<size_t>(ch) * 4;
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int tp = pos - 3 + j;
            if (tp >= 0) acc += bf16_to_f32(w[j]) * a.ring[static_cast<size_t>(tp & 3) * a.qkv_dim + ch];
        }
        const float u = silu_f(acc);
        if (t < DK) qs[t] = u;
        else if (t < 2 * DK) ks[t - DK] = u;
        else vs[t - 2 * DK] = u;
    }
    __syncthreads();
    pdl_launch_dependents();

    // ---- k normalisation, decay, beta ----
    float kl[CPL], ql[CPL];
    float ss = 0.0f;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
        kl[c] = ks[lane * CPL + c];
        ql[c] = qs[lane * CPL + c];
        ss = fmaf(kl[c], kl[c], ss);
    }
    ss = warp_sum(ss);
    const float inv_nk = 1.0f / (sqrtf(ss) + a.eps);
#pragma unroll
    for (int c = 0; c < CPL; ++c) kl[c] *= inv_nk;
    const float g = expf(-expf(alog) * softplus_ref(av + dtb));
    const float beta = sigmoid_f(bv);

    // ---- delta-rule update and o = S q, one row at a time per warp ----
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int rl = warp * 4 + i;
        const int r = rb * RB + rl;
        float sk = 0.0f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) sk = fmaf(srow[i][c], kl[c], sk);
        sk = warp_sum(sk);
        const float vr = vs[rl];
        const float bsk = beta * sk, bvr = beta * vr;
        float oacc = 0.0f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
            const float sn = g * (srow[i][c] - bsk * kl[c]) + bvr * kl[c];
            srow[i][c] = sn;
            oacc = fmaf(sn, ql[c], oacc);
        }
        oacc = warp_sum(oacc);
        float* dst = Sh + static_cast<size_t>(r) * DK + lane * CPL;
        if (CPL == 4) {
            *reinterpret_cast<float4*>(dst) = make_float4(srow[i][0], srow[i][1], srow[i][2], srow[i][3]);
        } else {
#pragma unroll
            for (int c = 0; c < CPL; ++c) dst[c] = srow[i][c];
        }
        if (lane == 0) a.o[h * DV + r] = oacc;
    }
    if (a.kt) {
        __syncthreads();
        kt_end(a.kt);
    }
}

cudaError_t launch_gdn_rec(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                           const Buffers& b, int slot) {
    GdnRecArgs a{};
    const size_t ls = static_cast<size_t>(w.sub) * d.max_seqs + slot;
    a.ring = b.ring + ls * kConvRing * d.qkv_dim;
    a.conv_w = w.conv_w;
    a.S = b.S + ls * static_cast<size_t>(d.nv) * d.dv * d.dk;
    a.a_log = w.a_log;
    a.dt_bias = w.dt_bias;
    a.ab = b.ab;
    a.o = b.o;
    a.pos = b.pos + slot;
    a.nk = d.nk;
    a.nv = d.nv;
    a.qkv_dim = d.qkv_dim;
    a.eps = d.eps;
    a.next_w = lc.l2_prefetch ? w.w_out : nullptr;
    a.next_bytes = static_cast<size_t>(d.H) * d.z_dim * 2;
    a.kt = lc.kt;
    const dim3 grid(d.nv, d.dv / 16);
    if (d.dk == 128) return launch_kernel(lc, gdn_rec_kernel<128>, grid, dim3(128), 0, a);
    if (d.dk == 64) return launch_kernel(lc, gdn_rec_kernel<64>, grid, dim3(128), 0, a);
    return cudaErrorInvalidValue;
}

}  // namespace dm
