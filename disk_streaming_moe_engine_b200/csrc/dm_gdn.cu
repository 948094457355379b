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
    uint64_t* kt;
    // batched launch (grid.z = batch rows): row b works on sequence slots[b]; ring, S and
    // pos advance by the slot, ab and o by the row.  slots == nullptr: one sequence.
    const int* slots;
    size_t ring_ss, S_ss;
    int ab_bs, o_bs;
};


// RPW state rows per warp, NW warps: RB = RPW * NW rows of one head per CTA (the batched
// step takes all dv rows in one CTA, so the conv, the k norm and the gates of a (row, head)
// are computed once instead of once per 16-row block).
template <int DK, int RPW = 4, int NW = 4>
__global__ void __launch_bounds__(NW * 32) gdn_rec_kernel(const __grid_constant__ GdnRecArgs a) {
    constexpr int DV = DK;
    constexpr int RB = RPW * NW;    // state rows per CTA
    constexpr int NT = NW * 32;
    constexpr int CPL = DK / 32;    // columns per lane
    __shared__ float qs[DK], ks[DK], vs[RB];
    const int h = blockIdx.x, rb = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g_qk = h / (a.nv / a.nk);
    const int bz = blockIdx.z;
    const int slot = a.slots ? a.slots[bz] : 0;  // host-written before the step
    const float* ring = a.ring + slot * a.ring_ss;
    const float* ab = a.ab + bz * a.ab_bs;
    float* o_out = a.o + bz * a.o_bs;

    kt_start(a.kt);
    // ---- prologue: this CTA's state rows (4 per warp) into registers ----
    float* Sh = a.S + slot * a.S_ss + static_cast<size_t>(h) * DV * DK;
    float srow[RPW][CPL];
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        const int r = rb * RB + warp * RPW + i;
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
    const int pos = a.pos[slot];
    const float av = ab[h], bv = ab[a.nv + h];

    // ---- causal conv + SiLU for q (DK), k (DK) and this CTA's 16 v channels ----
    const int q0 = g_qk * DK, k0 = a.nk * DK + g_qk * DK, v0 = 2 * a.nk * DK + h * DV + rb * RB;
    for (int t = threadIdx.x; t < 2 * DK + RB; t += NT) {
        const int ch = t < DK ? q0 + t : (t < 2 * DK ? k0 + (t - DK) : v0 + (t - 2 * DK));
        const uint16_t* w = a.conv_w + static_cast<size_t>(ch) * 4;
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int tp = pos - 3 + j;
            if (tp >= 0) acc += bf16_to_f32(w[j]) * ring[static_cast<size_t>(tp & 3) * a.qkv_dim + ch];
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
    for (int i = 0; i < RPW; ++i) {
        const int rl = warp * RPW + i;
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
        if (lane == 0) o_out[h * DV + r] = oacc;
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
    a.kt = lc.kt;
    const dim3 grid(d.nv, d.dv / 16);
    if (d.dk == 128) return launch_kernel(lc, gdn_rec_kernel<128>, grid, dim3(128), 0, a);
    if (d.dk == 64) return launch_kernel(lc, gdn_rec_kernel<64>, grid, dim3(128), 0, a);
    return cudaErrorInvalidValue;
}

cudaError_t launch_gdn_rec_batch(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& bb,
                                 const Buffers& b, int n) {
    GdnRecArgs a{};
    const size_t ls = static_cast<size_t>(w.sub) * d.max_seqs;
    a.ring = b.ring + ls * kConvRing * d.qkv_dim;
    a.conv_w = w.conv_w;
    a.S = b.S + ls * static_cast<size_t>(d.nv) * d.dv * d.dk;
    a.a_log = w.a_log;
    a.dt_bias = w.dt_bias;
    a.ab = bb.ab;
    a.o = bb.o;
    a.pos = b.pos;
    a.nk = d.nk;
    a.nv = d.nv;
    a.qkv_dim = d.qkv_dim;
    a.eps = d.eps;
    a.kt = lc.kt;
    a.slots = bb.slots;
    a.ring_ss = static_cast<size_t>(kConvRing) * d.qkv_dim;
    a.S_ss = static_cast<size_t>(d.nv) * d.dv * d.dk;
    a.ab_bs = 2 * d.nv;
    a.o_bs = d.z_dim;
    // one CTA per (row, head): all dv state rows, 16 warps x dv / 16 rows
    const dim3 grid(d.nv, 1, n);
    if (d.dk == 128 && d.dv == 128) return launch_kernel(lc, gdn_rec_kernel<128, 8, 16>, grid, dim3(512), 0, a);
    if (d.dk == 64 && d.dv == 64) return launch_kernel(lc, gdn_rec_kernel<64, 4, 16>, grid, dim3(512), 0, a);
    return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------------------
// GDN recurrence + output projection in one kernel (grid = #SMs, all CTAs co-resident).
//   pre-wait  each CTA copies its contiguous block of out-projection rows into shared
//             memory (one 1-D bulk copy per row): the projection's weights stream while
//             the input projection and the recurrence run; each 128-thread group loads the
//             state rows of its recurrence item (nv x dv/16 items: item = group * G + CTA)
//   phase 1   the recurrence of gdn_rec_kernel per item (named barrier per group)
//   barrier   grid-wide (release add + bounded acquire spin)
//   phase 2   every CTA: head RMSNorm * w * SiLU(z) of the full o, then its rows of
//             W_out from shared memory, + residual (one row per warp)
//   exit      the last CTA out resets the counters for the next launch
struct GdnFusedArgs {
    GdnRecArgs rec;
    const uint16_t* W_out;  // [H][nv*dv]
    const float* z;         // [nv*dv] SiLU(z) from the input projection
    const uint16_t* gnorm;  // [dv]
    const float* x_res;     // [H]
    float* x_mid;           // [H]
    int H, rmax;
    unsigned long long* arrivals;  // grid-barrier arrivals of every launch so far (never reset)
    uint64_t* trace;        // phase stamps: [0..7] CTA 0, [8..15] latest over the CTAs; or null
    uint32_t* err;
};

constexpr int kGfThreads = 512;

// Phase k of the fused GDN kernel reached by this CTA (thread 0): CTA 0's time in slot k,
// the latest CTA's in slot 8 + k.  Phases: 0 start, 1 wait released, 2 recurrence done,
// 3 grid barrier passed, 4 head norm done, 5 out-projection rows landed, 6 end.
DM_DEV void gdn_stamp(uint64_t* tr, int k) {
    if (tr == nullptr || threadIdx.x != 0) return;
    const unsigned long long t = globaltimer_ns();
    if (blockIdx.x == 0) tr[k] = t;
    atomicMax(reinterpret_cast<unsigned long long*>(tr + 8 + k), t);
}

template <int DK>
__global__ void __launch_bounds__(kGfThreads, 1) gdn_core_out_kernel(const __grid_constant__ GdnFusedArgs f) {
    constexpr int DV = DK;
    constexpr int RB = 16;
    constexpr int CPL = DK / 32;
    const GdnRecArgs& a = f.rec;
    extern __shared__ __align__(128) uint8_t gsm[];
    __shared__ float qs[4][DK], ks[4][DK], vs[4][RB];
    __shared__ __align__(8) uint64_t wbar;
    __shared__ unsigned long long s_gen;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int grp = warp >> 2, gw = warp & 3, gt = tid & 127;
    const int c = blockIdx.x, G = gridDim.x;
    const int KO = a.nv * DV;
    const int r0 = static_cast<int>(static_cast<long long>(c) * f.H / G);
    const int r1 = static_cast<int>(static_cast<long long>(c + 1) * f.H / G);
    const int nr = r1 - r0;
    uint8_t* wsm = gsm;                                                       // [rmax][KO] bf16
    float* xs = reinterpret_cast<float*>(gsm + static_cast<size_t>(f.rmax) * KO * 2);  // [KO]
    kt_start(a.kt);
    gdn_stamp(f.trace, 0);

    if (tid == 0) {
        mbar_init(&wbar, 1);
        mbar_fence_init();
        if (nr > 0) {
            mbar_arrive_expect_tx(&wbar, static_cast<uint32_t>(nr) * KO * 2);
            for (int r = 0; r < nr; ++r)
                bulk_g2s(wsm + static_cast<size_t>(r) * KO * 2, f.W_out + static_cast<size_t>(r0 + r) * KO, KO * 2, &wbar);
        } else {
            mbar_arrive(&wbar);
        }
    }
    // this group's recurrence item
    const int nrb = DV / RB;
    const int item = grp * G + c;
    const bool has_item = item < a.nv * nrb;
    const int h = has_item ? item / nrb : 0, rb = has_item ? item % nrb : 0;
    const int g_qk = h / (a.nv / a.nk);
    float* Sh = a.S + static_cast<size_t>(h) * DV * DK;
    float srow[4][CPL];
    float alog = 0.0f, dtb = 0.0f;
    if (has_item) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float* src = Sh + static_cast<size_t>(rb * RB + gw * 4 + i) * DK + lane * CPL;
#pragma unroll
            for (int cc = 0; cc < CPL; ++cc) srow[i][cc] = src[cc];
        }
        alog = a.a_log[h];
        dtb = a.dt_bias[h];
    }
    pdl_wait();
    kt_ready(a.kt);
    gdn_stamp(f.trace, 1);
    // launch generation: the arrival count (grown by G per launch, never reset) read before
    // this CTA arrives, when fewer than G arrivals of this launch can have happened
    if (tid == 0) s_gen = ld_relaxed_u64(f.arrivals) / static_cast<unsigned long long>(G);

    // ---- phase 1: recurrence ----
    if (has_item) {
        const int pos = *a.pos;
        const float av = a.ab[h], bv = a.ab[a.nv + h];
        const int q0 = g_qk * DK, k0 = a.nk * DK + g_qk * DK, v0 = 2 * a.nk * DK + h * DV + rb * RB;
        for (int t = gt; t < 2 * DK + RB; t += 128) {
            const int ch = t < DK ? q0 + t : (t < 2 * DK ? k0 + (t - DK) : v0 + (t - 2 * DK));
            const uint16_t* w = a.conv_w + static_cast<size_t>(ch) * 4;
            float acc = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int tp = pos - 3 + j;
                if (tp >= 0) acc += bf16_to_f32(w[j]) * a.ring[static_cast<size_t>(tp & 3) * a.qkv_dim + ch];
            }
            const float u = silu_f(acc);
            if (t < DK) qs[grp][t] = u;
            else if (t < 2 * DK) ks[grp][t - DK] = u;
            else vs[grp][t - 2 * DK] = u;
        }
        named_bar_sync(1 + grp, 128);
        float kl[CPL], ql[CPL];
        float ss = 0.0f;
#pragma unroll
        for (int cc = 0; cc < CPL; ++cc) {
            kl[cc] = ks[grp][lane * CPL + cc];
            ql[cc] = qs[grp][lane * CPL + cc];
            ss = fmaf(kl[cc], kl[cc], ss);
        }
        ss = warp_sum(ss);
        const float inv_nk = 1.0f / (sqrtf(ss) + a.eps);
#pragma unroll
        for (int cc = 0; cc < CPL; ++cc) kl[cc] *= inv_nk;
        const float g = expf(-expf(alog) * softplus_ref(av + dtb));
        const float beta = sigmoid_f(bv);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int rl = gw * 4 + i;
            const int r = rb * RB + rl;
            float sk = 0.0f;
#pragma unroll
            for (int cc = 0; cc < CPL; ++cc) sk = fmaf(srow[i][cc], kl[cc], sk);
            sk = warp_sum(sk);
            const float vr = vs[grp][rl];
            const float bsk = beta * sk, bvr = beta * vr;
            float oacc = 0.0f;
#pragma unroll
            for (int cc = 0; cc < CPL; ++cc) {
                const float sn = g * (srow[i][cc] - bsk * kl[cc]) + bvr * kl[cc];
                srow[i][cc] = sn;
                oacc = fmaf(sn, ql[cc], oacc);
            }
            oacc = warp_sum(oacc);
            float* dst = Sh + static_cast<size_t>(r) * DK + lane * CPL;
#pragma unroll
            for (int cc = 0; cc < CPL; ++cc) dst[cc] = srow[i][cc];
            if (lane == 0) a.o[h * DV + r] = oacc;
        }
    }
    __syncthreads();
    gdn_stamp(f.trace, 2);
    pdl_launch_dependents();
    if (tid == 0) {
        const unsigned long long target = (s_gen + 1) * static_cast<unsigned long long>(G);
        __threadfence();
        red_release_add_u64(f.arrivals, 1ull);
        spin_geq_u64(f.arrivals, target, f.err);
    }
    __syncthreads();
    gdn_stamp(f.trace, 3);

    // ---- phase 2: head RMSNorm * w * SiLU(z) of the whole o (dv <= 128).  Warp w takes
    // heads w and w + 16 and issues the loads of both before reducing either, so the
    // phase waits for one L2 round trip, not two ----
    float* xlo = xs;
    float* xhi = xs + KO / 2;
    constexpr int NW = kGfThreads / 32;
    for (int hh0 = warp; hh0 < a.nv; hh0 += 2 * NW) {
        float ov[2][4], zv[2][4], wv[4];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int hh = hh0 + u * NW;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int d = lane + 32 * i;
                const bool on = d < DV && hh < a.nv;
                ov[u][i] = on ? __ldcg(a.o + hh * DV + d) : 0.0f;
                zv[u][i] = on ? __ldcg(f.z + hh * DV + d) : 0.0f;
            }
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int d = lane + 32 * i;
            wv[i] = d < DV ? bf16_to_f32(f.gnorm[d]) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int hh = hh0 + u * NW;
            if (hh >= a.nv) break;
            float acc = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) acc = fmaf(ov[u][i], ov[u][i], acc);
            acc = warp_sum(acc);
            const float rs = 1.0f / sqrtf(acc / static_cast<float>(DV) + a.eps);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int d = lane + 32 * i;
                if (d < DV) {
                    const int k = hh * DV + d;  // element 8j + e goes to (e < 4 ? xlo : xhi)[4j + e % 4]
                    (((k & 7) < 4) ? xlo : xhi)[(k >> 3) * 4 + (k & 3)] = ov[u][i] * rs * wv[i] * zv[u][i];
                }
            }
        }
    }
    __syncthreads();
    gdn_stamp(f.trace, 4);
    const bool wok = mbar_wait_bounded(&wbar, 0, f.err, nullptr);
    gdn_stamp(f.trace, 5);
    const float4* x4lo = reinterpret_cast<const float4*>(xlo);
    const float4* x4hi = reinterpret_cast<const float4*>(xhi);
    // warp w takes rows w and w + RH (RH = ceil(nr / 2)), so each activation vector read
    // from shared memory serves two rows (the phase is bound by shared-memory reads)
    const int RH = (nr + 1) / 2;
    for (int r = warp; r < RH; r += kGfThreads / 32) {
        const int r2 = r + RH;
        const bool two = r2 < nr;
        const uint4* wr = reinterpret_cast<const uint4*>(wsm + static_cast<size_t>(r) * KO * 2);
        const uint4* wr2 = reinterpret_cast<const uint4*>(wsm + static_cast<size_t>(two ? r2 : r) * KO * 2);
        float s0 = 0.0f, s1 = 0.0f, t0 = 0.0f, t1 = 0.0f;
        for (int j = lane; j < KO / 8; j += 32) {
            const uint4 w = wr[j];
            const uint4 v = two ? wr2[j] : make_uint4(0u, 0u, 0u, 0u);
            const float4 lo = x4lo[j], hi = x4hi[j];
            s0 = fmaf(bf16lo(w.x), lo.x, s0);
            s1 = fmaf(bf16hi(w.x), lo.y, s1);
            s0 = fmaf(bf16lo(w.y), lo.z, s0);
            s1 = fmaf(bf16hi(w.y), lo.w, s1);
            s0 = fmaf(bf16lo(w.z), hi.x, s0);
            s1 = fmaf(bf16hi(w.z), hi.y, s1);
            s0 = fmaf(bf16lo(w.w), hi.z, s0);
            s1 = fmaf(bf16hi(w.w), hi.w, s1);
            t0 = fmaf(bf16lo(v.x), lo.x, t0);
            t1 = fmaf(bf16hi(v.x), lo.y, t1);
            t0 = fmaf(bf16lo(v.y), lo.z, t0);
            t1 = fmaf(bf16hi(v.y), lo.w, t1);
            t0 = fmaf(bf16lo(v.z), hi.x, t0);
            t1 = fmaf(bf16hi(v.z), hi.y, t1);
            t0 = fmaf(bf16lo(v.w), hi.z, t0);
            t1 = fmaf(bf16hi(v.w), hi.w, t1);
        }
        const float acc = warp_sum(s0 + s1);
        const float acc2 = warp_sum(t0 + t1);
        if (lane == 0) {
            f.x_mid[r0 + r] = f.x_res[r0 + r] + (wok ? acc : 0.0f);
            if (two) f.x_mid[r0 + r2] = f.x_res[r0 + r2] + (wok ? acc2 : 0.0f);
        }
    }
    __syncthreads();
    gdn_stamp(f.trace, 6);
    kt_end(a.kt);  // nothing to reset: the barrier counter is generation-based
}

static size_t gdn_fused_smem(const Dims& d, int G) {
    const int rmax = (d.H + G - 1) / G;
    return static_cast<size_t>(rmax) * d.z_dim * 2 + static_cast<size_t>(d.z_dim) * 4;
}

constexpr size_t kGdnFusedMaxSmem = 200 * 1024;

bool gdn_fused_supported(const Dims& d, int num_sms) {
    return (d.dk == 128 || d.dk == 64) && d.dv == d.dk && d.z_dim % 256 == 0 &&
           d.nv * (d.dv / 16) <= 4 * num_sms && gdn_fused_smem(d, num_sms) <= kGdnFusedMaxSmem;
}

cudaError_t gdn_set_attrs() {
    cudaError_t e = cudaFuncSetAttribute(gdn_core_out_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kGdnFusedMaxSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gdn_core_out_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kGdnFusedMaxSmem));
    return e;
}

// One CTA per SM with a grid-wide barrier between its phases: every CTA must fit on an SM
// at once (queried once per context; the separate-kernel path is used otherwise).
bool gdn_fused_fits(const Dims& d, int num_sms) {
    if (!gdn_fused_supported(d, num_sms)) return false;
    int per_sm = 0;
    const size_t smem = gdn_fused_smem(d, num_sms);
    const cudaError_t e = d.dk == 128
        ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gdn_core_out_kernel<128>, kGfThreads, smem)
        : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gdn_core_out_kernel<64>, kGfThreads, smem);
    return e == cudaSuccess && per_sm >= 1;
}

cudaError_t launch_gdn_core_out(const LaunchCfg& lc, const Dims& d, const LayerW& w, const Buffers& b, int slot) {
    if (!gdn_fused_supported(d, lc.num_sms)) return cudaErrorInvalidValue;
    GdnFusedArgs f{};
    GdnRecArgs& a = f.rec;
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
    a.kt = lc.kt;
    f.W_out = w.w_out;
    f.z = b.z;
    f.gnorm = w.gdn_norm;
    f.x_res = b.xres + static_cast<size_t>(slot) * d.H;
    f.x_mid = b.xmid + static_cast<size_t>(slot) * d.H;
    f.H = d.H;
    const int G = lc.num_sms;
    f.rmax = (d.H + G - 1) / G;
    f.arrivals = reinterpret_cast<unsigned long long*>(b.counters + kCntGdnSync);
    f.err = b.err;
    f.trace = b.trace ? b.trace + kTrGdn : nullptr;
    const size_t smem = gdn_fused_smem(d, G);
    if (d.dk == 128) return launch_kernel(lc, gdn_core_out_kernel<128>, dim3(G), dim3(kGfThreads), smem, f);
    return launch_kernel(lc, gdn_core_out_kernel<64>, dim3(G), dim3(kGfThreads), smem, f);
}

// ---- prefill: the recurrence over a chunk of n prompt tokens of one sequence ------------
// The semantics above applied token after token (reference forward_gdn_block runs its
// recurrence token by token, gdn.mojo:1040-1133), in two kernels:
//   pf_conv_kernel  every (token, channel) at once: causal conv + SiLU of the pre-conv rows
//                   (position p < 0: zero; p < pos0: the conv window, ring slot p % 4; else
//                   row p - pos0 of the chunk), each k head divided by (||k|| + eps)
//                   -> pf_u [n][qkv_dim]
//   pf_gdn_kernel   grid (nv, dv / 16), 128 threads: 16 state rows of one head stay in
//                   registers for the whole chunk, 8 lanes per row (dk / 8 columns each).
//                   Tokens go in blocks of kPfTok: the block's q, k, this CTA's v channels,
//                   decay and beta (computed by the projection's epilogue) are copied into
//                   shared memory with cp.async while the previous block is scanned (two
//                   buffers, one block barrier per block); every warp runs its 4 rows through
//                   the block: sk = S k, sq = S q and k.q from one pass over the row (one
//                   3-level butterfly for the three sums), S <- g (S - beta sk k^T) + beta v
//                   k^T, and o = S_new q = g sq + beta (k.q) (v - g sk).
// pf_ring_kernel then moves the conv window to the chunk's last positions.
constexpr int kPfTok = 16;

struct PfConvArgs {
    const float* raw;       // [n][qkv_dim] pre-conv rows of the chunk
    const float* ring;      // [4][qkv_dim] of (layer, slot)
    const uint16_t* conv_w; // [qkv_dim][4]
    float* u;               // [n][qkv_dim]
    int n, pos0, qkv_dim, k0, k1, dk;
    float eps;
};

__global__ void __launch_bounds__(256) pf_conv_kernel(const __grid_constant__ PfConvArgs a) {
    __shared__ float red[8];
    const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ch = blockIdx.y * 256 + tid;
    pdl_wait();
    pdl_launch_dependents();
    const int pos = a.pos0 + t;
    float u = 0.0f;
    if (ch < a.qkv_dim) {
        const uint16_t* w = a.conv_w + static_cast<size_t>(ch) * 4;
        float acc = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int tp = pos - 3 + j;
            if (tp >= 0) {
                const float pre = tp < a.pos0 ? a.ring[static_cast<size_t>(tp & 3) * a.qkv_dim + ch]
                                              : a.raw[static_cast<size_t>(tp - a.pos0) * a.qkv_dim + ch];
                acc += bf16_to_f32(w[j]) * pre;
            }
        }
        u = silu_f(acc);
    }
    const int blk0 = blockIdx.y * 256;
    if (blk0 + 256 > a.k0 && blk0 < a.k1) {  // the block holds k channels (uniform per block)
        const bool isk = ch >= a.k0 && ch < a.k1;
        const float ss = warp_sum(isk ? u * u : 0.0f);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        const int wpg = a.dk / 32, g0 = (warp / wpg) * wpg;  // the warps of this thread's head
        float tot = 0.0f;
        for (int i = 0; i < wpg; ++i) tot += red[g0 + i];
        if (isk) u *= 1.0f / (sqrtf(tot) + a.eps);
    }
    if (ch < a.qkv_dim) a.u[static_cast<size_t>(t) * a.qkv_dim + ch] = u;
}


struct PfGdnArgs {
    const float* u;         // [n][qkv_dim] conv outputs (k normalised)
    float* S;               // [nv][dv][dk] of (layer, slot)
    const float* gb;        // [n][2 nv]: decay g, then beta, of every V head
    float* o;               // [n][nv dv]
    int n, nk, nv, qkv_dim;
};

template <int DK>
__global__ void __launch_bounds__(128) pf_gdn_kernel(const __grid_constant__ PfGdnArgs a) {
    constexpr int DV = DK;
    constexpr int RB = 16;          // state rows per CTA
    constexpr int CPL = DK / 8;     // columns per lane (8 lanes per row)
    constexpr int NF4 = CPL / 4;    // float4 groups per lane: columns 4 sub + 32 m + i
    static_assert(CPL % 4 == 0, "whole float4 groups");
    // two buffers of one token block: q, k [kPfTok][DK], v [kPfTok][RB], g, beta [kPfTok]
    constexpr int BUF = kPfTok * (2 * DK + RB + 2);
    __shared__ __align__(16) float sm[2 * BUF];
    const int h = blockIdx.x, rb = blockIdx.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int sub = lane & 7, rr = lane >> 3;
    const int rl = warp * 4 + rr;  // row of the CTA
    const int row = rb * RB + rl;
    const int g_qk = h / (a.nv / a.nk);
    float* Srow = a.S + (static_cast<size_t>(h) * DV + row) * DK;
    float s[CPL];
#pragma unroll
    for (int m = 0; m < NF4; ++m) {
        const float4 t = *reinterpret_cast<const float4*>(Srow + 4 * sub + 32 * m);
        s[4 * m] = t.x; s[4 * m + 1] = t.y; s[4 * m + 2] = t.z; s[4 * m + 3] = t.w;
    }
    pdl_wait();
    pdl_launch_dependents();
    const float* uq = a.u + g_qk * DK;
    const float* uk = a.u + a.nk * DK + g_qk * DK;
    const float* uv = a.u + 2 * a.nk * DK + h * DV + rb * RB;
    auto stage = [&](int blk, int buf) {
        const int t0 = blk * kPfTok, nt = min(kPfTok, a.n - t0);
        float* qs = sm + buf * BUF;
        float* ks = qs + kPfTok * DK;
        float* vs = ks + kPfTok * DK;
        float* gs = vs + kPfTok * RB;
        for (int i = tid; i < nt * (DK / 4); i += 128) {
            const int tt = i / (DK / 4), c4 = i % (DK / 4);
            const size_t off = static_cast<size_t>(t0 + tt) * a.qkv_dim + 4 * c4;
            cp_async16(qs + tt * DK + 4 * c4, uq + off);
            cp_async16(ks + tt * DK + 4 * c4, uk + off);
        }
        for (int i = tid; i < nt * (RB / 4); i += 128) {
            const int tt = i / (RB / 4), c4 = i % (RB / 4);
            cp_async16(vs + tt * RB + 4 * c4, uv + static_cast<size_t>(t0 + tt) * a.qkv_dim + 4 * c4);
        }
        for (int i = tid; i < 2 * nt; i += 128) {
            const int tt = i >> 1, which = i & 1;
            cp_async4(gs + which * kPfTok + tt, a.gb + static_cast<size_t>(t0 + tt) * 2 * a.nv + which * a.nv + h);
        }
        cp_async_commit();
    };
    const int nblk = (a.n + kPfTok - 1) / kPfTok;
    stage(0, 0);
    for (int blk = 0; blk < nblk; ++blk) {
        cp_async_wait_all();
        __syncthreads();  // block blk has landed; every warp is done with the other buffer
        if (blk + 1 < nblk) stage(blk + 1, (blk + 1) & 1);
        const float* qs = sm + (blk & 1) * BUF;
        const float* ks = qs + kPfTok * DK;
        const float* vs = ks + kPfTok * DK;
        const float* gs = vs + kPfTok * RB;
        const int t0 = blk * kPfTok, nt = min(kPfTok, a.n - t0);
        for (int tt = 0; tt < nt; ++tt) {
            float kl[CPL], ql[CPL];
#pragma unroll
            for (int m = 0; m < NF4; ++m) {
                const float4 k4 = *reinterpret_cast<const float4*>(ks + tt * DK + 4 * sub + 32 * m);
                const float4 q4 = *reinterpret_cast<const float4*>(qs + tt * DK + 4 * sub + 32 * m);
                kl[4 * m] = k4.x; kl[4 * m + 1] = k4.y; kl[4 * m + 2] = k4.z; kl[4 * m + 3] = k4.w;
                ql[4 * m] = q4.x; ql[4 * m + 1] = q4.y; ql[4 * m + 2] = q4.z; ql[4 * m + 3] = q4.w;
            }
            float sk0 = 0.0f, sk1 = 0.0f, sq0 = 0.0f, sq1 = 0.0f, kq = 0.0f;
#pragma unroll
            for (int c = 0; c < CPL; c += 2) {
                sk0 = fmaf(s[c], kl[c], sk0);
                sk1 = fmaf(s[c + 1], kl[c + 1], sk1);
                sq0 = fmaf(s[c], ql[c], sq0);
                sq1 = fmaf(s[c + 1], ql[c + 1], sq1);
                kq = fmaf(kl[c], ql[c], fmaf(kl[c + 1], ql[c + 1], kq));
            }
            float sk = sk0 + sk1, sq = sq0 + sq1;
#pragma unroll
            for (int m = 4; m >= 1; m >>= 1) {
                sk += __shfl_xor_sync(0xffffffffu, sk, m);
                sq += __shfl_xor_sync(0xffffffffu, sq, m);
                kq += __shfl_xor_sync(0xffffffffu, kq, m);
            }
            const float g = gs[tt], beta = gs[kPfTok + tt], vr = vs[tt * RB + rl];
            const float bsk = beta * sk, bvr = beta * vr;
#pragma unroll
            for (int c = 0; c < CPL; ++c) s[c] = g * (s[c] - bsk * kl[c]) + bvr * kl[c];
            if (sub == 0)
                a.o[static_cast<size_t>(t0 + tt) * a.nv * DV + h * DV + row] = g * sq + beta * kq * (vr - g * sk);
        }
    }
#pragma unroll
    for (int m = 0; m < NF4; ++m)
        *reinterpret_cast<float4*>(Srow + 4 * sub + 32 * m) = make_float4(s[4 * m], s[4 * m + 1], s[4 * m + 2], s[4 * m + 3]);
}

// The conv window after the chunk: the pre-conv rows of its last min(n, 4) positions into
// their ring slots (after pf_conv_kernel, which read the window the chunk started from).
__global__ void __launch_bounds__(256) pf_ring_kernel(const float* __restrict__ raw, float* ring, int n, int pos0,
                                                      int qkv_dim) {
    pdl_wait();
    pdl_launch_dependents();
    const int j = blockIdx.y;  // 0..3: position pos0 + n - 4 + j
    const int p = pos0 + n - 4 + j;
    if (p < pos0) return;
    const float* src = raw + static_cast<size_t>(p - pos0) * qkv_dim;
    float* dst = ring + static_cast<size_t>(p & 3) * qkv_dim;
    for (int c = blockIdx.x * 256 + threadIdx.x; c < qkv_dim; c += gridDim.x * 256) dst[c] = src[c];
}

bool pf_gdn_supported(const Dims& d) {
    return (d.dk == 128 || d.dk == 64) && d.dv == d.dk && 256 % d.dk == 0 && d.qkv_dim % 32 == 0;
}

cudaError_t launch_pf_gdn(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& pb,
                          const Buffers& b, int slot, int pos0, int n) {
    if (!pf_gdn_supported(d)) return cudaErrorInvalidValue;
    const size_t ls = static_cast<size_t>(w.sub) * d.max_seqs + slot;
    float* ring = b.ring + ls * kConvRing * d.qkv_dim;
    PfConvArgs c{};
    c.raw = pb.pf_raw;
    c.ring = ring;
    c.conv_w = w.conv_w;
    c.u = pb.pf_u;
    c.n = n;
    c.pos0 = pos0;
    c.qkv_dim = d.qkv_dim;
    c.k0 = d.nk * d.dk;
    c.k1 = 2 * d.nk * d.dk;
    c.dk = d.dk;
    c.eps = d.eps;
    cudaError_t e = launch_kernel(lc, pf_conv_kernel, dim3(n, (d.qkv_dim + 255) / 256), dim3(256), 0, c);
    if (e != cudaSuccess) return e;
    PfGdnArgs a{};
    a.u = pb.pf_u;
    a.S = b.S + ls * static_cast<size_t>(d.nv) * d.dv * d.dk;
    a.gb = pb.ab;
    a.o = pb.o;
    a.n = n;
    a.nk = d.nk;
    a.nv = d.nv;
    a.qkv_dim = d.qkv_dim;
    const dim3 grid(d.nv, d.dv / 16);
    e = d.dk == 128 ? launch_kernel(lc, pf_gdn_kernel<128>, grid, dim3(128), 0, a)
                    : launch_kernel(lc, pf_gdn_kernel<64>, grid, dim3(128), 0, a);
    if (e != cudaSuccess) return e;
    return launch_kernel(lc, pf_ring_kernel, dim3((d.qkv_dim + 255) / 256, 4), dim3(256), 0, pb.pf_raw, ring, n, pos0,
                         d.qkv_dim);
}

}  // namespace dm
