// dm_router.cuh — the router's canonical arithmetic, shared by the single-token router
// kernel and the batched router kernel so that both give the same bits as the CPU
// restatement for the same input (reference router.mojo:15-185, topk.mojo:11-131).
//
//   RMSNorm: NT threads, thread t: fma-accumulate x[k]^2 for k = t, t+NT, ...; warp
//            butterfly (xor 16..1); the NT/32 warp sums added in warp order; denom =
//            sqrt(ss / K + eps); y = (x / denom) * gamma.
//   dot:     lane l: fma over elements 8(l + 32i) + j, i then j ascending; butterfly.
//   softmax: m = max; e = det_exp(z - m); lane l sums e[l], e[l+32], ... in order;
//            butterfly; p = e * (1 / sum).  Top-k: max p, ties to the lower id.
#pragma once
#include "dismoen_detmath.h"
#include "dm_common.cuh"

namespace dm {

// xs split layout: float4 lo[K/8] holds x[8j..8j+3], hi[K/8] holds x[8j+4..8j+7].
DM_DEV void xs_store_split(float* xs, int K, int k, float v) {
    int j = k >> 3, e = k & 7;
    xs[(e < 4 ? 0 : K / 2) + j * 4 + (e & 3)] = v;
}

// Canonical RMSNorm of x[0..K) by all NT threads of the CTA into the split layout xs
// (and xn_out when non-null).  `red` holds NT/32 floats; the caller synchronises before
// red is reused.
template <int K, int NT>
DM_DEV void canon_rmsnorm_split(const float* x, const uint16_t* gamma, float eps, float* xs, float* xn_out,
                                float* red) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float xv[(K + NT - 1) / NT];
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i * NT + tid < K; ++i) {
        xv[i] = x[i * NT + tid];
        acc = __fmaf_rn(xv[i], xv[i], acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    float ss = 0.0f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) ss = __fadd_rn(ss, red[w]);
    const float denom = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps));
#pragma unroll
    for (int i = 0; i * NT + tid < K; ++i) {
        const int k = i * NT + tid;
        const float y = __fmul_rn(__fdiv_rn(xv[i], denom), bf16_to_f32(gamma[k]));
        xs_store_split(xs, K, k, y);
        if (xn_out) xn_out[k] = y;
    }
}

// The same RMSNorm with this thread's elements (k = t, t + NT, ...) already loaded into xv,
// so that the loads of several rows can be in flight together.
template <int K, int NT>
DM_DEV void canon_rmsnorm_split_loaded(const float (&xv)[(K + NT - 1) / NT], const uint16_t* gamma, float eps,
                                       float* xs, float* xn_out, float* red) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i * NT + tid < K; ++i) acc = __fmaf_rn(xv[i], xv[i], acc);
    acc = warp_sum(acc);
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    float ss = 0.0f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) ss = __fadd_rn(ss, red[w]);
    const float denom = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps));
#pragma unroll
    for (int i = 0; i * NT + tid < K; ++i) {
        const int k = i * NT + tid;
        const float y = __fmul_rn(__fdiv_rn(xv[i], denom), bf16_to_f32(gamma[k]));
        xs_store_split(xs, K, k, y);
        if (xn_out) xn_out[k] = y;
    }
}

// The same RMSNorm for RB rows at once (rows r < nr valid): every row's sum of squares is
// formed exactly as above (thread fma order, warp butterfly, warp partials in warp order),
// so each row gets the bits of canon_rmsnorm_split_loaded, with one block barrier for all
// RB rows instead of one per row.  red holds RB * NT/32 floats; xs / xn_out row r at
// xs + r * K (xn_out may be null).  The caller synchronises before xs is read.
template <int K, int NT, int RB>
DM_DEV void canon_rmsnorm_split_loaded_rows(const float (&xv)[RB][(K + NT - 1) / NT], int nr, const uint16_t* gamma,
                                            float eps, float* xs, float* xn_out, float* red) {
    constexpr int XPT = (K + NT - 1) / NT;
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float acc[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) {
        acc[r] = 0.0f;
#pragma unroll
        for (int i = 0; i * NT + tid < K && i < XPT; ++i) acc[r] = __fmaf_rn(xv[r][i], xv[r][i], acc[r]);
    }
#pragma unroll
    for (int r = 0; r < RB; ++r) acc[r] = warp_sum(acc[r]);
    if (lane == 0)
#pragma unroll
        for (int r = 0; r < RB; ++r) red[r * NW + warp] = acc[r];
    __syncthreads();
#pragma unroll
    for (int r = 0; r < RB; ++r) {
        if (r >= nr) break;
        float ss = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; ++w) ss = __fadd_rn(ss, red[r * NW + w]);
        const float denom = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), eps));
#pragma unroll
        for (int i = 0; i * NT + tid < K && i < XPT; ++i) {
            const int k = i * NT + tid;
            const float y = __fmul_rn(__fdiv_rn(xv[r][i], denom), bf16_to_f32(gamma[k]));
            xs_store_split(xs + static_cast<size_t>(r) * K, K, k, y);
            if (xn_out) xn_out[static_cast<size_t>(r) * K + k] = y;
        }
    }
}

// Canonical dot of one bf16 router row (VPL 16-byte vectors per lane, vector i of lane l
// holding elements 8(l + 32i) .. +7) with x in the split layout; every lane gets the sum.
template <int VPL>
DM_DEV float canon_router_dot(const uint4 (&wreg)[VPL], const float4* xlo, const float4* xhi, int lane) {
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int j = lane + 32 * i;
        const uint4 w = wreg[i];
        const float4 x0 = xlo[j], x1 = xhi[j];
        acc = __fmaf_rn(bf16lo(w.x), x0.x, acc);
        acc = __fmaf_rn(bf16hi(w.x), x0.y, acc);
        acc = __fmaf_rn(bf16lo(w.y), x0.z, acc);
        acc = __fmaf_rn(bf16hi(w.y), x0.w, acc);
        acc = __fmaf_rn(bf16lo(w.z), x1.x, acc);
        acc = __fmaf_rn(bf16hi(w.z), x1.y, acc);
        acc = __fmaf_rn(bf16lo(w.w), x1.z, acc);
        acc = __fmaf_rn(bf16hi(w.w), x1.w, acc);
    }
    return warp_sum(acc);
}

// Softmax over lg[0..E) and top-k selection by one warp (lg in shared memory, lg[E] the
// shared-expert gate logit).  The probabilities overwrite lg[0..E).  Lane 0 writes
// ids[0..topk), probs[0..topk) and *shared_g (when non-null).
DM_DEV void canon_softmax_topk_warp(float* lg, int E, int topk, int* ids, float* probs, float* shared_g,
                                    uint32_t* err) {
    const int lane = threadIdx.x & 31;
    float m = -INFINITY;
    for (int e = lane; e < E; e += 32) m = fmaxf(m, lg[e]);
    m = warp_max(m);
    float s = 0.0f;
    float* pe = lg;
    for (int e = lane; e < E; e += 32) {
        const float ev = dm_det_exp(DM_DET_SUB(lg[e], m));
        pe[e] = ev;
        s = DM_DET_ADD(s, ev);
    }
    s = warp_sum(s);
    const float inv = DM_DET_DIV(1.0f, s);
    for (int e = lane; e < E; e += 32) pe[e] = DM_DET_MUL(pe[e], inv);
    __syncwarp();
    for (int r = 0; r < topk; ++r) {
        float bv = -1.0f;
        int bi = 0x7fffffff;
        for (int e = lane; e < E; e += 32)
            if (pe[e] > bv) { bv = pe[e]; bi = e; }
#pragma unroll
        for (int mm = 16; mm >= 1; mm >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, mm);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, mm);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (bi < 0 || bi >= E) {  // only when probabilities are NaN: keep ids in range
            if (lane == 0) raise_error(err, DM_DEVERR_NONFINITE);
            bi = r;
            bv = 0.0f;
        }
        if (lane == 0) {
            ids[r] = bi;
            probs[r] = bv;
            pe[bi] = -2.0f;
        }
        __syncwarp();
    }
    if (lane == 0) {
        if (shared_g) *shared_g = sigmoid_f(lg[E]);
        if (s != s || isinf(s)) raise_error(err, DM_DEVERR_NONFINITE);
    }
    __syncwarp();
}

}  // namespace dm
