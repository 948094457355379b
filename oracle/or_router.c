/*
 * or_router.c — router and canonical RMSNorm of the CPU oracle (TEST INFRASTRUCTURE).
 * Compiled with -ffp-contract=off: every rounding step below is one IEEE operation, in
 * the order the CUDA router kernel uses, so the selected expert ids and probabilities
 * can be compared with the device bit for bit.
 *
 * Semantics: reference src/layers/router.mojo:15-185 (logits = W x; softmax with max
 * shift, exp, multiply by 1/sum) and src/layers/topk.mojo:11-131 (top-k on probabilities,
 * ties to the lower expert id, no renormalisation); shared gate sigmoid per
 * src/layers/moe.mojo:17.
 */
#include <math.h>
#include <string.h>

#include "../include/dismoen_detmath.h"
#include "dm_oracle.h"

static inline float bf16f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

float or_det_exp(float x) { return dm_det_exp(x); }

/* butterfly over 32 lanes: xor 16, 8, 4, 2, 1; every lane ends with lane-order-free sums */
static float butterfly32(float* v) {
    float t[32];
    for (int m = 16; m >= 1; m >>= 1) {
        for (int l = 0; l < 32; ++l) t[l] = v[l] + v[l ^ m];
        memcpy(v, t, sizeof t);
    }
    return v[0];
}

void or_rmsnorm_canonical(const float* x, const uint16_t* gamma, int n, float eps, float* y) {
    float lanes[16][32];
    for (int t = 0; t < 512; ++t) {
        float acc = 0.0f;
        for (int k = t; k < n; k += 512) acc = fmaf(x[k], x[k], acc);
        lanes[t >> 5][t & 31] = acc;
    }
    float ss = 0.0f;
    for (int w = 0; w < 16; ++w) ss = ss + butterfly32(lanes[w]);
    const float denom = sqrtf(ss / (float)n + eps);
    for (int k = 0; k < n; ++k) y[k] = (x[k] / denom) * bf16f(gamma[k]);
}

/* Router dot product in the device order: lane l accumulates elements 8(l + 32i) + j,
 * i ascending then j ascending, one fma each; then the 32-lane butterfly. */
static float router_dot(const uint16_t* w, const float* x, int K) {
    float lanes[32];
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int i = 0; i < K / 256; ++i)
            for (int j = 0; j < 8; ++j) {
                const int k = 8 * (l + 32 * i) + j;
                acc = fmaf(bf16f(w[k]), x[k], acc);
            }
        lanes[l] = acc;
    }
    return butterfly32(lanes);
}

static inline float sigm(float z) {
    if (z != z) return z;
    if (z < -88.0f) return 0.0f;
    if (z > 88.0f) return 1.0f;
    if (z < 0.0f) {
        float e = expf(z);
        return e / (1.0f + e);
    }
    return 1.0f / (1.0f + expf(-z));
}

void or_router(const or_dims* d, const or_layer* w, const float* xn, int* ids, float* probs, float* shared_g,
               float* logits_out) {
    const int E = d->E, K = d->H;
    float z[1024], p[1024];
    for (int e = 0; e < E; ++e) z[e] = router_dot(w->router + (size_t)e * K, xn, K);
    const float zs = router_dot(w->shared_gate, xn, K);
    if (logits_out) {
        memcpy(logits_out, z, sizeof(float) * E);
        logits_out[E] = zs;
    }
    float m = -INFINITY;
    for (int e = 0; e < E; ++e) m = fmaxf(m, z[e]);
    /* sum: lane l adds e = l, l+32, ... in order, then the butterfly */
    float lanes[32];
    for (int l = 0; l < 32; ++l) {
        float s = 0.0f;
        for (int e = l; e < E; e += 32) {
            p[e] = dm_det_exp(z[e] - m);
            s = s + p[e];
        }
        lanes[l] = s;
    }
    const float s = butterfly32(lanes);
    const float inv = 1.0f / s;
    for (int e = 0; e < E; ++e) p[e] = p[e] * inv;
    /* selection: highest probability, ties to the lower id (topk.mojo:80-96) */
    for (int r = 0; r < d->topk; ++r) {
        int bi = -1;
        float bv = -1.0f;
        for (int e = 0; e < E; ++e)
            if (p[e] > bv) {
                bv = p[e];
                bi = e;
            }
        ids[r] = bi;
        probs[r] = bv;
        p[bi] = -2.0f;
    }
    if (shared_g) *shared_g = sigm(zs);
}
