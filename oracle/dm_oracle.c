/*
 * dm_oracle.c — CPU restatement of DISMOEN's decode step (TEST INFRASTRUCTURE; see
 * dm_oracle.h).  Only tests, the smoke check and the benchmark's CPU-baseline leg use it.
 * Built by oracle/Makefile with -O3 -fopenmp; GEMV rows are split across OpenMP threads,
 * each row reduced in a fixed order, so results do not depend on the thread count.
 */
#include "dm_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_threads = 0;
void or_set_threads(int n) {
    g_threads = n;
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#endif
}
int or_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

static inline float bf16f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static inline uint16_t f2bf16(float f) { /* round to nearest even */
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
static inline float f16f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1f, m = h & 0x3ff, u;
    if (e == 0) {
        if (m == 0) u = sign;
        else { /* subnormal: m * 2^-24 */
            float f = (float)m * (1.0f / 16777216.0f);
            memcpy(&u, &f, 4);
            u |= sign;
        }
    } else if (e == 31) u = sign | 0x7f800000u | (m << 13);
    else u = sign | ((e + 112) << 23) | (m << 13);
    float f;
    memcpy(&f, &u, 4);
    return f;
}

/* Stable logistic and SiLU (reference src/layers/swiglu.mojo:11-40). */
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
static inline float silu(float z) {
    if (isinf(z)) return z > 0 ? z : 0.0f;
    return z * sigm(z);
}
/* reference _gdn_softplus (gdn.mojo:889-894) */
static inline float softplus_ref(float v) {
    if (v > 20.0f) return v;
    if (v < -20.0f) return expf(v);
    return logf(1.0f + expf(v));
}

/* 16 interleaved partial sums, halving reduction. */
static inline float dot16_bf16(const uint16_t* w, const float* x, int n) {
    float acc[16] = {0};
    int k = 0;
    for (; k + 16 <= n; k += 16)
        for (int j = 0; j < 16; ++j) acc[j] += bf16f(w[k + j]) * x[k + j];
    for (int s = 8; s >= 1; s >>= 1)
        for (int j = 0; j < s; ++j) acc[j] += acc[j + s];
    float r = acc[0];
    for (; k < n; ++k) r += bf16f(w[k]) * x[k];
    return r;
}
static inline float dot16_f32(const float* w, const float* x, int n) {
    float acc[16] = {0};
    int k = 0;
    for (; k + 16 <= n; k += 16)
        for (int j = 0; j < 16; ++j) acc[j] += w[k + j] * x[k + j];
    for (int s = 8; s >= 1; s >>= 1)
        for (int j = 0; j < s; ++j) acc[j] += acc[j + s];
    float r = acc[0];
    for (; k < n; ++k) r += w[k] * x[k];
    return r;
}

/* y[r] = W[r, :] . x for r in [0, rows) */
static void gemv_bf16(const uint16_t* W, const float* x, int rows, int cols, float* y) {
#pragma omp parallel for schedule(static) if (rows >= 256)
    for (int r = 0; r < rows; ++r) y[r] = dot16_bf16(W + (size_t)r * cols, x, cols);
}

void or_dequant_q4(const uint8_t* q, const uint16_t* s, const uint8_t* z, int rows, int cols, int group,
                   float* out) {
    const int ng = cols / group;
#pragma omp parallel for schedule(static) if (rows >= 256)
    for (int r = 0; r < rows; ++r) {
        for (int c = 0; c < cols; ++c) {
            const uint8_t byte = q[(size_t)r * (cols / 2) + c / 2];
            const int qv = (c & 1) ? (byte >> 4) : (byte & 15);
            const int g = c / group;
            const uint8_t zb = z[(size_t)r * (ng / 2) + g / 2];
            const int zv = (g & 1) ? (zb >> 4) : (zb & 15);
            out[(size_t)r * cols + c] = f16f(s[(size_t)r * ng + g]) * (float)(qv - zv);
        }
    }
}

/* The reference's custom 4-bit format: restates dequant_kernel_simd
 * (src/quant/dequant_kernel.mojo:22-121) and dequant_kernel_simd_f32: signed nibbles in
 * [-7, 7], low nibble first, w = fp32(s_g) * q, bf16 by one round-to-nearest-even.
 * Returns 0, -2 on a NaN / Inf / non-positive scale (nothing written), or -1 on a reserved
 * nibble 0b1000 (the outputs are then incomplete). */
int or_dequant_sym4(const uint8_t* packed, const uint16_t* scales, long long n, int group, uint16_t* out_bf16,
                    float* out_f32) {
    for (long long g = 0; g < n / group; ++g) { /* NaN / Inf / non-positive scales (:66-78) */
        const uint16_t u = scales[g];
        if (((u >> 10) & 0x1F) == 0x1F || (u & 0x8000u) || (u & 0x7FFFu) == 0) return -2;
    }
    int bad = 0;
    for (long long i = 0; i < n; ++i) {
        const uint8_t byte = packed[i / 2];
        const int u = (i & 1) ? (byte >> 4) : (byte & 15);
        if (u == 8) bad = 1;
        const int q = u >= 8 ? u - 16 : u;
        const float y = f16f(scales[i / group]) * (float)q;
        if (out_bf16) out_bf16[i] = f2bf16(y);
        if (out_f32) out_f32[i] = y;
    }
    return bad ? -1 : 0;
}

/* One row of a canonical 4-bit matrix dequantised then dotted with x (fp32). */
static float q4_row_dot(const uint8_t* qrow, const uint16_t* srow, const uint8_t* zrow, int cols, int group,
                        const float* x, float* scratch) {
    for (int c = 0; c < cols; ++c) {
        const uint8_t byte = qrow[c / 2];
        const int qv = (c & 1) ? (byte >> 4) : (byte & 15);
        const int g = c / group;
        const uint8_t zb = zrow[g / 2];
        const int zv = (g & 1) ? (zb >> 4) : (zb & 15);
        scratch[c] = f16f(srow[g]) * (float)(qv - zv);
    }
    return dot16_f32(scratch, x, cols);
}

/* ---- MoE (reference moe_block / port_scheduler MoE half) ----------------------------- */
static void expert_forward(const or_dims* d, const or_layer* w, int e, const float* xn, float* out) {
    const int H = d->H, I = d->I, G = d->G;
    float* h = (float*)malloc(sizeof(float) * I);
#pragma omp parallel if (I * H >= (1 << 18))
    {
        float* scratch = (float*)malloc(sizeof(float) * (H > I ? H : I));
#pragma omp for schedule(static)
        for (int n = 0; n < I; ++n) {
            const size_t row = (size_t)e * I + n;
            const float g = q4_row_dot(w->gq + row * (H / 2), w->gs + row * (H / G), w->gz + row * (H / G / 2), H,
                                       G, xn, scratch);
            const float u = q4_row_dot(w->uq + row * (H / 2), w->us + row * (H / G), w->uz + row * (H / G / 2), H,
                                       G, xn, scratch);
            h[n] = silu(g) * u; /* swiglu_forward, swiglu.mojo:52 */
        }
#pragma omp for schedule(static)
        for (int r = 0; r < H; ++r) {
            const size_t row = (size_t)e * H + r;
            out[r] = q4_row_dot(w->dq + row * (I / 2), w->ds + row * (I / G), w->dz + row * (I / G / 2), I, G, h,
                                scratch);
        }
        free(scratch);
    }
    free(h);
}

void or_moe_block(const or_dims* d, const or_layer* w, const float* x_mid, float* x_out, int* ids_out,
                  float* probs_out) {
    const int H = d->H, K = d->topk;
    float* xn = (float*)malloc(sizeof(float) * H);
    float* eo = (float*)malloc(sizeof(float) * (size_t)(K + 1) * H);
    int ids[64];
    float probs[64], sg;
    or_rmsnorm_canonical(x_mid, w->post_norm, H, d->eps, xn);
    or_router(d, w, xn, ids, probs, &sg, NULL);
    for (int k = 0; k < K; ++k) expert_forward(d, w, ids[k], xn, eo + (size_t)k * H);
    expert_forward(d, w, d->E, xn, eo + (size_t)K * H);
    /* moe_aggregate_forward (moe.mojo:105-177): sum_k p_k E_k + g_sh E_sh + x */
    for (int r = 0; r < H; ++r) {
        float routed = 0.0f;
        for (int k = 0; k < K; ++k) routed += probs[k] * eo[(size_t)k * H + r];
        x_out[r] = routed + sg * eo[(size_t)K * H + r] + x_mid[r];
    }
    if (ids_out) memcpy(ids_out, ids, sizeof(int) * K);
    if (probs_out) memcpy(probs_out, probs, sizeof(float) * K);
    free(xn);
    free(eo);
}

/* ---- Gated DeltaNet, one token (reference forward_gdn_block, gdn.mojo:897-1183) ------- */
void or_gdn_block(const or_dims* d, const or_layer* w, float* S, float* conv, int pos, const float* x,
                  float* x_mid) {
    const int H = d->H, nk = d->nk, nv = d->nv, dk = d->dk, dv = d->dv;
    const int qkv_dim = 2 * nk * dk + nv * dv, zdim = nv * dv;
    float* xn = (float*)malloc(sizeof(float) * H);
    float* p = (float*)malloc(sizeof(float) * qkv_dim);
    float* u = (float*)malloc(sizeof(float) * qkv_dim);
    float* z = (float*)malloc(sizeof(float) * zdim);
    float* ab = (float*)malloc(sizeof(float) * 2 * nv);
    float* o = (float*)malloc(sizeof(float) * zdim);
    float* y = (float*)malloc(sizeof(float) * H);
    float* kn = (float*)malloc(sizeof(float) * dk);
    (void)pos;
    or_rmsnorm_canonical(x, w->in_norm, H, d->eps, xn);          /* step 1 */
    gemv_bf16(w->qkv, xn, qkv_dim, H, p);                         /* step 2 */
    /* step 3: causal depthwise conv k=4 + SiLU; conv holds the 3 previous projections */
    for (int c = 0; c < qkv_dim; ++c) {
        float acc = 0.0f;
        for (int j = 0; j < 4; ++j) {
            const float in = (j < 3) ? conv[(size_t)j * qkv_dim + c] : p[c];
            acc += bf16f(w->conv[(size_t)c * 4 + j]) * in;
        }
        u[c] = silu(acc);
    }
    memmove(conv, conv + qkv_dim, sizeof(float) * 2 * qkv_dim);
    memcpy(conv + 2 * (size_t)qkv_dim, p, sizeof(float) * qkv_dim);
    gemv_bf16(w->z, xn, zdim, H, z);                              /* step 4 */
    for (int i = 0; i < zdim; ++i) z[i] = silu(z[i]);
    gemv_bf16(w->a, xn, nv, H, ab);
    gemv_bf16(w->b, xn, nv, H, ab + nv);
    /* step 5: delta rule per V head */
    for (int h = 0; h < nv; ++h) {
        const int src = h / (nv / nk);
        const float* q = u + (size_t)src * dk;
        const float* k = u + (size_t)nk * dk + (size_t)src * dk;
        const float* v = u + (size_t)2 * nk * dk + (size_t)h * dv;
        const float g = expf(-expf(w->a_log[h]) * softplus_ref(ab[h] + w->dt_bias[h]));
        const float beta = sigm(ab[nv + h]);
        float ss = 0.0f;
        for (int c = 0; c < dk; ++c) ss += k[c] * k[c];
        const float inv = 1.0f / (sqrtf(ss) + d->eps);
        for (int c = 0; c < dk; ++c) kn[c] = k[c] * inv;
        float* Sh = S + (size_t)h * dv * dk;
        for (int r = 0; r < dv; ++r) {
            float* Sr = Sh + (size_t)r * dk;
            const float sk = dot16_f32(Sr, kn, dk);
            for (int c = 0; c < dk; ++c) Sr[c] = g * (Sr[c] - beta * sk * kn[c]) + beta * v[r] * kn[c];
            o[(size_t)h * dv + r] = dot16_f32(Sr, q, dk);
        }
    }
    /* step 6: head RMSNorm * norm_weight * z */
    for (int h = 0; h < nv; ++h) {
        float* oh = o + (size_t)h * dv;
        float ss = 0.0f;
        for (int c = 0; c < dv; ++c) ss += oh[c] * oh[c];
        const float rs = 1.0f / sqrtf(ss / (float)dv + d->eps);
        for (int c = 0; c < dv; ++c) oh[c] = oh[c] * rs * bf16f(w->gnorm[c]) * z[(size_t)h * dv + c];
    }
    gemv_bf16(w->out, o, H, zdim, y);                             /* step 7 */
    for (int i = 0; i < H; ++i) x_mid[i] = x[i] + y[i];           /* step 8 */
    free(xn); free(p); free(u); free(z); free(ab); free(o); free(y); free(kn);
}

/* ---- gated attention, one token (reference forward_attention_qwen36 + KV cache) ------ */
static void head_rmsnorm(float* v, const uint16_t* w, int D, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < D; ++i) ss += v[i] * v[i];
    const float rs = 1.0f / sqrtf(ss / (float)D + eps);
    for (int i = 0; i < D; ++i) v[i] = v[i] * rs * bf16f(w[i]);
}
static void rope_partial(float* v, int rot, float theta, int pos) {
    const int half = rot / 2;
    const float m = (float)pos;
    for (int i = 0; i < half; ++i) {
        const float inv_freq = 1.0f / powf(theta, (float)(2 * i) / (float)rot);
        const float cs = cosf(m * inv_freq), sn = sinf(m * inv_freq);
        const float x0 = v[i], x1 = v[i + half];
        v[i] = x0 * cs - x1 * sn;
        v[i + half] = x0 * sn + x1 * cs;
    }
}

void or_attn_block(const or_dims* d, const or_layer* w, void* kcache, void* vcache, int pos, const float* x,
                   float* x_mid) {
    const int H = d->H, Hq = d->Hq, Hkv = d->Hkv, D = d->D;
    const int qd = Hq * D, kd = Hkv * D, grp = Hq / Hkv;
    float* xn = (float*)malloc(sizeof(float) * H);
    float* qg = (float*)malloc(sizeof(float) * 2 * qd);
    float* kv = (float*)malloc(sizeof(float) * 2 * kd);
    float* att = (float*)malloc(sizeof(float) * qd);
    float* y = (float*)malloc(sizeof(float) * H);
    float* sc = (float*)malloc(sizeof(float) * (size_t)(pos + 1));
    or_rmsnorm_canonical(x, w->in_norm, H, d->eps, xn);
    gemv_bf16(w->q, xn, 2 * qd, H, qg);
    gemv_bf16(w->k, xn, kd, H, kv);
    gemv_bf16(w->v, xn, kd, H, kv + kd);
    for (int h = 0; h < Hq; ++h) {
        head_rmsnorm(qg + (size_t)h * D, w->qn, D, d->eps);
        rope_partial(qg + (size_t)h * D, d->rot_dim, d->theta, pos);
    }
    for (int h = 0; h < Hkv; ++h) {
        head_rmsnorm(kv + (size_t)h * D, w->kn, D, d->eps);
        rope_partial(kv + (size_t)h * D, d->rot_dim, d->theta, pos);
    }
    /* append at pos (LayerKVCache.append_decode_token, kv_cache.mojo:302-375) */
    for (int i = 0; i < kd; ++i) {
        if (d->kv_bf16) {
            ((uint16_t*)kcache)[(size_t)pos * kd + i] = f2bf16(kv[i]);
            ((uint16_t*)vcache)[(size_t)pos * kd + i] = f2bf16(kv[kd + i]);
        } else {
            ((float*)kcache)[(size_t)pos * kd + i] = kv[i];
            ((float*)vcache)[(size_t)pos * kd + i] = kv[kd + i];
        }
    }
    const float scale = 1.0f / sqrtf((float)D);
    for (int h = 0; h < Hq; ++h) {
        const int g = h / grp;
        const float* q = qg + (size_t)h * D;
        float mx = -1e30f;
        for (int t = 0; t <= pos; ++t) {
            float dot = 0.0f;
            for (int i = 0; i < D; ++i) {
                const size_t idx = (size_t)t * kd + (size_t)g * D + i;
                const float kval = d->kv_bf16 ? bf16f(((const uint16_t*)kcache)[idx]) : ((const float*)kcache)[idx];
                dot += q[i] * kval;
            }
            sc[t] = dot * scale;
            if (sc[t] > mx) mx = sc[t];
        }
        float sum = 0.0f;
        for (int t = 0; t <= pos; ++t) {
            sc[t] = expf(sc[t] - mx);
            sum += sc[t];
        }
        const float inv = 1.0f / sum;
        for (int t = 0; t <= pos; ++t) sc[t] *= inv;
        for (int i = 0; i < D; ++i) {
            float acc = 0.0f;
            for (int t = 0; t <= pos; ++t) {
                const size_t idx = (size_t)t * kd + (size_t)g * D + i;
                const float vval = d->kv_bf16 ? bf16f(((const uint16_t*)vcache)[idx]) : ((const float*)vcache)[idx];
                acc += sc[t] * vval;
            }
            att[(size_t)h * D + i] = acc * sigm(qg[(size_t)qd + (size_t)h * D + i]);
        }
    }
    gemv_bf16(w->o, att, H, qd, y);
    for (int i = 0; i < H; ++i) x_mid[i] = x[i] + y[i];
    free(xn); free(qg); free(kv); free(att); free(y); free(sc);
}

/* ---- block / step -------------------------------------------------------------------- */
static int is_attn(const or_dims* d, int l) { return l % d->interval == d->interval - 1; }

void or_block_forward(const or_model* m, or_state* st, int layer, const float* x, float* x_out, int* ids_out) {
    const or_dims* d = &m->d;
    const int H = d->H;
    int gi = 0, ai = 0;
    for (int l = 0; l < layer; ++l) {
        if (is_attn(d, l)) ++ai;
        else ++gi;
    }
    const int qkv_dim = 2 * d->nk * d->dk + d->nv * d->dv;
    const size_t esz = d->kv_bf16 ? 2 : 4;
    float* xm = (float*)malloc(sizeof(float) * H);
    if (is_attn(d, layer)) {
        const size_t off = (size_t)ai * st->cap * d->Hkv * d->D * esz;
        or_attn_block(d, &m->layers[layer], (char*)st->kcache + off, (char*)st->vcache + off, st->len, x, xm);
    } else {
        or_gdn_block(d, &m->layers[layer], st->S + (size_t)gi * d->nv * d->dv * d->dk,
                     st->conv + (size_t)gi * 3 * qkv_dim, st->len, x, xm);
    }
    or_moe_block(d, &m->layers[layer], xm, x_out, ids_out, NULL);
    free(xm);
}

int or_head(const or_model* m, const float* x, float* logits) {
    const or_dims* d = &m->d;
    float* xn = (float*)malloc(sizeof(float) * d->H);
    or_rmsnorm_canonical(x, m->final_norm, d->H, d->eps, xn);
    gemv_bf16(m->lm_head, xn, d->V, d->H, logits);
    int best = 0;
    float bv = logits[0];
    for (int i = 1; i < d->V; ++i)
        if (logits[i] > bv) { bv = logits[i]; best = i; }
    free(xn);
    return best;
}

int or_decode_step(const or_model* m, or_state* st, int token, float* logits, float* hidden) {
    const or_dims* d = &m->d;
    const int H = d->H, V = d->V;
    float* x = (float*)malloc(sizeof(float) * H);
    float* x2 = (float*)malloc(sizeof(float) * H);
    float* lg = logits ? logits : (float*)malloc(sizeof(float) * V);
    if (token < 0 || token >= V) token = 0;
    for (int i = 0; i < H; ++i) x[i] = bf16f(m->embed[(size_t)token * H + i]);
    for (int l = 0; l < d->L; ++l) {
        or_block_forward(m, st, l, x, x2, NULL);
        memcpy(x, x2, sizeof(float) * H);
        if (hidden) memcpy(hidden + (size_t)l * H, x, sizeof(float) * H);
    }
    or_rmsnorm_canonical(x, m->final_norm, H, d->eps, x2);
    gemv_bf16(m->lm_head, x2, V, H, lg);
    int best = 0;
    float bv = lg[0];
    for (int i = 1; i < V; ++i)
        if (lg[i] > bv) { bv = lg[i]; best = i; }
    st->len += 1;
    if (!logits) free(lg);
    free(x);
    free(x2);
    return best;
}
