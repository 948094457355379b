/*
 * dm_oracle.h — CPU restatement of DISMOEN's decode step (TEST INFRASTRUCTURE).
 *
 * This library is the checker for libdismoen_cuda.so: only the tests, the smoke check and
 * the benchmark's CPU-baseline leg load it.  It is never part of the product path.
 *
 * It restates, in plain fp32 C, the full-shape Qwen3.6 semantics of the reference engine:
 *   RMSNorm                 reference src/layers/rmsnorm.mojo:10-48
 *   Gated DeltaNet block    reference src/layers/gdn.mojo:897-1183 (decode form: the conv
 *                           window and recurrent state are carried between tokens)
 *   gated attention block   reference src/layers/attention.mojo:219-435 with the KV cache
 *                           of reference src/layers/kv_cache.mojo:302-375 (bf16 store)
 *   router + top-k          reference src/layers/router.mojo:109-185, topk.mojo:11-131
 *   SwiGLU experts + shared gate + aggregation
 *                           reference src/layers/swiglu.mojo:11-230, moe.mojo:17-177
 *   embedding / head        reference src/layers/gguf_port_loader.mojo:274-326,
 *                           argmax reference src/cli/cmd_decode.mojo:115-131
 *   4-bit expert weights    w = fp32(scale) * (q - zero), low nibble first
 *                           (nibble order of reference docs/format/quant_format.md:831-854)
 *
 * Arithmetic: fp32 everywhere; dense dot products use 16 interleaved partial sums
 * reduced by halving (the SIMD-16 accumulation of the reference's Mojo GEMVs, e.g.
 * gdn.mojo:938-951).  The router (RMSNorm of its input, its dot products, softmax and
 * top-k) instead follows the fixed order documented in include/dismoen_detmath.h and the
 * CUDA router kernel, so that expert ids can be compared bit for bit.
 */
#ifndef DM_ORACLE_H
#define DM_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct or_dims {
    int H, L, interval, V;
    float eps;
    int Hq, Hkv, D, rot_dim;
    float theta;
    int nk, nv, dk, dv;
    int E, topk, I, G;
    int kv_bf16; /* 1: KV stored as bf16 (product semantics); 0: fp32 (prefill oracle) */
} or_dims;

/* One layer's weights in canonical host layouts (bf16 as uint16 bit patterns). */
typedef struct or_layer {
    const uint16_t *in_norm, *post_norm;
    /* GDN */
    const uint16_t *qkv, *z, *a, *b, *conv, *gnorm, *out;
    const float *dt_bias, *a_log;
    /* attention */
    const uint16_t *q, *k, *v, *qn, *kn, *o;
    /* MoE: router [E][H], shared gate [H]; experts index 0..E-1 routed, E = shared:
     * gate/up q [E+1][I][H/2], s [E+1][I][H/G], z [E+1][I][H/G/2];
     * down q [E+1][H][I/2], s [E+1][H][I/G], z [E+1][H][I/G/2] */
    const uint16_t *router, *shared_gate;
    const uint8_t *gq, *gz, *uq, *uz, *dq, *dz;
    const uint16_t *gs, *us, *ds;
} or_layer;

typedef struct or_model {
    or_dims d;
    const or_layer* layers; /* [L] */
    const uint16_t *embed, *final_norm, *lm_head;
} or_model;

/* Per-sequence state for the decode form. */
typedef struct or_state {
    float* S;        /* [n_gdn][nv][dv][dk] */
    float* conv;     /* [n_gdn][3][qkv_dim] pre-conv projections of the last 3 tokens, oldest first */
    void* kcache;    /* [n_att][cap][Hkv][D] bf16 (uint16) or fp32 per kv_bf16 */
    void* vcache;
    int cap;
    int len;         /* tokens processed (position of the next token) */
} or_state;

void or_set_threads(int n);
int or_get_threads(void);

/* Canonical RMSNorm (device order): y = (x / sqrt(ss/n + eps)) * gamma. */
void or_rmsnorm_canonical(const float* x, const uint16_t* gamma, int n, float eps, float* y);

/* Router on an already-normalised input: ids/probs [topk], shared gate sigmoid. */
void or_router(const or_dims* d, const or_layer* w, const float* xn, int* ids, float* probs,
               float* shared_g, float* logits_out /* [E+1] or NULL */);

/* fp32 dequantisation of one canonical 4-bit tensor. */
void or_dequant_q4(const uint8_t* q, const uint16_t* s, const uint8_t* z, int rows, int cols,
                   int group, float* out);

/* The reference's custom 4-bit format (dequant_kernel_simd): 0, -2 on a bad scale, or -1 on
 * a reserved nibble. */
int or_dequant_sym4(const uint8_t* packed, const uint16_t* scales, long long n, int group, uint16_t* out_bf16,
                    float* out_f32);

/* On-disk weight formats (or_formats.c): GGUF block dequantisation (type = GGML type id;
 * flags bit 0 = the Q4_K reading of gguf.mojo; returns -1 for an unsupported type, -2 when
 * n is not a multiple of the block), the exact custom-4-bit -> pool conversion and the
 * round-to-nearest re-quantisation into the pool; fp16 conversions. */
float or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_f16(float f);
int or_gguf_dequant(int type, const uint8_t* raw, long long n, unsigned flags, float* out);
unsigned or_sym4_to_pool(const uint8_t* packed, const uint16_t* scales, long long e0, int rows, int cols, int gf,
                         int gp, uint8_t* q, uint16_t* s, uint8_t* z);
unsigned or_requant_pool(const float* w, int rows, int cols, int gp, uint8_t* q, uint16_t* s, uint8_t* z,
                         float* max_err);

/* MoE sublayer with residual: x_out = x_mid + moe(norm(x_mid)); ids optional [topk]. */
void or_moe_block(const or_dims* d, const or_layer* w, const float* x_mid, float* x_out, int* ids_out,
                  float* probs_out);

/* Token mixers with residual for one token at position pos. */
void or_gdn_block(const or_dims* d, const or_layer* w, float* S, float* conv, int pos, const float* x,
                  float* x_mid);
void or_attn_block(const or_dims* d, const or_layer* w, void* kcache, void* vcache, int pos,
                   const float* x, float* x_mid);

/* Full block (mixer + MoE) for layer l of the model, updating the state at st->len
 * (the caller advances st->len after the last layer). */
void or_block_forward(const or_model* m, or_state* st, int layer, const float* x, float* x_out,
                      int* ids_out);

/* One decode step: embed token, all layers, final norm, lm_head; returns argmax (first
 * maximum).  hidden [L][H] (optional) receives every layer's output; logits [V] optional. */
int or_decode_step(const or_model* m, or_state* st, int token, float* logits, float* hidden);

/* Final RMSNorm + lm_head + argmax (first maximum) of one hidden state. */
int or_head(const or_model* m, const float* x, float* logits);

/* The seeded synthetic-checkpoint generator (or_synth.c), bit-identical to the library's
 * host generator; same signatures and distributions as dm_synth_* in dismoen_cuda.h. */
int or_synth_bf16(uint64_t seed, uint64_t sid, uint64_t n, float mean, float std, uint16_t* out);
int or_synth_f32(uint64_t seed, uint64_t sid, uint64_t n, float mean, float std, float* out);
int or_synth_u8(uint64_t seed, uint64_t sid, uint64_t n, uint8_t* out);
int or_synth_f16_absnormal(uint64_t seed, uint64_t sid, uint64_t n, float std, uint16_t* out);

/* Deterministic exponential shared with the device router (include/dismoen_detmath.h). */
float or_det_exp(float x);

#ifdef __cplusplus
}
#endif
#endif
