/*
 * dismoen_cuda.h — C ABI of libdismoen_cuda.so, the B200 (sm_100a) implementation of
 * DISMOEN's per-token decode step for a Qwen3.6-35B-A3B-shaped hybrid MoE
 * (blocks [GDN, GDN, GDN, GatedAttn] x N, MoE top-k + 1 shared expert per block).
 *
 * The reference engine is Mojo and reaches native code through `external_call`
 * (reference src/core/worker_pool.mojo:202-457, src/cli/cmd_decode.mojo:78).  Every
 * symbol below is a plain `extern "C"` function taking plain pointers and sizes so that
 * the same binding works from Mojo `external_call`, Python `ctypes` or C.
 *
 * Conventions
 *  - Every function returns int32 status: DM_OK (0) or one of DM_ERR_*.  The message of
 *    the last failure is a JSON object in the reference error shape
 *    {"error_type":..., "detail":..., "stage":..., "layer":...}
 *    (reference src/layers/router.mojo:28-33), read with dm_last_error().
 *  - Pointers named *_host are host memory owned by the caller; the library never keeps
 *    or frees them.  All device memory is owned by the context.
 *  - One host thread per context; all work runs on the context's CUDA stream.  Calls
 *    with host outputs synchronise that stream before returning.
 *  - Activations are fp32, dense weights bf16 (raw uint16 bit patterns), routed and
 *    shared experts in the asymmetric 4-bit group format described at
 *    dm_expert_upload().
 */
#ifndef DISMOEN_CUDA_H
#define DISMOEN_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DM_ABI_VERSION 2

/* ---- status codes ------------------------------------------------------------------ */
#define DM_OK 0
#define DM_ERR_INVALID_ARG 1   /* bad pointer, size, index or config                  */
#define DM_ERR_CUDA 2          /* a CUDA runtime call failed                           */
#define DM_ERR_OOM 3           /* device allocation failed                             */
#define DM_ERR_POSITION 4      /* KV append position contract violated                 */
#define DM_ERR_CAPACITY 5      /* KV capacity / page table exhausted                   */
#define DM_ERR_NONFINITE 6     /* NaN/Inf reached a checked output (logits)            */
#define DM_ERR_TIMEOUT 7       /* a bounded device-side wait ran out                   */
#define DM_ERR_NOT_READY 8     /* weights missing for the requested computation        */
#define DM_ERR_ROUTER 9        /* router contract violated (e.g. norm_topk_prob)       */
#define DM_ERR_IO 10           /* a session or weight file could not be read / written */
#define DM_ERR_FORMAT 11       /* a session or weight file failed its format checks    */

/* ---- configuration ----------------------------------------------------------------- */
/* Field names and meaning follow the reference ModelConfig
 * (reference src/core/config.mojo:11-175) plus the GDN shape fields that the reference
 * hard-codes in forward_gdn_block (reference src/layers/gdn.mojo:897-1183). */
typedef struct dm_model_config {
    int32_t hidden_size;                     /* H                                    */
    int32_t num_hidden_layers;               /* L                                    */
    int32_t full_attention_interval;         /* layer l is attention iff l%I == I-1  */
    int32_t vocab_size;                      /* V                                    */
    float rms_norm_eps;                      /* > 0                                  */
    /* gated attention */
    int32_t num_attention_heads;             /* Hq                                   */
    int32_t num_key_value_heads;             /* Hkv, Hq % Hkv == 0                   */
    int32_t head_dim;                        /* D (multiple of 64)                   */
    float rope_theta;
    float partial_rotary_factor;             /* rotary_dim = int(D * factor)         */
    /* gated DeltaNet */
    int32_t linear_num_key_heads;            /* QK heads                             */
    int32_t linear_num_value_heads;          /* V heads (multiple of QK heads)       */
    int32_t linear_key_head_dim;             /* dk (64 or 128)                       */
    int32_t linear_value_head_dim;           /* dv (== dk)                           */
    int32_t linear_conv_kernel_dim;          /* 4                                    */
    /* MoE */
    int32_t num_experts;                     /* E                                    */
    int32_t num_experts_per_tok;             /* top-k                                */
    int32_t moe_intermediate_size;           /* I                                    */
    int32_t shared_expert_intermediate_size; /* must equal I                         */
    int32_t norm_topk_prob;                  /* must be 0 (no renormalisation)       */
    int32_t quant_group_size;                /* 64                                   */
} dm_model_config;

typedef struct dm_runtime_config {
    int32_t max_seqs;          /* number of sequence slots (KV + GDN state owners)     */
    int32_t kv_page_tokens;    /* tokens per KV page; must be 16                       */
    int32_t kv_num_pages;      /* pages in the shared pool (per attention layer)       */
    int32_t max_pages_per_seq; /* page-table width; capacity = this * 16 tokens        */
    int32_t expert_cache_slots; /* 0: every expert resident in HBM.  C in
                                 * [num_experts_per_tok, num_experts): C routed expert
                                 * records per layer in HBM, all of them in pinned host
                                 * memory, loaded on demand (see dm_spill_stats)         */
} dm_runtime_config;

typedef struct dm_ctx dm_ctx;

/* ---- lifecycle ----------------------------------------------------------------------- */
/* Validates the config (the checks of reference ModelConfig.__init__, config.mojo:31-147,
 * plus kernel shape limits), selects `device`, allocates every weight, state and scratch
 * buffer up front (no allocation happens during compute). */
int32_t dm_ctx_create(const dm_model_config* model, const dm_runtime_config* rt,
                      int32_t device, dm_ctx** out_ctx);
int32_t dm_ctx_destroy(dm_ctx* ctx);
/* Copies the JSON message of the last failure (empty string if none) into buf. */
int32_t dm_last_error(const dm_ctx* ctx, char* buf, uint64_t buf_size);
/* Validation only, no GPU use: writes the JSON error into buf on failure. */
int32_t dm_config_validate(const dm_model_config* model, char* buf, uint64_t buf_size);
int32_t dm_abi_version(void);
/* Bytes of device memory held by the context. */
int32_t dm_ctx_device_bytes(const dm_ctx* ctx, uint64_t* out_bytes);

/* ---- weights: the quant-loader / tensor-name contract ---------------------------------
 * Replaces the per-layer streaming loader load_port_block_from_gguf
 * (reference src/layers/gguf_port_loader.mojo:115) and stream_gguf_tensor_f32
 * (reference src/format/gguf.mojo:563): tensors are uploaded once into an HBM-resident
 * pool instead of being read and dequantised per layer per step.  Tensor ids mirror the
 * checkpoint names the reference loads (gdn.mojo:785-795, attention.mojo:504,
 * router.mojo:213, gguf_port_loader.mojo:274-326). */
enum dm_tensor_id {
    DM_T_INPUT_NORM = 0,     /* input_layernorm.weight            [H]                  */
    DM_T_POST_NORM = 1,      /* post_attention_layernorm.weight   [H]                  */
    DM_T_GDN_QKV = 2,        /* linear_attn.in_proj_qkv.weight    [2*nk*dk + nv*dv, H] */
    DM_T_GDN_CONV = 3,       /* linear_attn.conv1d.weight         [2*nk*dk + nv*dv, 4] */
    DM_T_GDN_Z = 4,          /* linear_attn.in_proj_z.weight      [nv*dv, H]           */
    DM_T_GDN_A = 5,          /* linear_attn.in_proj_a.weight      [nv, H]              */
    DM_T_GDN_B = 6,          /* linear_attn.in_proj_b.weight      [nv, H]              */
    DM_T_GDN_DT_BIAS = 7,    /* linear_attn.dt_bias               [nv]      (f32)      */
    DM_T_GDN_A_LOG = 8,      /* linear_attn.A_log                 [nv]      (f32)      */
    DM_T_GDN_NORM = 9,       /* linear_attn.norm.weight           [dv]                 */
    DM_T_GDN_OUT = 10,       /* linear_attn.out_proj.weight       [H, nv*dv]           */
    DM_T_ATTN_Q = 11,        /* self_attn.q_proj.weight (q rows then gate rows) [2*Hq*D, H] */
    DM_T_ATTN_K = 12,        /* self_attn.k_proj.weight           [Hkv*D, H]           */
    DM_T_ATTN_V = 13,        /* self_attn.v_proj.weight           [Hkv*D, H]           */
    DM_T_ATTN_Q_NORM = 14,   /* self_attn.q_norm.weight           [D]                  */
    DM_T_ATTN_K_NORM = 15,   /* self_attn.k_norm.weight           [D]                  */
    DM_T_ATTN_O = 16,        /* self_attn.o_proj.weight           [H, Hq*D]            */
    DM_T_ROUTER = 17,        /* mlp.gate.weight                   [E, H]               */
    DM_T_SHARED_GATE = 18,   /* mlp.shared_expert_gate.weight     [1, H]               */
    DM_T_EMBED = 19,         /* embed_tokens.weight (layer -1)    [V, H]               */
    DM_T_FINAL_NORM = 20,    /* norm.weight (layer -1)            [H]                  */
    DM_T_LM_HEAD = 21,       /* lm_head.weight (layer -1)         [V, H]               */
    DM_T_COUNT = 22
};

#define DM_DTYPE_BF16 0
#define DM_DTYPE_F32 1

/* Uploads one dense tensor.  `dtype` is DM_DTYPE_BF16 for every tensor except
 * DM_T_GDN_DT_BIAS / DM_T_GDN_A_LOG, which are DM_DTYPE_F32.  `n_elems` must equal the
 * tensor's element count.  layer = -1 for the global tensors (embed, final norm, lm_head). */
int32_t dm_upload_tensor(dm_ctx* ctx, int32_t layer, int32_t tensor_id, int32_t dtype,
                         const void* data_host, uint64_t n_elems);

/* Uploads one projection of one expert into the HBM-resident 4-bit expert pool.
 *   expert: 0..E-1 for routed experts, -1 for the shared expert of the layer.
 *   proj:   DM_PROJ_GATE [I, H], DM_PROJ_UP [I, H], DM_PROJ_DOWN [H, I]  (rows, cols).
 * Format (asymmetric 4-bit, group g = quant_group_size along the column axis):
 *   q_host      uint8  [rows, cols/2]   two weights per byte, LOW nibble first
 *                                       (weight 2j in bits 0-3, 2j+1 in bits 4-7; the
 *                                       nibble order of reference docs/format/
 *                                       quant_format.md:831-854)
 *   scales_host fp16   [rows, cols/g]   raw IEEE binary16 bit patterns
 *   zeros_host  uint8  [rows, cols/g/2] uint4 zero points, low nibble first
 *   w[r, c] = fp32(scale[r, c/g]) * (q[r, c] - zero[r, c/g])
 * The library repacks rows into its chunked HBM layout (16-row chunks, nibbles then
 * scales then zeros) so that one contiguous bulk copy feeds one chunk of a GEMV. */
#define DM_PROJ_GATE 0
#define DM_PROJ_UP 1
#define DM_PROJ_DOWN 2
int32_t dm_expert_upload(dm_ctx* ctx, int32_t layer, int32_t expert, int32_t proj,
                         const uint8_t* q_host, const uint16_t* scales_host,
                         const uint8_t* zeros_host);

/* Read-back of what the loaders wrote: a dense weight (dtype and n as for the upload) and
 * one expert projection in the upload format above. */
int32_t dm_tensor_download(dm_ctx* ctx, int32_t layer, int32_t tensor_id, int32_t dtype, void* out_host,
                           uint64_t n_elems);
int32_t dm_expert_download(dm_ctx* ctx, int32_t layer, int32_t expert, int32_t proj, uint8_t* q_host,
                           uint16_t* scales_host, uint8_t* zeros_host);

/* Coverage check over every tensor the configured model needs (the role of
 * validate_gguf_port_coverage, reference gguf_port_loader.mojo:70).  DM_ERR_NOT_READY
 * names the first missing tensor. */
int32_t dm_weights_check(dm_ctx* ctx);

/* Dequantises `rows x cols` weights of the 4-bit format above on the GPU and writes fp32
 * to out_host (the role of pread_and_dequant_tensor_f32, reference
 * src/format/quant_reader.mojo:710, and dequant_kernel_simd,
 * reference src/quant/dequant_kernel.mojo:22). */
int32_t dm_dequant_q4(dm_ctx* ctx, const uint8_t* q_host, const uint16_t* scales_host,
                      const uint8_t* zeros_host, int32_t rows, int32_t cols,
                      int32_t group, float* out_host);

/* The reference's own custom 4-bit file format (reference docs quant_format.md, reader
 * src/format/quant_reader.mojo:520-724): signed two's-complement nibbles in [-7, 7], low
 * nibble first, one fp16 scale per group of G in {32, 64, 128, 256}.  Dequantises n
 * elements on the GPU like dequant_kernel_simd (reference src/quant/dequant_kernel.mojo:22):
 * out_bf16_host = bf16(fp32(s_g) * q) by one round-to-nearest-even, and/or
 * out_f32_host = fp32(s_g) * q (dequant_kernel_simd_f32, :130); either may be NULL.
 * Rejects what the reference rejects, with DM_ERR_INVALID_ARG and the reason in
 * dm_last_error: G outside the set, N % G != 0, a NaN / Inf / non-positive scale (checked
 * before any copy) and the reserved nibble 0b1000 (found by the kernel; nothing is
 * written to the outputs). */
int32_t dm_dequant_sym4(dm_ctx* ctx, const uint8_t* packed_host, const uint16_t* scales_host,
                        int64_t num_elements, int32_t group_size, uint16_t* out_bf16_host,
                        float* out_f32_host);

/* ---- sequence state: the KV-cache object and GDN state -------------------------------
 * KV cache: paged bf16, 16-token pages.  Page p of slot s holds tokens
 * [16p, 16p+16) at physical page page_table[s][p]; layout per attention layer
 * [page][K|V][Hkv][16][D].  Append contract of reference LayerKVCache.append_decode_token
 * (reference src/layers/kv_cache.mojo:302-345): pos == current_len and
 * current_len + 1 <= capacity; bf16 store by single round-to-nearest-even. */

/* Resets slot: length 0, GDN recurrent state and conv window zeroed (reference
 * GDNState.zero, gdn.mojo:64-124; GatedAttnKVCache.zero, gated_attention.mojo:148), and
 * assigns the identity page table [s*max_pages_per_seq + p] when the pool is large enough
 * (otherwise the caller must set one with dm_seq_set_page_table). */
int32_t dm_seq_reset(dm_ctx* ctx, int32_t slot);
/* Installs an explicit page table (pages[n_pages], each in [0, kv_num_pages)). */
int32_t dm_seq_set_page_table(dm_ctx* ctx, int32_t slot, const int32_t* pages_host,
                              int32_t n_pages);
/* Current length (= position of the next token) of the slot. */
int32_t dm_seq_get_len(dm_ctx* ctx, int32_t slot, int32_t* len_out);
/* Sets the slot length (position of the next decode token) without touching KV or GDN
 * contents, e.g. before importing a KV cache and GDN state for an existing context.  The
 * GDN conv window of dm_gdn_state_import/export is relative to this length. */
int32_t dm_seq_set_len(dm_ctx* ctx, int32_t slot, int32_t len);
/* Writes n_tokens of K and V (bf16 bits, [n_tokens][Hkv][D] each) for attention layer
 * att_layer (0-based among attention layers) into the slot's pages, positions
 * [0, n_tokens), and sets the slot length to n_tokens (reference store_prefill,
 * kv_cache.mojo:245). */
int32_t dm_kv_import(dm_ctx* ctx, int32_t att_layer, int32_t slot, const uint16_t* k_host,
                     const uint16_t* v_host, int32_t n_tokens);
/* Gathers positions [0, n_tokens) back through the page table (reference get_k_slice,
 * kv_cache.mojo:377). */
int32_t dm_kv_export(dm_ctx* ctx, int32_t att_layer, int32_t slot, uint16_t* k_host,
                     uint16_t* v_host, int32_t n_tokens);
/* GDN state of gdn_layer (0-based among GDN layers) for slot:
 *   S_host    fp32 [nv][dv][dk] (row = dv, col = dk as reference GDNState, gdn.mojo:64)
 *   conv_host fp32 [conv_k-1][2*nk*dk + nv*dv]: pre-convolution projections of the last
 *             conv_k-1 tokens, oldest first (may be NULL = zeros / not exported). */
int32_t dm_gdn_state_import(dm_ctx* ctx, int32_t gdn_layer, int32_t slot, const float* S_host,
                            const float* conv_host);
int32_t dm_gdn_state_export(dm_ctx* ctx, int32_t gdn_layer, int32_t slot, float* S_host,
                            float* conv_host);

/* ---- compute: reference-facing entry points (host buffers, one sequence) -------------- */

/* router_forward (reference src/layers/router.mojo:188): logits = W_router x, fp32
 * softmax over all experts (max-shift, exp, multiply by 1/sum; router.mojo:109-185),
 * top-k on probabilities with ties to the lower expert id and no renormalisation
 * (reference src/layers/topk.mojo:11-131), plus the shared-expert gate
 * sigmoid(w_sh . x) (reference src/layers/moe.mojo:17).  x_host [n][H] is the
 * post-attention-normalised activation; outputs ids [n][k], probs [n][k],
 * shared_gate [n] (may be NULL). */
int32_t dm_router(dm_ctx* ctx, int32_t layer, const float* x_host, int32_t n,
                  int32_t* ids_host, float* probs_host, float* shared_gate_host);

/* MoE channel mixer with residual (reference forward_port_block second half,
 * port_scheduler.mojo:286, with swiglu_forward swiglu.mojo:52, shared_gate_forward
 * moe.mojo:17 and moe_aggregate_forward moe.mojo:105):
 *   x_out = x_mid + sum_k p_k E_k(norm(x_mid)) + sigmoid(w_sh . norm(x_mid)) E_sh(norm(x_mid)) */
int32_t dm_moe_block(dm_ctx* ctx, int32_t layer, const float* x_mid_host, int32_t n,
                     float* x_out_host);

/* Token mixer with residual for layer `layer` (GDN or gated attention by layer type),
 * tokens at positions [pos_offset, pos_offset + n) of `slot`:
 *   GDN:  forward_gdn_block semantics (reference gdn.mojo:897-1183) carried across
 *         calls by the slot's conv window and recurrent state;
 *   attn: forward_attention_qwen36 semantics (reference attention.mojo:219-435) with the
 *         slot's paged KV cache (append contract above). */
int32_t dm_mixer_block(dm_ctx* ctx, int32_t layer, int32_t slot, int32_t pos_offset,
                       const float* x_host, int32_t n, float* x_mid_host);

/* forward_port_block (reference src/layers/port_scheduler.mojo:286): mixer + residual +
 * MoE + residual for one layer. */
int32_t dm_block_forward(dm_ctx* ctx, int32_t layer, int32_t slot, int32_t pos_offset,
                         const float* x_host, int32_t n, float* x_out_host);

/* Macro scheduler over all layers for n tokens appended to `slot` at its current length
 * (reference forward_port_macro_scheduler_gguf, gguf_port_loader.mojo:329, with the
 * embedding gguf_embed_tokens :274, final norm + lm_head gguf_logits_from_hidden :291 and
 * argmax_sample cmd_decode.mojo:115).  Tokens are processed one at a time through the
 * captured decode graph.  logits_host [V] receives the logits of the last token (may be
 * NULL); next_token receives their argmax (first maximum wins). */
int32_t dm_forward(dm_ctx* ctx, int32_t slot, const int32_t* tokens_host, int32_t n,
                   float* logits_host, int32_t* next_token);

/* The same call as dm_forward for a prompt (reference cmd_decode.mojo:1958-1971: the prefill
 * call of forward_port_macro_scheduler_gguf with seq = n; cmd_forward.mojo:1221), run as
 * chunked prefill: chunks of up to dm_prefill_rows tokens go through every layer together
 * (dense projections and experts as tensor-core GEMMs over the chunk's tokens, the GDN
 * recurrence over the chunk, causal attention over the cache plus the chunk), the K/V of every
 * prompt token appended and the GDN state and conv window advanced as n decode steps would.
 * Numerics are those of the batched step (experts with fp16-rounded weights).  logits_host
 * [V] receives the last token's logits (may be NULL), next_token their argmax. */
int32_t dm_prefill(dm_ctx* ctx, int32_t slot, const int32_t* tokens_host, int32_t n, float* logits_host,
                   int32_t* next_token);
/* Rows (prompt tokens) of one prefill chunk, and the kernel launches of a chunk. */
int32_t dm_prefill_rows(dm_ctx* ctx, int32_t* rows_out, int32_t* kernels_per_chunk_out);

/* One decode step (the per-step call of reference cmd_decode.mojo:2014-2045): embeds
 * token_in at the slot's current position, runs every block and the head, appends KV,
 * advances the slot by one and returns the greedy next token (and logits if non-NULL). */
int32_t dm_decode_step(dm_ctx* ctx, int32_t slot, int32_t token_in, int32_t* token_out,
                       float* logits_host);

/* Greedy generation: n_steps decode steps fed back on the device (no host round trip
 * between steps); tokens_out_host [n_steps] receives the generated ids. */
int32_t dm_generate(dm_ctx* ctx, int32_t slot, int32_t token_in, int32_t n_steps,
                    int32_t* tokens_out_host);

/* ---- batched decode (B sequences, one token each per step) ---------------------------
 * The batched form of the decode step the reference runs per sequence (cmd_decode.mojo
 * 2014-2045 over forward_port_macro_scheduler_gguf, gguf_port_loader.mojo:329): row i
 * decodes one token of sequence slot slots[i].  Per row the semantics equal
 * dm_decode_step's; the dense projections run as tensor-core GEMMs of the rows (fp32
 * activations split into two bf16 terms), the routing is the same canonical router, the
 * experts run on the tensor cores grouped by expert.  Slots must be distinct; every slot
 * must be ready to decode (as for dm_decode_step).  The batch holds at most
 * dm_batch_capacity rows (min(max_seqs, 64)). */
int32_t dm_batch_capacity(dm_ctx* ctx, int32_t* cap_out);
/* One step: tokens_out_host [n] greedy next tokens; logits_host [n][V] (may be NULL). */
int32_t dm_decode_batch(dm_ctx* ctx, const int32_t* slots_host, const int32_t* tokens_in_host, int32_t n,
                        int32_t* tokens_out_host, float* logits_host);
/* n_steps greedy steps fed back on the device; tokens_out_host [n_steps][n]. */
int32_t dm_generate_batch(dm_ctx* ctx, const int32_t* slots_host, const int32_t* tokens_in_host, int32_t n,
                          int32_t n_steps, int32_t* tokens_out_host);
/* Enqueues n_steps batched steps without synchronising (tokens recorded on the device);
 * dm_batch_read_generated copies the [n_steps][n] tokens of the last enqueue to the host
 * after synchronising. */
int32_t dm_enqueue_decode_batch(dm_ctx* ctx, const int32_t* slots_host, const int32_t* tokens_in_host, int32_t n,
                                int32_t n_steps);
int32_t dm_batch_read_generated(dm_ctx* ctx, int32_t n, int32_t n_steps, int32_t* tokens_out_host);
/* ---- expert-parallel batched decode (one process per GPU of one node) ------------------
 * Every rank holds the same weights and runs dm_decode_batch on its own sequences with the
 * same row count n.  Expert e is computed by rank e / (num_experts / world) for the rows
 * of every rank: its kernels read the row from the source rank's memory and write the
 * result into the source rank's memory (CUDA IPC mappings over NVLink), with two
 * cross-GPU flag barriers per MoE layer (bounded waits, DM_ERR_TIMEOUT on expiry).
 * dm_ep_ipc_handle gives this context's DM_EP_HANDLE_BYTES-byte handle; the caller
 * exchanges the handles of all ranks (e.g. with torch.distributed) and passes them in
 * rank order to dm_ep_attach on every rank, then joins the ranks before the first step.
 * The world must divide num_experts; world <= 8. */
#define DM_EP_HANDLE_BYTES 64
int32_t dm_ep_ipc_handle(dm_ctx* ctx, void* handle_out);
int32_t dm_ep_attach(dm_ctx* ctx, int32_t rank, int32_t world, const void* handles);
int32_t dm_ep_detach(dm_ctx* ctx);
/* Launches per batched step: own kernels and library GEMMs. */
int32_t dm_batch_kernels_per_step(dm_ctx* ctx, int32_t n, int32_t* own_out, int32_t* gemms_out);
/* Times `iters` launches of one batched kernel (DM_BKERNEL_*) for the n rows of the last
 * batched call, each alone after an L2-evicting read; bytes = algorithmic bytes/launch. */
int32_t dm_time_batch_kernel(dm_ctx* ctx, int32_t n, int32_t which, int32_t layer, int32_t iters, float* avg_ms,
                             uint64_t* bytes);

/* ---- device-resident entry points (for callers that keep data in HBM) ---------------- */
/* Enqueues n_steps greedy decode steps for `slot` on the context stream with the input
 * token already on the device (the token produced by the previous step, or the one set by
 * dm_set_token); returns without synchronising. */
int32_t dm_enqueue_decode(dm_ctx* ctx, int32_t slot, int32_t n_steps);
int32_t dm_set_token(dm_ctx* ctx, int32_t slot, int32_t token);
/* Waits for the context stream and returns the device error word as a status. */
int32_t dm_sync(dm_ctx* ctx);
/* The context's CUDA stream (cudaStream_t) for event timing by the caller. */
int32_t dm_get_stream(dm_ctx* ctx, void** stream_out);
/* Number of kernel launches one decode step performs (for launch accounting). */
int32_t dm_kernels_per_step(dm_ctx* ctx, int32_t* out);

/* Times `iters` launches of one kernel kind of layer `layer` (inputs as left by the last
 * step) with CUDA events on the context stream, each launch alone and after a 256 MB read
 * that evicts the L2 (allocated on the first call, freed with the context); avg_ms = mean
 * launch time, bytes = the algorithmic HBM bytes one launch must move (weights, state, KV). */
#define DM_KERNEL_MIXER_IN 0   /* GDN or attention input projection GEMV (+RMSNorm)     */
#define DM_KERNEL_MIXER_OUT 1  /* output projection GEMV (+head norm / gate, residual)  */
#define DM_KERNEL_MIXER_CORE 2 /* paged decode attention; GDN recurrence (fused with the
                                  output projection when the step runs them as one)    */
#define DM_KERNEL_ROUTER 3     /* router + top-k alone (the dm_router kernel)           */
#define DM_KERNEL_MOE 4        /* the whole MoE mixer: router, experts, residual        */
#define DM_KERNEL_HEAD 6
/* kernels of the batched step for dm_time_batch_kernel */
#define DM_BKERNEL_ATTN 0      /* batched paged decode attention of an attention layer  */
#define DM_BKERNEL_GDN_REC 1   /* batched GDN recurrence of a GDN layer                  */
#define DM_BKERNEL_EXPERTS 2   /* gate/up + down expert kernels (last layer's grouping)  */
#define DM_BKERNEL_ROUTER 3    /* canonical RMSNorm + router rows + softmax/top-k        */
#define DM_BKERNEL_GEMM_IN 4   /* the layer's input projection on the tensor-core GEMM  */
int32_t dm_time_kernel(dm_ctx* ctx, int32_t which, int32_t layer, int32_t iters, float* avg_ms,
                       uint64_t* bytes);

/* Phase tracing (the role of the reference's SchedulerTimings, port_scheduler.mojo:46):
 * when on, kernels stamp %globaltimer (ns) at their phase boundaries into a 1024-slot
 * device buffer; slots 64.. hold 6 per decode-attention CTA (CTA = split * Hkv + kv head:
 * start, ready, pages done, cluster merged, end, SM id); slots 0-7 decode attention (start, page loads issued, inputs ready,
 * q/k ready, pages done, cluster merged, counted in, output), slots 16-24 the MoE kernel
 * of CTA 0 (start, inputs ready, normalised, router rows done, router complete, ids known,
 * experts up done, barrier passed, done) and 26-34 the same for the last CTA; 36-39 the
 * top-k steps of CTA 0, 40-55 decode attention per page (pages 0-3: waited, scores,
 * softmax, P V), 56-58 the MoE down phase of CTA 0 (h staged, chunks waited, computed),
 * 59 / 60 SM cycles of the MoE down-phase arithmetic / top-k rounds, 1024.. 8 per MoE CTA.  Turning
 * tracing on or off drops captured decode graphs (they are recaptured on next use). */
int32_t dm_trace_enable(dm_ctx* ctx, int32_t on);
int32_t dm_trace_read(dm_ctx* ctx, uint64_t* stamps_host, int32_t n);
/* Timeline of the last traced decode step: for launch i, rec[4i..4i+2] = %globaltimer ns at
 * the first CTA's start, at the end of its griddepcontrol.wait and at the last CTA's end;
 * kinds[i] = (kind << 16) | layer with kind 0 embed, 1 GDN in-proj, 2 GDN recurrence,
 * 3 GDN out-proj, 4 attention in-proj, 5 decode attention, 6 attention out-proj, 7 MoE,
 * 8 head.  count receives the number of records (<= n). */
int32_t dm_trace_timeline(dm_ctx* ctx, uint64_t* rec_host, int32_t* kinds_host, int32_t n,
                          int32_t* count);

/* ---- MoE mixer without allocation ---------------------------------------------------
 * No counterpart in the reference: its MoE block (forward_port_block second half,
 * port_scheduler.mojo:286) always runs inside its own engine, which owns every buffer.
 *
 * dm_moe_layer_noalloc computes what dm_moe_block computes for one token (post-attention
 * RMSNorm, router, top-k, the k routed experts and the shared expert, residual) with the
 * same fused kernel, but over buffers the CALLER owns on the current device, and it
 * allocates nothing: no cudaMalloc/cudaFree and no allocating library routine.  It is for
 * a host runtime that keeps expert records in a cache of its own (streamed from disk) and
 * has committed the rest of device memory to that cache, and so cannot let a library
 * allocate during a step.  No dm_ctx is involved.
 *
 * Scratch: one fixed array of DM_NOALLOC_SCRATCH_BYTES (64 KiB) compiled into the library,
 * per device.  A layer needs 512 + 8192 + 256 + 4*H + 4*(k + 1)*I bytes of it; larger
 * layers are rejected with DM_ERR_INVALID_ARG and a SCRATCH_LIMIT message.  Supported
 * (hidden, intermediate) pairs: (256,128) (1024,256) (2048,256) (2048,512), and
 * (4096,512) only on a GPU with at least 256 SMs (the kernel needs hidden/16 <= SMs; a
 * B200 has 148); num_experts <= 512, num_experts_per_tok <= 16, group size 64.  Other
 * shapes are rejected with DM_ERR_INVALID_ARG and a CONFIG_ERROR message.
 *   - Calls that overlap on the GPU share the one array and race.  Within one process
 *     the library serialises them (a mutex held from the first enqueue to the final
 *     stream synchronisation); callers in different processes on the same device must
 *     serialise themselves.
 *   - The kernel keeps one CTA resident on every SM and its phases wait on each other
 *     with bounded waits: kernels the caller runs at the same time on other streams can
 *     delay residency past the bound, and the call then returns DM_ERR_TIMEOUT.
 *   - The array keeps what the last call left in it; each call clears the part that must
 *     start at zero (counters, flags, error word) on `stream` before its launch.
 *   - The first call on a device does the set-up (scratch address, kernel attributes)
 *     with that device current; make it before any stream capture.
 * Buffers (device memory of the current device):
 *   router_dev    bf16 [num_experts + 1][H]: router rows, then the shared-expert gate row
 *   post_norm_dev bf16 [H]
 *   experts_dev   num_experts expert records, shared_dev one record, each in the chunked
 *                 4-bit layout dm_expert_upload writes (gate/up chunks, then down chunks;
 *                 record bytes = (I/8) * 16*(H/2 + H/32 + H/128) + (H/16) * 16*(I/2 + I/32 + I/128))
 *   x_mid_dev fp32 [H] in, x_out_dev fp32 [H] out (must not overlap x_mid_dev)
 *   ids_dev int32 [k], probs_dev fp32 [k]: top-k ids / probabilities, or NULL
 * The call runs on `stream` (a cudaStream_t, NULL = legacy default stream) and returns
 * after it has synchronised that stream.  err_buf (may be NULL) receives a JSON error
 * object like dm_last_error's. */
#define DM_NOALLOC_SCRATCH_BYTES 65536
int32_t dm_moe_layer_noalloc(int32_t hidden_size, int32_t moe_intermediate_size,
                             int32_t num_experts, int32_t num_experts_per_tok, float rms_norm_eps,
                             const uint16_t* router_dev, const uint16_t* post_norm_dev,
                             const uint8_t* experts_dev, const uint8_t* shared_dev,
                             const float* x_mid_dev, float* x_out_dev, int32_t* ids_dev,
                             float* probs_dev, void* stream, char* err_buf, uint64_t err_buf_size);

/* ---- synthetic checkpoint (seeded; host and device generate the same distributions) --
 * Counter-based generator: element i of stream `stream_id` under `seed` is a pure
 * function of (seed, stream_id, i), so any subrange can be produced independently. */
/* bf16 N(mean, std) */
int32_t dm_synth_bf16(uint64_t seed, uint64_t stream_id, uint64_t n, float mean, float std,
                      uint16_t* out_host);
/* f32 N(mean, std) */
int32_t dm_synth_f32(uint64_t seed, uint64_t stream_id, uint64_t n, float mean, float std,
                     float* out_host);
/* uniform bytes (two uniform nibbles per byte) */
int32_t dm_synth_u8(uint64_t seed, uint64_t stream_id, uint64_t n, uint8_t* out_host);
/* fp16 |N(0, std)| scales */
int32_t dm_synth_f16_absnormal(uint64_t seed, uint64_t stream_id, uint64_t n, float std,
                               uint16_t* out_host);
/* Seeded synthetic sequence state for every slot (benchmarks): the whole KV page pool bf16
 * N(0, kv_std), every GDN state and conv window fp32 N(0, state_std); every slot's length
 * becomes len.  Page tables are unchanged. */
int32_t dm_synth_state_device(dm_ctx* ctx, uint64_t seed, float kv_std, float state_std, int32_t len);
/* W += beta u^T on an uploaded bf16 dense tensor (rows x cols), one rounding per element. */
int32_t dm_tensor_add_rank1(dm_ctx* ctx, int32_t layer, int32_t tensor_id, const float* beta_host, int64_t rows,
                            const float* u_host, int32_t cols);
/* Routing statistics of batched steps since the last reset: [0] sum over (layer, step) of
 * routed experts touched, [1] sum of expert segments, [2] max rows of one routed expert,
 * [3] (layer, step) count.  reset != 0 clears them afterwards; out4 may be NULL. */
int32_t dm_batch_stats(dm_ctx* ctx, int32_t reset, uint32_t* out4);
/* Per-expert router logit offsets of layer `layer` (n == num_experts values), added after
 * the canonical dot product; NULL removes them.  Not part of the reference model (whose
 * router has no bias): a synthetic-workload device to draw a skewed expert load. */
int32_t dm_set_router_bias(dm_ctx* ctx, int32_t layer, const float* bias_host, int32_t n);
/* ---- session files (reference format KMSS v1, src/format/kmss.mojo) -------------------
 * Header 128 B (magic "KMSS", version 1, architecture 2, manifest hash, dimensions, byte
 * counts), KV cache [K|V][pos][attention layer][kv head][head_dim] as fp32 (kv_dtype 1) or
 * bf16 (2), GDN states [gdn layer][nv * dv][dk] fp32 (the reference's [layers][dv][dk]
 * with the V heads stacked), token ids u32, SHA-256 of all of it; written to path.tmp and
 * renamed.  seq_len = max(the slot's length, n_tokens).  Loading checks magic, version,
 * architecture, byte counts, file size and checksum (reference error types
 * FORMAT_MISMATCH, VERSION_MISMATCH, CONFIG_MISMATCH, LAYOUT_MISMATCH,
 * CORRUPT_SESSION_CHECKSUM) and that the dimensions match this context, then imports the
 * KV pages and GDN states into `slot` and sets its length.  The format has no field for
 * the GDN conv window: a loaded slot starts with it zero.  tokens_out receives up to cap
 * ids; *n_tokens the file's seq_len. */
int32_t dm_kmss_save(dm_ctx* ctx, int32_t slot, const char* path, const int32_t* tokens, int32_t n_tokens,
                     int32_t kv_dtype, const uint8_t* manifest_hash32);
int32_t dm_kmss_load(dm_ctx* ctx, int32_t slot, const char* path, int32_t* tokens_out, int32_t cap,
                     int32_t* n_tokens);
/* Lossless resume: the GDN conv window (not a KMSS v1 field) in a sidecar file bound to the
 * KMSS file by its SHA-256 trailer ("KMCV", version, layers, qkv_dim, length, the KMSS
 * trailer, fp32 [layers][3][qkv_dim], SHA-256).  save: after dm_kmss_save of the same slot;
 * load: after dm_kmss_load into the slot (rejects another file's sidecar, a length or size
 * mismatch and a corrupted file).  Without a sidecar a loaded slot starts from a zero window,
 * as the reference's port semantics have none. */
int32_t dm_kmss_save_conv(dm_ctx* ctx, int32_t slot, const char* kmss_path, const char* conv_path);
int32_t dm_kmss_load_conv(dm_ctx* ctx, int32_t slot, const char* kmss_path, const char* conv_path);
/* Copies the whole sequence state of slot src into slot dst on the device (K/V of every
 * position through both page tables, GDN states and conv windows, length, next token): the
 * snapshot and restore of the prefix cache (reference PrefixCache, core/prefix_cache.mojo:102,
 * whose entries hold a copy of the KV cache and GDN state). */
int32_t dm_seq_copy(dm_ctx* ctx, int32_t src_slot, int32_t dst_slot);
/* SHA-256 of n bytes (FIPS 180-4); needs no device. */
int32_t dm_sha256(const uint8_t* data, uint64_t n, uint8_t* out32);

/* ---- spilling expert pool (expert_cache_slots = C > 0) --------------------------------
 * The routed experts of every layer live in pinned host memory; C of them per layer are
 * resident in HBM.  Each batched step brings, per layer, the experts its rows selected into
 * HBM before the expert kernels run (host -> device copies on the context stream) and
 * evicts the least recently used unpinned ones (the contract of the reference's expert
 * cache, src/io/lru_cache.mojo:225-610).  Single-sequence decode (dm_decode_step,
 * dm_forward, dm_generate) runs as one-row batched steps; dm_enqueue_decode,
 * dm_block_forward, dm_moe_block, the kernel timers and expert-parallel groups need every
 * expert resident and return DM_ERR_INVALID_ARG.  A step needs n * top-k + pinned <= C
 * (DM_ERR_CAPACITY otherwise, before any work).
 * out8: accesses, hits, misses, evictions, records loaded, pins kept unpinned (over the
 * 25 % pin budget), bytes copied host -> device, C (0 when the pool does not spill). */
int32_t dm_spill_stats(dm_ctx* ctx, uint64_t* out8);
/* Makes expert `expert` of `layer` resident and pins it while the pinned records of the
 * layer stay within 25 % of C; *pinned = 1 if pinned, 0 if kept unpinned. */
int32_t dm_spill_pin(dm_ctx* ctx, int32_t layer, int32_t expert, int32_t* pinned);
/* The residency policy alone on a trace of routed ids ([steps][L][n][topk]) after the
 * given (layer, expert) pins, no device: stats_out as out8[0..5]; slot_of_out [L][E] the
 * final slot of every expert (-1 = host only).  Either output may be NULL. */
int32_t dm_spill_simulate(int32_t L, int32_t E, int32_t C, int32_t steps, int32_t n, int32_t topk, const int32_t* ids,
                          const int32_t* pins, int32_t npins, uint64_t* stats_out, int32_t* slot_of_out);

/* Fills every weight of the context with the synthetic distributions of the benchmark
 * configs directly on the device (same generator; used for multi-GB models). */
int32_t dm_synth_model_device(dm_ctx* ctx, uint64_t seed);

/* ---- quant-file loaders: the reference's on-disk weight formats ----------------------
 * GGUF v2/v3 (reference src/format/gguf.mojo) and the reference's custom 4-bit quant file
 * (src/format/quant_reader.mojo), parsed on the host and streamed into the HBM pool:
 * dense tensors are dequantised on the GPU straight into the context's weights, experts
 * are converted into the pool's asymmetric 4-bit form (exactly for the custom format with
 * group >= the pool group; otherwise by round-to-nearest re-quantisation, which the
 * caller has to ask for).  The index functions need no device and no context; `err`
 * receives the reference-shaped error JSON. */
#define DM_GGML_F32 0
#define DM_GGML_F16 1
#define DM_GGML_Q8_0 8
#define DM_GGML_Q3_K 11
#define DM_GGML_Q4_K 12
#define DM_GGML_BF16 30
/* Q4_K sub-blocks 4..7: read scale and min as gguf.mojo:478-485 does (byte j-4 and byte j
 * of the 12 scale bytes) instead of the GGUF layout oracle_port.py:108-112 follows
 * (bytes j-4, j and j+4).  The two agree when those bytes are equal. */
#define DM_GGUF_Q4K_MOJO 1u
/* Expert loads may re-quantise (lossy) what the pool cannot hold exactly. */
#define DM_LOAD_REQUANT 2u

typedef struct dm_gguf dm_gguf;
typedef struct {
    const char* name;      /* valid until dm_gguf_close */
    int32_t ndim;
    int32_t ggml_type;
    uint64_t dims[8];      /* GGUF order: dims[0] is the innermost (contiguous) axis */
    uint64_t offset;       /* relative to the data section */
    uint64_t file_offset;  /* absolute */
    uint64_t num_elements;
    uint64_t raw_bytes;
} dm_gguf_tensor_info;

/* parse_gguf_index (gguf.mojo:257-411): magic, version 2 or 3, tensor count <= 100000,
 * metadata (general.alignment), tensor directory (ndim 1..8), data section aligned, every
 * tensor inside the file, and the exact file size data_start + max tensor end.
 * DM_ERR_IO when the file cannot be read, DM_ERR_FORMAT with error_type
 * GGUF_FILE_CORRUPT and the reference's message otherwise. */
int32_t dm_gguf_open(const char* path, dm_gguf** out, char* err, uint64_t err_size);
void dm_gguf_close(dm_gguf* g);
int32_t dm_gguf_summary(const dm_gguf* g, uint32_t* version, uint64_t* tensor_count, uint64_t* kv_count,
                        uint64_t* alignment, uint64_t* data_offset, uint64_t* file_size);
int32_t dm_gguf_tensor(const dm_gguf* g, int64_t index, dm_gguf_tensor_info* out);
int64_t dm_gguf_find(const dm_gguf* g, const char* name); /* -1 when absent */
/* Metadata as the reference's index.metadata strings: integers (and f32/f64 as their raw
 * bit patterns) in decimal, strings verbatim, arrays "[Array of N elements]". */
int32_t dm_gguf_meta_key(const dm_gguf* g, int64_t index, char* buf, uint64_t size);
int32_t dm_gguf_meta(const dm_gguf* g, const char* key, char* buf, uint64_t size);
/* Raw bytes [byte_offset, byte_offset + n) of tensor `index` (pread). */
int32_t dm_gguf_read(const dm_gguf* g, int64_t index, uint64_t byte_offset, void* dst, uint64_t n);
/* (elements, bytes) per block of a GGML type (get_ggml_block_specs, gguf.mojo:76-102). */
int32_t dm_ggml_block_spec(int32_t type, int32_t* block_elems, int32_t* block_bytes);

/* Dequantises n elements of GGML blocks on the GPU (dequantize_q8_0 / _q4_k / _q3_k,
 * gguf.mojo:414-561, oracle_port.py:68-159; F32, F16, BF16 converted): fp32 with the
 * reference's roundings into out_f32_host and/or its bf16 rounding (nearest even) into
 * out_bf16_host.  raw_bytes must hold the n / block elements blocks; n a multiple of the
 * block.  flags: DM_GGUF_Q4K_MOJO. */
int32_t dm_gguf_dequant(dm_ctx* ctx, int32_t ggml_type, const void* raw_host, uint64_t raw_bytes,
                        uint64_t n_elements, uint32_t flags, float* out_f32_host, uint16_t* out_bf16_host);
/* GGUF tensor `name` -> dense weight (layer, tensor_id) of the context (the role of
 * stream_gguf_tensor_f32, gguf.mojo:563-626, for one weight): element counts must match;
 * bf16 weights take the fp32 value rounded to nearest even, fp32 weights take it as is. */
int32_t dm_gguf_load_tensor(dm_ctx* ctx, const dm_gguf* g, const char* name, int32_t layer, int32_t tensor_id,
                            uint32_t flags);
/* One expert projection from a GGUF tensor: rows x cols = the projection's shape, taken
 * from element slab * slab_elems + row0 * cols, slab_elems = the product of the inner two
 * dims (slab = 0 and row0 = 0 for a 2-D tensor; for stacked experts [E][rows][cols]
 * slab = expert).  The pool cannot hold GGML blocks exactly, so this needs
 * DM_LOAD_REQUANT; *max_abs_err (may be NULL) receives the largest |w - w'|. */
int32_t dm_gguf_load_expert(dm_ctx* ctx, const dm_gguf* g, const char* name, int64_t slab, int64_t row0,
                            int32_t layer, int32_t expert, int32_t proj, uint32_t flags, float* max_abs_err);

typedef struct dm_quant_file dm_quant_file;
typedef struct {
    const char* name;  /* valid until dm_quant_file_close */
    const char* dtype; /* the source dtype the record names ("BF16") */
    int32_t ndim;
    int32_t group_size;
    uint64_t shape[8]; /* numpy order: shape[ndim-1] is contiguous */
    uint64_t num_groups;
    uint64_t num_elements;
    uint64_t record_offset;
    uint64_t scales_offset; /* absolute: fp16 scales, num_groups of them */
    uint64_t data_offset;   /* absolute: packed nibbles, low nibble first */
    uint64_t scales_bytes;
    uint64_t weights_bytes;
} dm_quant_tensor_info;

/* scan_quant_file (quant_reader.mojo:520-662): 256-byte JSON header (version 1, format
 * "4-bit per-group", scale dtype FP16, group in {32, 64, 128, 256}, num_tensors,
 * total_bytes == file size), then records [u32 meta_len][meta JSON][scales][nibbles]
 * back to back to the end of the file.  DM_ERR_FORMAT (error_type QUANT_FILE_CORRUPT)
 * with the reference's message on any violation. */
int32_t dm_quant_file_open(const char* path, dm_quant_file** out, char* err, uint64_t err_size);
void dm_quant_file_close(dm_quant_file* q);
int32_t dm_quant_file_summary(const dm_quant_file* q, int32_t* version, int32_t* group_size, int64_t* num_tensors,
                              uint64_t* total_bytes, char* model, uint64_t model_size);
int32_t dm_quant_file_tensor(const dm_quant_file* q, int64_t index, dm_quant_tensor_info* out);
int64_t dm_quant_file_find(const dm_quant_file* q, const char* name);
/* part 0: scale bytes, 1: nibble bytes; [byte_offset, byte_offset + n) of that part. */
int32_t dm_quant_file_read(const dm_quant_file* q, int64_t index, int32_t part, uint64_t byte_offset, void* dst,
                           uint64_t n);
/* Quant-file tensor -> dense weight (load_one_quant_tensor_bf16 / _f32,
 * src/layers/quant_loader.mojo:27-58): bf16 weights take dequant_kernel_simd's bits
 * bf16(fp32(s) q), fp32 weights fp32(s) q; the reference's rejections apply. */
int32_t dm_quant_file_load_tensor(dm_ctx* ctx, const dm_quant_file* q, const char* name, int32_t layer,
                                  int32_t tensor_id);
/* Quant-file tensor slice -> one expert projection (slab / row0 as in
 * dm_gguf_load_expert).  Exact (nibble n -> n XOR 8, zero 8, the group's scale) when the
 * file's group is a multiple of the pool group, or when the file's groups inside each
 * pool group share one scale; otherwise DM_LOAD_REQUANT re-quantises. */
int32_t dm_quant_file_load_expert(dm_ctx* ctx, const dm_quant_file* q, const char* name, int64_t slab, int64_t row0,
                                  int32_t layer, int32_t expert, int32_t proj, uint32_t flags, float* max_abs_err);
/* Every weight of the configured model from a quant file, by checkpoint names: prefix
 * "model.language_model.layers.<l>." or "model.layers.<l>." + the names of enum
 * dm_tensor_id; experts as "mlp.experts.<e>.{gate,up,down}_proj.weight" or the stacked
 * "mlp.experts.gate_up_proj" [E][2I][H] (gate rows first) and "mlp.experts.down_proj"
 * [E][H][I]; the shared expert "mlp.shared_expert.{gate,up,down}_proj.weight"; globals
 * "[model.language_model.|model.]embed_tokens.weight", "[...]norm.weight",
 * "lm_head.weight".  A weight the file lacks but that was uploaded before is kept (the
 * format's groups of >= 32 cannot hold e.g. a 4-element dt_bias); DM_ERR_NOT_READY names
 * the first weight that is still missing. */
int32_t dm_quant_file_load(dm_ctx* ctx, const dm_quant_file* q, uint32_t flags);

#ifdef __cplusplus
}
#endif
#endif /* DISMOEN_CUDA_H */
