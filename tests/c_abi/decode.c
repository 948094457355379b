/* A plain C host driving the decode path on the GPU through the C ABI alone (what the
 * Mojo external_call stubs do): a context for the config-0 model, its weights synthesised
 * on the device (seed 0), then
 *   slot 0: the prompt through dm_forward, 8 greedy steps through dm_generate;
 *   slot 1: the same prompt through dm_prefill;
 *   both:   one dm_decode_batch step (slot 0 continues its generation, slot 1 its prompt);
 *   a bad call: a token out of range, its status and dm_last_error.
 * Prints the ids as one JSON object.
 *   decode <prompt tokens...>
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "dismoen_cuda.h"

#define CHECK(call)                                                                 \
    do {                                                                            \
        const int32_t rc_ = (call);                                                 \
        if (rc_ != DM_OK) {                                                         \
            char e_[1024];                                                          \
            dm_last_error(ctx, e_, sizeof e_);                                      \
            fprintf(stderr, "%s failed: %d %s\n", #call, (int)rc_, e_);             \
            return 1;                                                               \
        }                                                                           \
    } while (0)

int main(int argc, char** argv) {
    if (argc < 2 || argc > 65) {
        fprintf(stderr, "usage: decode <1..64 prompt tokens>\n");
        return 2;
    }
    int32_t prompt[64];
    const int n = argc - 1;
    for (int i = 0; i < n; ++i) prompt[i] = (int32_t)atoi(argv[i + 1]);

    dm_model_config m;
    memset(&m, 0, sizeof m);
    m.hidden_size = 256; m.num_hidden_layers = 4; m.full_attention_interval = 4; m.vocab_size = 1024;
    m.rms_norm_eps = 1e-6f; m.num_attention_heads = 4; m.num_key_value_heads = 1; m.head_dim = 64;
    m.rope_theta = 1e7f; m.partial_rotary_factor = 0.25f; m.linear_num_key_heads = 2;
    m.linear_num_value_heads = 4; m.linear_key_head_dim = 64; m.linear_value_head_dim = 64;
    m.linear_conv_kernel_dim = 4; m.num_experts = 16; m.num_experts_per_tok = 4;
    m.moe_intermediate_size = 128; m.shared_expert_intermediate_size = 128; m.norm_topk_prob = 0;
    m.quant_group_size = 64;
    dm_runtime_config rt;
    memset(&rt, 0, sizeof rt);
    rt.max_seqs = 2;
    rt.kv_page_tokens = 16;
    rt.max_pages_per_seq = 8;  /* 128 tokens per slot */
    rt.kv_num_pages = 16;
    rt.expert_cache_slots = 0;
    dm_ctx* ctx = NULL;
    if (dm_ctx_create(&m, &rt, 0, &ctx) != DM_OK) {
        fprintf(stderr, "dm_ctx_create failed\n");
        return 1;
    }
    CHECK(dm_synth_model_device(ctx, 0));
    CHECK(dm_weights_check(ctx));
    CHECK(dm_seq_reset(ctx, 0));
    CHECK(dm_seq_reset(ctx, 1));

    int32_t next0 = -1, next1 = -1, gen[8];
    CHECK(dm_forward(ctx, 0, prompt, n, NULL, &next0));
    CHECK(dm_generate(ctx, 0, next0, 8, gen));
    CHECK(dm_prefill(ctx, 1, prompt, n, NULL, &next1));
    int32_t len0 = 0, len1 = 0;
    CHECK(dm_seq_get_len(ctx, 0, &len0));
    CHECK(dm_seq_get_len(ctx, 1, &len1));

    const int32_t slots[2] = {0, 1};
    const int32_t toks[2] = {gen[7], next1};
    int32_t bout[2] = {-1, -1};
    CHECK(dm_decode_batch(ctx, slots, toks, 2, bout, NULL));

    const int32_t bad_tok = m.vocab_size;
    int32_t ignored = 0;
    const int32_t bad_rc = dm_forward(ctx, 0, &bad_tok, 1, NULL, &ignored);
    char bad_msg[1024];
    dm_last_error(ctx, bad_msg, sizeof bad_msg);
    for (char* p = bad_msg; *p; ++p)
        if (*p == '"' || *p == '\\') *p = '\'';

    printf("{\"next_forward\": %d, \"generate\": [", (int)next0);
    for (int i = 0; i < 8; ++i) printf("%s%d", i ? ", " : "", (int)gen[i]);
    printf("], \"next_prefill\": %d, \"len\": [%d, %d], \"batch\": [%d, %d], \"bad_rc\": %d, \"bad_msg\": \"%s\"}\n",
           (int)next1, (int)len0, (int)len1, (int)bout[0], (int)bout[1], (int)bad_rc, bad_msg);
    dm_ctx_destroy(ctx);
    return 0;
}
