/* A plain C host of libdismoen_cuda.so: what a non-Python binding (the Mojo external_call
 * stubs, a C++ engine) sees.  Calls only entry points that need no device: the ABI
 * version, config validation, SHA-256, the GGUF and quant-file index parsers and the spill
 * residency policy, and prints their results as one JSON object.
 *   harness <file.gguf> <file.q4>
 */
#include <stdio.h>
#include <string.h>

#include "dismoen_cuda.h"

int main(int argc, char** argv) {
    if (argc != 3) {
        fprintf(stderr, "usage: harness <file.gguf> <file.q4>\n");
        return 2;
    }
    dm_model_config m;
    memset(&m, 0, sizeof m);
    m.hidden_size = 256; m.num_hidden_layers = 4; m.full_attention_interval = 4; m.vocab_size = 1024;
    m.rms_norm_eps = 1e-6f; m.num_attention_heads = 4; m.num_key_value_heads = 1; m.head_dim = 64;
    m.rope_theta = 1e7f; m.partial_rotary_factor = 0.25f; m.linear_num_key_heads = 2;
    m.linear_num_value_heads = 4; m.linear_key_head_dim = 64; m.linear_value_head_dim = 64;
    m.linear_conv_kernel_dim = 4; m.num_experts = 16; m.num_experts_per_tok = 4;
    m.moe_intermediate_size = 128; m.shared_expert_intermediate_size = 128; m.norm_topk_prob = 0;
    m.quant_group_size = 64;
    char err[1024];
    const int cfg_ok = dm_config_validate(&m, err, sizeof err);
    m.norm_topk_prob = 1;
    const int cfg_bad = dm_config_validate(&m, err, sizeof err);

    uint8_t dig[32];
    dm_sha256((const uint8_t*)"abc", 3, dig);

    dm_gguf* g = NULL;
    const int g_rc = dm_gguf_open(argv[1], &g, err, sizeof err);
    uint64_t tc = 0, al = 0, dat = 0;
    uint32_t ver = 0;
    dm_gguf_tensor_info ti;
    memset(&ti, 0, sizeof ti);
    if (g_rc == DM_OK) {
        dm_gguf_summary(g, &ver, &tc, NULL, &al, &dat, NULL);
        dm_gguf_tensor(g, 0, &ti);
    }

    dm_quant_file* q = NULL;
    const int q_rc = dm_quant_file_open(argv[2], &q, err, sizeof err);
    int64_t nt = 0;
    int32_t qver = 0, qg = 0;
    if (q_rc == DM_OK) dm_quant_file_summary(q, &qver, &qg, &nt, NULL, NULL, 0);

    const int32_t ids[8] = {0, 1, 2, 3, 2, 3, 4, 5};  /* 2 steps x 1 layer x 1 row x top-4 */
    uint64_t st[6];
    const int sp_rc = dm_spill_simulate(1, 8, 4, 2, 1, 4, ids, NULL, 0, st, NULL);

    printf("{\"abi\": %d, \"cfg_ok\": %d, \"cfg_bad\": %d, \"sha_abc\": \"", dm_abi_version(), cfg_ok, cfg_bad);
    for (int i = 0; i < 32; ++i) printf("%02x", dig[i]);
    printf("\", \"gguf\": [%d, %u, %llu, %llu, %llu, \"%s\", %d], ", g_rc, ver, (unsigned long long)tc,
           (unsigned long long)al, (unsigned long long)dat, ti.name ? ti.name : "", ti.ggml_type);
    printf("\"quant\": [%d, %d, %d, %lld], ", q_rc, qver, qg, (long long)nt);
    printf("\"spill\": [%d, %llu, %llu, %llu, %llu]}\n", sp_rc, (unsigned long long)st[0], (unsigned long long)st[1],
           (unsigned long long)st[2], (unsigned long long)st[3]);
    if (g) dm_gguf_close(g);
    if (q) dm_quant_file_close(q);
    return 0;
}
