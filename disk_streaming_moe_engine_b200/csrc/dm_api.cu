// dm_api.cu — host runtime and C ABI of libdismoen_cuda.so.
//
// The context owns one device arena holding every weight, state and scratch buffer; it is
// sized from the config at creation, so no allocation happens on the decode path.  Layer
// kernels are issued on the context stream with programmatic dependent launch; the decode
// step (embedding, all blocks, head) is captured once per sequence slot into a CUDA graph
// and replayed per token.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "dismoen_cuda.h"
#include "dm_internal.h"
#include "dm_kernels.h"
#include "dm_synth.h"

namespace dm {
cudaError_t launch_dequant_q4_canonical(cudaStream_t st, const uint8_t* q, const uint16_t* s,
                                        const uint8_t* z, int rows, int cols, int group, float* out);
cudaError_t launch_repack_rows(cudaStream_t st, const uint8_t* q, const uint16_t* s, const uint8_t* z,
                               int rows, int cols, int group, int kind, uint8_t* dst);
bool moe_supported(int H, int I, int G);
bool attn_supported(int D, int grp);
int attn_scores_cap(int max_pages, int nsplit);
int attn_nsplit(int num_sms, int Hkv);
cudaError_t launch_rope_table(cudaStream_t st, float2* tab, int capacity, int rot_dim, float theta);
cudaError_t launch_dequant_sym4(cudaStream_t st, const uint8_t* packed, const uint16_t* scales, int64_t n, int group,
                                uint16_t* out_bf16, float* out_f32, unsigned* bad);
cudaError_t launch_l2_flush_read(cudaStream_t st, const void* buf, size_t bytes, int num_sms);
cudaError_t launch_kv_copy(cudaStream_t st, uint16_t* kv_layer, const int* page_table_row, int Hkv,
                           int D, uint16_t* k, uint16_t* v, int n_tokens, int to_cache);
cudaError_t launch_kv_seq_copy(cudaStream_t st, uint16_t* kv_layer, const int* pt_src, const int* pt_dst, int Hkv,
                               int D, int num_pages, int n_tokens, uint32_t* err);
cudaError_t launch_synth_bf16(cudaStream_t st, uint16_t* dst, uint64_t n, uint64_t seed,
                              uint64_t stream_id, float mean, float std);
cudaError_t launch_synth_f32(cudaStream_t st, float* dst, uint64_t n, uint64_t seed, uint64_t stream_id,
                             float mean, float std);
cudaError_t launch_synth_u8(cudaStream_t st, uint8_t* dst, uint64_t n, uint64_t seed, uint64_t stream_id);
cudaError_t launch_rank1_add_bf16(cudaStream_t st, uint16_t* W, int64_t rows, int cols, const float* beta,
                                  const float* u);
cudaError_t launch_synth_f16abs(cudaStream_t st, uint16_t* dst, uint64_t n, uint64_t seed,
                                uint64_t stream_id, float std);
bool gguf_type_supported(int type);
cudaError_t launch_gguf_dequant(cudaStream_t st, int type, const uint8_t* raw, int64_t n, unsigned flags,
                                float* out_f32, uint16_t* out_bf16);
cudaError_t launch_sym4_to_pool(cudaStream_t st, const uint8_t* packed, const uint16_t* scales, int64_t e0, int rows,
                                int cols, int gf, int gp, uint8_t* q_out, uint16_t* s_out, uint8_t* z_out,
                                unsigned* flags);
cudaError_t launch_requant_pool(cudaStream_t st, const float* w, int rows, int cols, int gp, uint8_t* q_out,
                                uint16_t* s_out, uint8_t* z_out, unsigned* flags, unsigned* max_err_bits);
}  // namespace dm

using namespace dm;

struct dm_ctx {
    CUtensorMap kv_map{};  // 2-D tiled view of the KV arena for the attention page copies
    std::vector<CUtensorMap> xmaps;  // [L][2] the expert pools' nibble rows (gate/up, down)
    std::vector<CUtensorMap> dmaps;  // [L][2] + 1: dense weights (input, output projection; lm_head last)
    dm_model_config mc{};
    dm_runtime_config rc{};
    Dims d{};
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0;
    std::vector<LayerW> layers;
    uint16_t* embed = nullptr;
    uint16_t* final_norm = nullptr;
    uint16_t* lm_head = nullptr;
    Buffers b{};
    // upload staging for one expert projection
    uint8_t* stage_q = nullptr;
    uint16_t* stage_s = nullptr;
    uint8_t* stage_z = nullptr;
    // quant-file loader staging (allocated on first use): pinned host chunk, device chunk,
    // an fp32 projection buffer and two status words
    void* ld_host = nullptr;
    uint8_t* ld_dev = nullptr;
    // spilling expert pool (expert_cache_slots > 0): every routed record in pinned host
    // memory, the residency policy, the device slot table and its pinned host mirror
    uint8_t* host_pool = nullptr;   // [L][E] records
    uint8_t* scratch_rec = nullptr; // device staging record of uploads
    int* d_slot_of = nullptr;       // [L][E] device
    int* h_slot_of = nullptr;       // [L][E] pinned host
    int* h_sids = nullptr;          // [kMaxBatch * topk] pinned host: the routed ids of a layer
    SpillPolicy spill;
    uint64_t spill_bytes = 0;
    float* ld_f32 = nullptr;
    unsigned* ld_word = nullptr;
    // pinned host staging for per-step transfers
    int* h_io = nullptr;  // [0] token in, [1] token out, [2] error word, [3] pos
    // coverage
    std::vector<uint8_t> have_dense;   // [(L+1) * DM_T_COUNT]
    std::vector<uint8_t> have_expert;  // [L * (E+1) * 3]
    // host mirror of sequence state
    std::vector<int> slot_len;         // [max_seqs]
    std::vector<int> att_len;          // [n_att * max_seqs]
    std::vector<int> dev_pos_valid;    // device pos[slot] == slot_len[slot]
    std::vector<cudaGraphExec_t> graphs;  // decode step per slot
    // batched decode: scratch, the GEMM library handle on the context stream (workspace in
    // the arena, so capture into a graph allocates nothing), one graph per (rows, logits)
    BatchBuffers bb{};
    BatchBuffers pb{};  // prefill chunk scratch (rows = prompt tokens of one sequence)
    std::vector<cudaGraphExec_t> bgraphs;  // [2 * (cap + 1)]
    int* h_bio = nullptr;                  // pinned [4 * kMaxBatch]: slots, tokens in, tokens out
    float* rbias = nullptr;                // [L][E] router logit offsets (dm_set_router_bias)
    // expert-parallel group: the peers' arenas mapped into this process (null for self)
    std::vector<uint8_t*> peer_arena;
    bool gdn_fused = false;  // the fused GDN kernel's grid fits one CTA per SM (set at creation)
    uint64_t* trace_buf = nullptr;
    uint64_t* ktrace_buf = nullptr;
    uint8_t* flush_buf = nullptr;  // L2 flush target of dm_time_kernel (allocated on first use)
    int trace_n = 0;
    std::vector<int> trace_kinds;
    std::string last_error;
};

// ------------------------------------------------------------------------------------
static int set_err(dm_ctx* c, int code, const char* type, const char* stage, int layer, const char* fmt, ...) {
    char detail[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(detail, sizeof detail, fmt, ap);
    va_end(ap);
    for (char* p = detail; *p; ++p)
        if (*p == '"' || *p == '\\') *p = '\'';
    char buf[768];
    snprintf(buf, sizeof buf, "{\"error_type\":\"%s\",\"detail\":\"%s\",\"stage\":\"%s\",\"layer\":%d}", type,
             detail, stage, layer);
    if (c) c->last_error = buf;
    return code;
}

#define DM_CUDA(c, call, stage)                                                                    \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess)                                                                     \
            return set_err((c), DM_ERR_CUDA, "CUDA_ERROR", (stage), -1, "%s: %s", #call,           \
                           cudaGetErrorString(e_));                                                \
    } while (0)

static int validate_config(const dm_model_config* m, char* msg, size_t n) {
    auto fail = [&](const char* type, const char* what) {
        if (msg && n) snprintf(msg, n, "{\"error_type\":\"%s\",\"detail\":\"%s\",\"stage\":\"config\",\"layer\":-1}", type, what);
        return DM_ERR_INVALID_ARG;
    };
    if (!m) return fail("CONFIG_ERROR", "null config");
    // reference ModelConfig.__init__ checks (config.mojo:31-147)
    if (m->hidden_size <= 0 || m->num_hidden_layers <= 0 || m->num_attention_heads <= 0 || m->vocab_size <= 0)
        return fail("CONFIG_ERROR", "invalid model dimensions: all sizes must be > 0");
    if (m->num_experts <= 0 || m->num_experts_per_tok <= 0 || m->num_experts_per_tok > m->num_experts)
        return fail("CONFIG_ERROR", "invalid MoE topology: 0 < num_experts_per_tok <= num_experts");
    if (m->moe_intermediate_size <= 0 || m->shared_expert_intermediate_size <= 0)
        return fail("CONFIG_ERROR", "invalid MoE intermediate sizes: must be > 0");
    if (m->num_key_value_heads <= 0 || m->num_attention_heads % m->num_key_value_heads != 0)
        return fail("CONFIG_ERROR", "num_attention_heads must be divisible by num_key_value_heads");
    if (m->norm_topk_prob)
        return fail("ROUTER_ERROR", "norm_topk_prob=true forbidden; unrenormalized routing invariant violated");
    if (!(m->rms_norm_eps > 0.0f) || std::isinf(m->rms_norm_eps))
        return fail("CONFIG_ERROR", "rms_norm_eps must be finite and > 0");
    if (m->full_attention_interval <= 0) return fail("CONFIG_ERROR", "full_attention_interval must be > 0");
    // shape limits of the sm_100a kernels
    if (!gemv_supported_k(m->hidden_size)) return fail("CONFIG_ERROR", "hidden_size must be 256, 512, 1024, 2048 or 4096");
    if (m->head_dim <= 0 || m->linear_key_head_dim <= 0) return fail("CONFIG_ERROR", "head dims must be > 0");
    if (!attn_supported(m->head_dim, m->num_attention_heads / m->num_key_value_heads))
        return fail("CONFIG_ERROR", "unsupported (head_dim, GQA group) for the decode attention kernel");
    if (!gemv_supported_k(m->num_attention_heads * m->head_dim))
        return fail("CONFIG_ERROR", "num_attention_heads * head_dim must be 256..4096 (power of two)");
    if (m->linear_key_head_dim != m->linear_value_head_dim ||
        (m->linear_key_head_dim != 64 && m->linear_key_head_dim != 128))
        return fail("CONFIG_ERROR", "GDN key/value head dims must be equal and 64 or 128");
    if (m->linear_num_key_heads <= 0 || m->linear_num_value_heads % m->linear_num_key_heads != 0)
        return fail("CONFIG_ERROR", "linear_num_value_heads must be a multiple of linear_num_key_heads");
    if (!gemv_supported_k(m->linear_num_value_heads * m->linear_value_head_dim))
        return fail("CONFIG_ERROR", "linear_num_value_heads * linear_value_head_dim must be 256..4096");
    if (m->linear_conv_kernel_dim != 4) return fail("CONFIG_ERROR", "linear_conv_kernel_dim must be 4");
    if (m->shared_expert_intermediate_size != m->moe_intermediate_size)
        return fail("CONFIG_ERROR", "shared_expert_intermediate_size must equal moe_intermediate_size");
    if (!moe_supported(m->hidden_size, m->moe_intermediate_size, m->quant_group_size))
        return fail("CONFIG_ERROR", "unsupported (hidden, moe_intermediate, group) for the 4-bit expert kernels");
    if (m->num_experts > 1023 || m->num_experts_per_tok > kMaxTopK)
        return fail("CONFIG_ERROR", "num_experts <= 1023 and num_experts_per_tok <= 16 required");
    const int rot = static_cast<int>(static_cast<float>(m->head_dim) * m->partial_rotary_factor);
    if (rot < 2 || rot > m->head_dim || (rot & 1)) return fail("CONFIG_ERROR", "invalid partial_rotary_factor");
    return DM_OK;
}

static Dims make_dims(const dm_model_config& m, const dm_runtime_config& r) {
    Dims d{};
    d.H = m.hidden_size;
    d.L = m.num_hidden_layers;
    d.interval = m.full_attention_interval;
    d.V = m.vocab_size;
    d.eps = m.rms_norm_eps;
    d.Hq = m.num_attention_heads;
    d.Hkv = m.num_key_value_heads;
    d.D = m.head_dim;
    d.rot_dim = static_cast<int>(static_cast<float>(m.head_dim) * m.partial_rotary_factor);
    d.theta = m.rope_theta;
    d.nk = m.linear_num_key_heads;
    d.nv = m.linear_num_value_heads;
    d.dk = m.linear_key_head_dim;
    d.dv = m.linear_value_head_dim;
    d.conv_k = m.linear_conv_kernel_dim;
    d.qkv_dim = 2 * d.nk * d.dk + d.nv * d.dv;
    d.z_dim = d.nv * d.dv;
    d.gdn_in_rows = d.qkv_dim + d.z_dim + 2 * d.nv;
    d.attn_in_rows = 2 * d.Hq * d.D + 2 * d.Hkv * d.D;
    d.E = m.num_experts;
    d.E_res = (r.expert_cache_slots > 0 && r.expert_cache_slots < m.num_experts) ? r.expert_cache_slots : m.num_experts;
    d.topk = m.num_experts_per_tok;
    d.I = m.moe_intermediate_size;
    d.G = m.quant_group_size;
    d.max_seqs = r.max_seqs;
    d.num_pages = r.kv_num_pages;
    d.max_pages = r.max_pages_per_seq;
    d.n_att = 0;
    for (int l = 0; l < d.L; ++l)
        if (l % d.interval == d.interval - 1) ++d.n_att;
    d.n_gdn = d.L - d.n_att;
    auto chunk = [&](int K) { return static_cast<int64_t>(16) * (K / 2 + 2 * (K / d.G) + K / d.G / 2); };
    d.gu_chunk_bytes = chunk(d.H);
    d.d_chunk_bytes = chunk(d.I);
    d.gu_chunks = d.I / 8;
    d.d_chunks = d.H / 16;
    d.expert_bytes = d.gu_chunks * d.gu_chunk_bytes + d.d_chunks * d.d_chunk_bytes;
    return d;
}

static inline bool is_attn_layer(const Dims& d, int l) { return l % d.interval == d.interval - 1; }

// Sub-allocator over the arena (256-byte alignment).
struct Plan {
    size_t off = 0;
    size_t take(size_t bytes) {
        size_t o = off;
        off += (bytes + 255) & ~static_cast<size_t>(255);
        return o;
    }
};

// The expert-parallel view of a context that is not part of a group: one rank, local buffers.
static void set_local_ep(dm_ctx* c);

static int plan_memory(dm_ctx* c, bool commit) {
    Dims& d = c->d;
    Plan p;
    const size_t H = d.H;
    std::vector<size_t> offs;
    auto T = [&](size_t bytes) {
        offs.push_back(p.take(bytes));
        return offs.back();
    };
    struct LayerOffs {
        size_t in_norm, post_norm, w_in, conv, dt, alog, gnorm, qn, kn, w_out, router, experts, shared;
    };
    std::vector<LayerOffs> lo(d.L);
    for (int l = 0; l < d.L; ++l) {
        LayerOffs& o = lo[l];
        o.in_norm = T(H * 2);
        o.post_norm = T(H * 2);
        if (is_attn_layer(d, l)) {
            o.w_in = T(static_cast<size_t>(d.attn_in_rows) * H * 2);
            o.qn = T(d.D * 2);
            o.kn = T(d.D * 2);
            o.w_out = T(H * d.Hq * d.D * 2);
        } else {
            o.w_in = T(static_cast<size_t>(d.gdn_in_rows) * H * 2);
            o.conv = T(static_cast<size_t>(d.qkv_dim) * 4 * 2);
            o.dt = T(d.nv * 4);
            o.alog = T(d.nv * 4);
            o.gnorm = T(d.dv * 2);
            o.w_out = T(H * d.z_dim * 2);
        }
        o.router = T(static_cast<size_t>(d.E + 1) * H * 2);
        o.experts = T(static_cast<size_t>(d.E_res) * d.expert_bytes);
        o.shared = T(static_cast<size_t>(d.expert_bytes));
    }
    const size_t o_embed = T(static_cast<size_t>(d.V) * H * 2);
    const size_t o_fnorm = T(H * 2);
    const size_t o_head = T(static_cast<size_t>(d.V) * H * 2);
    // a spilling pool: one staging record for uploads and the [L][E] slot table
    const bool spill = d.E_res < d.E;
    const size_t o_scr = spill ? T(static_cast<size_t>(d.expert_bytes)) : 0;
    const size_t o_slot = spill ? T(static_cast<size_t>(d.L) * d.E * 4) : 0;
    const size_t S = d.max_seqs;
    const size_t o_xres = T(S * H * 4), o_xmid = T(S * H * 4);
    const size_t o_ring = T(static_cast<size_t>(d.n_gdn) * S * kConvRing * d.qkv_dim * 4);
    const size_t o_S = T(static_cast<size_t>(d.n_gdn) * S * d.nv * d.dv * d.dk * 4);
    const size_t o_kv = T(static_cast<size_t>(d.n_att) * d.num_pages * 2 * d.Hkv * kPageTokens * d.D * 2);
    const size_t o_pt = T(S * d.max_pages * 4);
    const size_t o_pos = T(S * 4), o_tok = T(S * 4);
    const int gen_cap = 1 << 16;
    const size_t o_gen = T(gen_cap * 4), o_genidx = T(4), o_prompt = T(gen_cap * 4);
    const size_t o_z = T(d.z_dim * 4), o_ab = T(2 * d.nv * 4), o_o = T(d.z_dim * 4);
    const size_t o_qg = T(2 * d.Hq * d.D * 4), o_kvnew = T(2 * d.Hkv * d.D * 4);
    const size_t o_part = T(static_cast<size_t>(d.Hq) * kMaxSplits * (d.D + 2) * 4);
    const size_t o_aout = T(std::max(d.Hq * d.D, d.H) * 4);
    const size_t o_xn = T(H * 4), o_rl = T((d.E + 1) * 8), o_ids = T(kMaxTopK * 4), o_p = T(kMaxTopK * 4);
    const size_t o_sg = T(4), o_h = T(static_cast<size_t>(d.topk + 1) * d.I * 4), o_logits = T(static_cast<size_t>(d.V) * 4);
    const size_t o_cv = T(kMaxCtas * 4), o_ci = T(kMaxCtas * 4), o_cnt = T(64 * 4), o_err = T(4);
    const size_t o_trace = T(kTraceSlots * 8);
    const size_t o_ktrace = T(kMaxTraceKernels * 4 * 8);
    const size_t o_rope = T(static_cast<size_t>(d.max_pages) * kPageTokens * (d.rot_dim / 2) * 8);
    const size_t o_sq = T(static_cast<size_t>(d.I) * H / 2), o_ss = T(static_cast<size_t>(d.I) * H / d.G * 2),
                 o_sz = T(static_cast<size_t>(d.I) * H / d.G / 2 + 16);
    // batched decode scratch
    const size_t BC = static_cast<size_t>(std::min(d.max_seqs, kMaxBatch));
    const size_t kmax = std::max({static_cast<size_t>(d.H), static_cast<size_t>(d.z_dim), static_cast<size_t>(d.Hq) * d.D});
    const size_t nmax = std::max({static_cast<size_t>(d.gdn_in_rows), static_cast<size_t>(d.attn_in_rows),
                                  static_cast<size_t>(d.H), static_cast<size_t>(d.V)});
    // pairs one rank may compute: the routed choices of every row of a full group that land
    // on its experts, plus its own rows for the shared expert
    const size_t P = static_cast<size_t>(kMaxRanks) * BC * d.topk + BC;
    // segments: whole kSegTok runs, one tail per expert (two small-segment pieces at most)
    const int max_segs = static_cast<int>((P + kSegTok - 1) / kSegTok) + 2 * std::min(d.E + 1, static_cast<int>(P)) + 2;
    const int bgen_cap = 1 << 16;
    const size_t ob_slots = T(BC * 4), ob_tok = T(BC * 4), ob_x = T(BC * H * 4), ob_xm = T(BC * H * 4);
    // GEMM operand rows rounded up to 16 (the tensor map's box never leaves the buffer)
    const size_t xrows = (2 * BC + 15) / 16 * 16;
    const size_t ob_xcat = T(xrows * kmax * 2), ob_c = T(2 * BC * nmax * 4);
    const size_t ob_z = T(BC * d.z_dim * 4), ob_ab = T(BC * 2 * d.nv * 4), ob_o = T(BC * d.z_dim * 4);
    const size_t ob_qg = T(BC * 2 * d.Hq * d.D * 4), ob_kvn = T(BC * 2 * d.Hkv * d.D * 4);
    const size_t ob_part = T(BC * d.Hq * kMaxSplits * (d.D + 2) * 4), ob_aout = T(BC * d.Hq * d.D * 4);
    const size_t ob_acnt = T(BC * d.Hkv * 4), ob_xn = T(BC * H * 4), ob_lg = T(BC * (d.E + 1) * 4);
    const size_t ob_ids = T(BC * d.topk * 4), ob_pr = T(BC * d.topk * 4), ob_sg = T(BC * 4);
    const size_t ob_segs = T(static_cast<size_t>(max_segs) * 16), ob_work = T(16), ob_stats = T(16);
    const size_t ob_rcnt = T((BC + 1) * 4);  // one counter per router row block (down to one row)
    // staged expert operands: 2 rows (hi, lo) per pair, every segment padded to 16 rows
    const size_t max_cols = 2 * P + 16 * static_cast<size_t>(max_segs);
    const size_t ob_psrc = T(P * 4), ob_eout = T(BC * (d.topk + 1) * H * 4);
    const size_t ob_xgu = T(max_cols * H * 2), ob_xdn = T(max_cols * d.I * 2);
    const size_t ob_xrec = T(P * q4_vrec_bytes(d.H)), ob_hrec = T(P * q4_vrec_bytes(d.I));
    const size_t ob_flags = T(2 * kMaxRanks * 4), ob_epoch = T(2 * 4);
    const size_t ob_cv = T(BC * kHeadChunks * 4), ob_ci = T(BC * kHeadChunks * 4), ob_hl = T(BC * d.V * 4);
    const size_t ob_gen = T(static_cast<size_t>(bgen_cap) * 4), ob_genidx = T(4);
    const size_t o_rbias = T(static_cast<size_t>(d.L) * d.E * 4);
    // prefill chunk scratch: PR rows (prompt tokens of one sequence), no more than the
    // grouping kernel takes or the context can hold
    const size_t PR = static_cast<size_t>(std::min({kPfMaxRows, b_group_max_rows(d.E),
                                                    (d.max_pages * kPageTokens + 15) / 16 * 16}));
    const size_t nmax_dense = std::max({static_cast<size_t>(d.gdn_in_rows), static_cast<size_t>(d.attn_in_rows),
                                        static_cast<size_t>(d.H)});
    const size_t PP = PR * d.topk + PR;
    const int pmax_segs = static_cast<int>((PP + kSegTok - 1) / kSegTok) + 2 * std::min(d.E + 1, static_cast<int>(PP)) + 2;
    const size_t pmax_cols = 2 * PP + 16 * static_cast<size_t>(pmax_segs);
    const size_t pc_cap = std::max(2 * PR * nmax_dense, 2 * static_cast<size_t>(d.V));  // the head: one row
    const size_t op_slots = T(PR * 4), op_tok = T(PR * 4), op_x = T(PR * H * 4), op_xm = T(PR * H * 4);
    const size_t op_xcat = T((2 * PR + 15) / 16 * 16 * kmax * 2), op_c = T(pc_cap * 4);
    const size_t op_z = T(PR * d.z_dim * 4), op_ab = T(PR * 2 * d.nv * 4), op_o = T(PR * d.z_dim * 4);
    const size_t op_qg = T(PR * 2 * d.Hq * d.D * 4), op_kvn = T(PR * 2 * d.Hkv * d.D * 4);
    const size_t op_part = T(PR * d.Hq * kPfMaxSplits * (d.D + 2) * 4);
    const size_t op_xn = T(PR * H * 4), op_lg = T(PR * (d.E + 1) * 4);
    const size_t op_ids = T(PR * d.topk * 4), op_pr = T(PR * d.topk * 4), op_sg = T(PR * 4);
    const size_t op_segs = T(static_cast<size_t>(pmax_segs) * 16), op_work = T(16), op_stats = T(16);
    const size_t op_rcnt = T((PR + 1) * 4), op_psrc = T(PP * 4), op_eout = T(PR * (d.topk + 1) * H * 4);
    const size_t op_xgu = T(pmax_cols * H * 2), op_xdn = T(pmax_cols * d.I * 2);
    const size_t op_xrec = T(PP * q4_vrec_bytes(d.H)), op_hrec = T(PP * q4_vrec_bytes(d.I));
    const size_t op_cv = T(kHeadChunks * 4), op_ci = T(kHeadChunks * 4), op_hl = T(static_cast<size_t>(d.V) * 4);
    const size_t op_gen = T(16), op_genidx = T(4);
    const size_t op_u = T(PR * d.qkv_dim * 4);
    const size_t op_raw = T(PR * d.qkv_dim * 4), op_qhi = T(PR * d.Hq * d.D * 2), op_qlo = T(PR * d.Hq * d.D * 2);
    c->arena_bytes = p.off;
    if (!commit) return DM_OK;

    uint8_t* A = c->arena;
    c->layers.assign(d.L, LayerW{});
    int gi = 0, ai = 0;
    for (int l = 0; l < d.L; ++l) {
        LayerW& w = c->layers[l];
        const LayerOffs& o = lo[l];
        w.is_attn = is_attn_layer(d, l);
        w.sub = w.is_attn ? ai++ : gi++;
        w.in_norm = reinterpret_cast<uint16_t*>(A + o.in_norm);
        w.post_norm = reinterpret_cast<uint16_t*>(A + o.post_norm);
        w.w_in = reinterpret_cast<uint16_t*>(A + o.w_in);
        w.w_out = reinterpret_cast<uint16_t*>(A + o.w_out);
        if (w.is_attn) {
            w.q_norm = reinterpret_cast<uint16_t*>(A + o.qn);
            w.k_norm = reinterpret_cast<uint16_t*>(A + o.kn);
        } else {
            w.conv_w = reinterpret_cast<uint16_t*>(A + o.conv);
            w.dt_bias = reinterpret_cast<float*>(A + o.dt);
            w.a_log = reinterpret_cast<float*>(A + o.alog);
            w.gdn_norm = reinterpret_cast<uint16_t*>(A + o.gnorm);
        }
        w.w_router = reinterpret_cast<uint16_t*>(A + o.router);
        w.experts = A + o.experts;
        w.shared = A + o.shared;
    }
    c->embed = reinterpret_cast<uint16_t*>(A + o_embed);
    c->scratch_rec = spill ? A + o_scr : nullptr;
    c->d_slot_of = spill ? reinterpret_cast<int*>(A + o_slot) : nullptr;
    c->final_norm = reinterpret_cast<uint16_t*>(A + o_fnorm);
    c->lm_head = reinterpret_cast<uint16_t*>(A + o_head);
    Buffers& b = c->b;
    b.xres = reinterpret_cast<float*>(A + o_xres);
    b.xmid = reinterpret_cast<float*>(A + o_xmid);
    b.ring = reinterpret_cast<float*>(A + o_ring);
    b.S = reinterpret_cast<float*>(A + o_S);
    b.kv = reinterpret_cast<uint16_t*>(A + o_kv);
    b.page_table = reinterpret_cast<int*>(A + o_pt);
    b.pos = reinterpret_cast<int*>(A + o_pos);
    b.token = reinterpret_cast<int*>(A + o_tok);
    b.gen_out = reinterpret_cast<int*>(A + o_gen);
    b.gen_idx = reinterpret_cast<int*>(A + o_genidx);
    b.gen_capacity = gen_cap;
    b.prompt = reinterpret_cast<int*>(A + o_prompt);
    b.z = reinterpret_cast<float*>(A + o_z);
    b.ab = reinterpret_cast<float*>(A + o_ab);
    b.o = reinterpret_cast<float*>(A + o_o);
    b.qg = reinterpret_cast<float*>(A + o_qg);
    b.kvnew = reinterpret_cast<float*>(A + o_kvnew);
    b.attn_part = reinterpret_cast<float*>(A + o_part);
    b.attn_out = reinterpret_cast<float*>(A + o_aout);
    b.xn = reinterpret_cast<float*>(A + o_xn);
    b.rslots = reinterpret_cast<unsigned long long*>(A + o_rl);
    b.topk_ids = reinterpret_cast<int*>(A + o_ids);
    b.topk_p = reinterpret_cast<float*>(A + o_p);
    b.shared_g = reinterpret_cast<float*>(A + o_sg);
    b.h = reinterpret_cast<float*>(A + o_h);
    b.logits = reinterpret_cast<float*>(A + o_logits);
    b.cand_val = reinterpret_cast<float*>(A + o_cv);
    b.cand_idx = reinterpret_cast<int*>(A + o_ci);
    b.counters = reinterpret_cast<unsigned*>(A + o_cnt);
    b.err = reinterpret_cast<uint32_t*>(A + o_err);
    b.rope = reinterpret_cast<float2*>(A + o_rope);
    b.trace = nullptr;  // off until dm_trace_enable
    c->trace_buf = reinterpret_cast<uint64_t*>(A + o_trace);
    c->ktrace_buf = reinterpret_cast<uint64_t*>(A + o_ktrace);
    b.ktrace = nullptr;
    c->stage_q = A + o_sq;
    c->stage_s = reinterpret_cast<uint16_t*>(A + o_ss);
    c->stage_z = A + o_sz;
    BatchBuffers& bb = c->bb;
    bb.cap = static_cast<int>(BC);
    bb.max_segs = max_segs;
    bb.slots = reinterpret_cast<int*>(A + ob_slots);
    bb.tok = reinterpret_cast<int*>(A + ob_tok);
    bb.x = reinterpret_cast<float*>(A + ob_x);
    bb.xm = reinterpret_cast<float*>(A + ob_xm);
    bb.xcat = reinterpret_cast<uint16_t*>(A + ob_xcat);
    bb.c = reinterpret_cast<float*>(A + ob_c);
    bb.z = reinterpret_cast<float*>(A + ob_z);
    bb.ab = reinterpret_cast<float*>(A + ob_ab);
    bb.o = reinterpret_cast<float*>(A + ob_o);
    bb.qg = reinterpret_cast<float*>(A + ob_qg);
    bb.kvnew = reinterpret_cast<float*>(A + ob_kvn);
    bb.attn_part = reinterpret_cast<float*>(A + ob_part);
    bb.attn_out = reinterpret_cast<float*>(A + ob_aout);
    bb.attn_cnt = reinterpret_cast<unsigned*>(A + ob_acnt);
    bb.xn = reinterpret_cast<float*>(A + ob_xn);
    bb.logits = reinterpret_cast<float*>(A + ob_lg);
    bb.ids = reinterpret_cast<int*>(A + ob_ids);
    bb.probs = reinterpret_cast<float*>(A + ob_pr);
    bb.sg = reinterpret_cast<float*>(A + ob_sg);
    bb.segs = reinterpret_cast<int4*>(A + ob_segs);
    bb.work = reinterpret_cast<int*>(A + ob_work);
    bb.stats = reinterpret_cast<unsigned*>(A + ob_stats);
    bb.rcnt = reinterpret_cast<unsigned*>(A + ob_rcnt);
    bb.err = b.err;
    bb.pair_src = reinterpret_cast<int*>(A + ob_psrc);
    bb.max_pairs = static_cast<int>(P);
    bb.ep_flags = reinterpret_cast<unsigned*>(A + ob_flags);
    bb.ep_epoch = reinterpret_cast<unsigned*>(A + ob_epoch);
    bb.max_cols = static_cast<int>(max_cols);
    bb.xgu = A + ob_xgu;
    bb.xdn = A + ob_xdn;
    bb.xrec = A + ob_xrec;
    bb.hrec = A + ob_hrec;
    bb.eout = reinterpret_cast<float*>(A + ob_eout);
    bb.cand_val = reinterpret_cast<float*>(A + ob_cv);
    bb.cand_idx = reinterpret_cast<int*>(A + ob_ci);
    bb.head_logits = reinterpret_cast<float*>(A + ob_hl);
    bb.gen_out = reinterpret_cast<int*>(A + ob_gen);
    bb.gen_idx = reinterpret_cast<int*>(A + ob_genidx);
    bb.gen_cap = bgen_cap;
    bb.c_cap = 2 * BC * nmax;
    BatchBuffers& pb = c->pb;
    pb.cap = static_cast<int>(PR);
    pb.max_segs = pmax_segs;
    pb.max_pairs = static_cast<int>(PP);
    pb.max_cols = static_cast<int>(pmax_cols);
    pb.c_cap = pc_cap;
    pb.slots = reinterpret_cast<int*>(A + op_slots);
    pb.tok = reinterpret_cast<int*>(A + op_tok);
    pb.x = reinterpret_cast<float*>(A + op_x);
    pb.xm = reinterpret_cast<float*>(A + op_xm);
    pb.xcat = reinterpret_cast<uint16_t*>(A + op_xcat);
    pb.c = reinterpret_cast<float*>(A + op_c);
    pb.z = reinterpret_cast<float*>(A + op_z);
    pb.ab = reinterpret_cast<float*>(A + op_ab);
    pb.o = reinterpret_cast<float*>(A + op_o);
    pb.qg = reinterpret_cast<float*>(A + op_qg);
    pb.kvnew = reinterpret_cast<float*>(A + op_kvn);
    pb.attn_part = reinterpret_cast<float*>(A + op_part);
    pb.attn_out = nullptr;
    pb.attn_cnt = nullptr;
    pb.xn = reinterpret_cast<float*>(A + op_xn);
    pb.logits = reinterpret_cast<float*>(A + op_lg);
    pb.ids = reinterpret_cast<int*>(A + op_ids);
    pb.probs = reinterpret_cast<float*>(A + op_pr);
    pb.sg = reinterpret_cast<float*>(A + op_sg);
    pb.segs = reinterpret_cast<int4*>(A + op_segs);
    pb.work = reinterpret_cast<int*>(A + op_work);
    pb.stats = reinterpret_cast<unsigned*>(A + op_stats);
    pb.rcnt = reinterpret_cast<unsigned*>(A + op_rcnt);
    pb.err = b.err;
    pb.pair_src = reinterpret_cast<int*>(A + op_psrc);
    pb.ep_flags = bb.ep_flags;
    pb.ep_epoch = bb.ep_epoch;
    pb.xgu = A + op_xgu;
    pb.xdn = A + op_xdn;
    pb.xrec = A + op_xrec;
    pb.hrec = A + op_hrec;
    pb.eout = reinterpret_cast<float*>(A + op_eout);
    pb.cand_val = reinterpret_cast<float*>(A + op_cv);
    pb.cand_idx = reinterpret_cast<int*>(A + op_ci);
    pb.head_logits = reinterpret_cast<float*>(A + op_hl);
    pb.gen_out = reinterpret_cast<int*>(A + op_gen);
    pb.gen_idx = reinterpret_cast<int*>(A + op_genidx);
    pb.gen_cap = 0;
    pb.pf_raw = reinterpret_cast<float*>(A + op_raw);
    pb.pf_u = reinterpret_cast<float*>(A + op_u);
    pb.pf_qhi = reinterpret_cast<uint16_t*>(A + op_qhi);
    pb.pf_qlo = reinterpret_cast<uint16_t*>(A + op_qlo);
    set_local_ep(c);
    c->rbias = reinterpret_cast<float*>(A + o_rbias);
    return DM_OK;
}

static LaunchCfg lcfg(const dm_ctx* c) {
    return LaunchCfg{c->stream, c->num_sms, true, nullptr};
}

// Launch config for the next kernel of a traced sequence (timeline record n of kind k).
static LaunchCfg lcfg_traced(dm_ctx* c, int kind, int layer) {
    LaunchCfg lc = lcfg(c);
    if (c->b.ktrace && c->trace_n < kMaxTraceKernels) {
        lc.kt = c->b.ktrace + 4 * c->trace_n;
        c->trace_kinds.push_back((kind << 16) | (layer & 0xFFFF));
        ++c->trace_n;
    }
    return lc;
}

// Reads and clears the device error word; maps it to a status.
static int check_device_error(dm_ctx* c, const char* stage) {
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", stage, -1, "%s", cudaGetErrorString(e));
    uint32_t w = 0;
    e = cudaMemcpy(&w, c->b.err, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", stage, -1, "%s", cudaGetErrorString(e));
    if (w == 0) return DM_OK;
    cudaMemset(c->b.err, 0, 4);
    // a launch that gave up waiting may have left router logit words of its generation
    cudaMemset(c->b.rslots, 0, static_cast<size_t>(c->d.E + 1) * 8);
    if (w & DM_DEVERR_TIMEOUT) return set_err(c, DM_ERR_TIMEOUT, "DEVICE_TIMEOUT", stage, -1, "a bounded device wait ran out (word 0x%x)", w);
    if (w & DM_DEVERR_CAPACITY) return set_err(c, DM_ERR_CAPACITY, "M5_ERR_CONTEXT_SIZE", stage, -1, "KV cache capacity exceeded on token append");
    if (w & DM_DEVERR_PAGE) return set_err(c, DM_ERR_CAPACITY, "KV_PAGE_ERROR", stage, -1, "page table entry outside the page pool");
    if (w & DM_DEVERR_TOKEN) return set_err(c, DM_ERR_INVALID_ARG, "M4_ERR_INPUT", stage, -1, "token id out of range [0, vocab)");
    if (w & DM_DEVERR_RANGE)
        return set_err(c, DM_ERR_NONFINITE, "NONFINITE_ERROR", stage, -1,
                       "a batched expert activation exceeded the fp16 operand range (|x| > 65504)");
    return set_err(c, DM_ERR_NONFINITE, "NONFINITE_ERROR", stage, -1, "non-finite value detected (word 0x%x)", w);
}

template <typename F>
static void host_parallel(uint64_t n, F&& f) {
    unsigned nt = std::thread::hardware_concurrency();
    if (nt == 0) nt = 1;
    if (nt > 64) nt = 64;
    if (n < (1u << 16)) nt = 1;
    std::vector<std::thread> th;
    for (unsigned t = 0; t < nt; ++t) {
        const uint64_t a = n * t / nt, b = n * (t + 1) / nt;
        th.emplace_back([=, &f] { f(a, b); });
    }
    for (auto& x : th) x.join();
}

static void set_local_ep(dm_ctx* c) {
    BatchBuffers& bb = c->bb;
    EpView v{};
    v.rank = 0;
    v.world = 1;
    v.ids[0] = bb.ids;
    v.xn[0] = bb.xn;
    v.eout[0] = bb.eout;
    v.flags[0] = bb.ep_flags;
    bb.ep = v;
    BatchBuffers& pb = c->pb;  // prefill: always this rank alone
    EpView pv{};
    pv.rank = 0;
    pv.world = 1;
    pv.ids[0] = pb.ids;
    pv.xn[0] = pb.xn;
    pv.eout[0] = pb.eout;
    pv.flags[0] = pb.ep_flags;
    pb.ep = pv;
}

// Tensor map of the KV arena for the attention kernel's page copies: rows of D bf16
// ([att][page][K|V][Hkv][16] flattened), boxes of 16 rows x 64 columns (128 bytes, the
// swizzle span), 128-byte swizzle.  The encoder comes from the driver entry point table.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeTiledFn encode_fn() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn ||
        q != cudaDriverEntryPointSuccess) {
        fprintf(stderr, "dm_ctx_create: cuTensorMapEncodeTiled unavailable\n");
        return nullptr;
    }
    return reinterpret_cast<EncodeTiledFn>(fn);
}

// Tensor maps of every layer's expert pool for the batched expert kernels: the nibble rows
// of one projection as a 4-D byte tensor (row bytes, 16 rows of a chunk, chunks of a record,
// records; the shared expert's record follows the E routed ones), boxes of 16 rows x 128
// bytes (the swizzle span), 128-byte swizzle.  A layer whose shared record does not follow
// its pool keeps null maps (the kernels then use plain loads).
static bool encode_expert_maps(dm_ctx* c) {
    const Dims& d = c->d;
    c->xmaps.assign(static_cast<size_t>(d.L) * 2, CUtensorMap{});
    const bool gu_ok = expert_tc_supported(d.H), dn_ok = expert_tc_supported(d.I);
    if (!gu_ok && !dn_ok) return true;
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    for (int l = 0; l < d.L; ++l) {
        LayerW& w = c->layers[l];
        w.tm_gu = w.tm_dn = nullptr;
        if (w.shared != w.experts + static_cast<int64_t>(d.E_res) * d.expert_bytes) continue;
        for (int proj = 0; proj < 2; ++proj) {
            if (proj == 0 ? !gu_ok : !dn_ok) continue;
            const int K = proj == 0 ? d.H : d.I;
            const int64_t chunk = proj == 0 ? d.gu_chunk_bytes : d.d_chunk_bytes;
            const int nch = proj == 0 ? d.gu_chunks : d.d_chunks;
            uint8_t* base = const_cast<uint8_t*>(w.experts) + (proj == 0 ? 0 : static_cast<int64_t>(d.gu_chunks) * d.gu_chunk_bytes);
            const cuuint64_t dims[4] = {static_cast<cuuint64_t>(K / 2), 16, static_cast<cuuint64_t>(nch),
                                        static_cast<cuuint64_t>(d.E_res + 1)};
            const cuuint64_t strides[3] = {static_cast<cuuint64_t>(K / 2), static_cast<cuuint64_t>(chunk),
                                           static_cast<cuuint64_t>(d.expert_bytes)};
            // boxes of 16 rows x 128 bytes (256 columns) with the 128-byte swizzle; a 128-column
            // projection is one unswizzled box of 16 rows x 64 bytes
            const bool wide = K >= 256;
            const cuuint32_t box[4] = {wide ? 128u : 64u, 16, 1, 1};
            const cuuint32_t estr[4] = {1, 1, 1, 1};
            CUtensorMap* m = &c->xmaps[static_cast<size_t>(l) * 2 + proj];
            const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, base, dims, strides, box, estr,
                                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                                   wide ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
            if (r != CUDA_SUCCESS) {
                fprintf(stderr, "dm_ctx_create: expert tensor map of layer %d failed (%d)\n", l, static_cast<int>(r));
                return false;
            }
            (proj == 0 ? w.tm_gu : w.tm_dn) = m;
        }
    }
    return true;
}

// Tensor maps of every dense weight matrix for the batched step's tensor-core GEMMs: bf16
// rows of K elements, boxes of 128 rows x 64 columns (128 bytes) with the 128-byte swizzle.
static bool encode_dense_maps(dm_ctx* c) {
    const Dims& d = c->d;
    c->dmaps.assign(static_cast<size_t>(d.L) * 2 + 1, CUtensorMap{});
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    auto one = [&](CUtensorMap* m, const uint16_t* w, int N, int K) {
        const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(N)};
        const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
        const cuuint32_t box[2] = {64, 128};
        const cuuint32_t estr[2] = {1, 1};
        return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(w), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    for (int l = 0; l < d.L; ++l) {
        const LayerW& w = c->layers[l];
        const int nin = w.is_attn ? d.attn_in_rows : d.gdn_in_rows;
        const int kout = w.is_attn ? d.Hq * d.D : d.z_dim;
        if (!one(&c->dmaps[2 * l], w.w_in, nin, d.H) || !one(&c->dmaps[2 * l + 1], w.w_out, d.H, kout)) return false;
    }
    return one(&c->dmaps[2 * d.L], c->lm_head, d.V, d.H);
}

// The batched step's GEMM operand rows (xcat: 2n rows of K bf16, packed with row stride K by
// the prep and merge kernels) as a tensor map with boxes of ntile rows x 64 columns.
static bool encode_operand_map(const BatchBuffers& bb, int K, int ncols, CUtensorMap* m) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const int rows = (2 * bb.cap + 15) / 16 * 16;  // the buffer holds rows x kmax >= rows x K elements
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    // one column tile of at most 128 rows (the GEMM loads tile ct at row 128 ct)
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(ncols > 128 ? 128 : (ncols + 15) / 16 * 16)};
    const cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, bb.xcat, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool encode_kv_map(dm_ctx* c) {
    c->b.kv_tmap = &c->kv_map;
    const Dims& d = c->d;
    if (d.n_att == 0) return true;
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const uint64_t rows = static_cast<uint64_t>(d.n_att) * d.num_pages * 2 * d.Hkv * kPageTokens;
    if (rows >= (1ull << 31)) {
        fprintf(stderr, "dm_ctx_create: KV arena of %llu rows exceeds the 2^31 tensor-map coordinate range\n",
                static_cast<unsigned long long>(rows));
        return false;
    }
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(d.D), rows};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(d.D) * 2};
    const cuuint32_t box[2] = {64, kPageTokens};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = fn(&c->kv_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, c->b.kv, dims, strides,
                                                      box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        fprintf(stderr, "dm_ctx_create: cuTensorMapEncodeTiled failed (%d)\n", static_cast<int>(r));
        return false;
    }
    return true;
}

// ------------------------------------------------------------------------------------
extern "C" {

int32_t dm_abi_version(void) { return DM_ABI_VERSION; }

int32_t dm_config_validate(const dm_model_config* model, char* buf, uint64_t buf_size) {
    if (buf && buf_size) buf[0] = 0;
    return validate_config(model, buf, buf_size);
}

int32_t dm_last_error(const dm_ctx* ctx, char* buf, uint64_t buf_size) {
    if (!ctx || !buf || buf_size == 0) return DM_ERR_INVALID_ARG;
    snprintf(buf, buf_size, "%s", ctx->last_error.c_str());
    return DM_OK;
}

int32_t dm_ctx_create(const dm_model_config* model, const dm_runtime_config* rt, int32_t device,
                      dm_ctx** out_ctx) {
    if (!out_ctx || !rt) return DM_ERR_INVALID_ARG;
    *out_ctx = nullptr;
    char msg[512];
    int rc = validate_config(model, msg, sizeof msg);
    if (rc != DM_OK) {
        fprintf(stderr, "%s\n", msg);
        return rc;
    }
    if (rt->max_seqs <= 0 || rt->kv_page_tokens != kPageTokens || rt->kv_num_pages <= 0 || rt->max_pages_per_seq <= 0)
        return DM_ERR_INVALID_ARG;
    if (rt->expert_cache_slots < 0 ||
        (rt->expert_cache_slots > 0 && rt->expert_cache_slots < model->num_experts_per_tok)) {
        fprintf(stderr, "dm_ctx_create: expert_cache_slots must be 0 or at least num_experts_per_tok\n");
        return DM_ERR_INVALID_ARG;
    }
    dm_ctx* c = new dm_ctx();
    c->mc = *model;
    c->rc = *rt;
    c->d = make_dims(*model, *rt);
    c->device = device;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = gemv_set_attrs();
    if (e == cudaSuccess) e = moe_set_attrs();
    if (e == cudaSuccess) e = gdn_set_attrs();
    if (e == cudaSuccess) e = router_set_attrs();
    // function attributes are per process: always the kernel's fixed maximum, never a
    // per-context value that a later, smaller context would lower
    if (e == cudaSuccess) e = attn_set_attrs(kAttnMaxScoreSmem);
    if (e == cudaSuccess) e = batch_set_attrs();
    if (e == cudaSuccess) e = pf_attn_set_attrs();
    if (e == cudaSuccess) e = tc_gemm_set_attrs();
    bool moe_fits = false;
    if (e == cudaSuccess) e = moe_fused_fits(c->d, c->num_sms, &moe_fits);
    if (e == cudaSuccess) c->gdn_fused = gdn_fused_fits(c->d, c->num_sms);
    if (e != cudaSuccess) {
        fprintf(stderr, "dm_ctx_create: %s\n", cudaGetErrorString(e));
        delete c;
        return DM_ERR_CUDA;
    }
    if (!moe_fits) {
        fprintf(stderr, "dm_ctx_create: the fused MoE kernel for hidden %d / intermediate %d cannot keep one CTA "
                "resident on each of the %d SMs\n", c->d.H, c->d.I, c->num_sms);
        delete c;
        return DM_ERR_INVALID_ARG;
    }
    plan_memory(c, false);
    e = cudaMalloc(&c->arena, c->arena_bytes);
    if (e != cudaSuccess) {
        fprintf(stderr, "dm_ctx_create: cudaMalloc(%zu): %s\n", c->arena_bytes, cudaGetErrorString(e));
        cudaStreamDestroy(c->stream);
        delete c;
        return DM_ERR_OOM;
    }
    plan_memory(c, true);
    // zero everything (weights stay zero until uploaded; state starts empty)
    e = cudaMemsetAsync(c->arena, 0, c->arena_bytes, c->stream);
    if (e == cudaSuccess)
        e = launch_rope_table(c->stream, c->b.rope, c->d.max_pages * kPageTokens, c->d.rot_dim, c->d.theta);
    if (e == cudaSuccess) e = cudaMallocHost(&c->h_io, 64);
    if (e == cudaSuccess) e = cudaMallocHost(&c->h_bio, 4 * kMaxBatch * sizeof(int));
    if (e == cudaSuccess && c->d.E_res < c->d.E) {  // the spilling pool's host side
        const Dims& d = c->d;
        e = cudaHostAlloc(reinterpret_cast<void**>(&c->host_pool), static_cast<size_t>(d.L) * d.E * d.expert_bytes,
                          cudaHostAllocDefault);
        if (e == cudaSuccess) e = cudaMallocHost(&c->h_slot_of, static_cast<size_t>(d.L) * d.E * 4);
        if (e == cudaSuccess) e = cudaMallocHost(&c->h_sids, static_cast<size_t>(kMaxBatch) * d.topk * 4);
        if (e == cudaSuccess) e = cudaMemsetAsync(c->d_slot_of, 0xFF, static_cast<size_t>(d.L) * d.E * 4, c->stream);
        if (e == cudaSuccess) {
            memset(c->host_pool, 0, static_cast<size_t>(d.L) * d.E * d.expert_bytes);
            c->spill.init(d.L, d.E, d.E_res);
        }
    }
    if (e == cudaSuccess && !encode_kv_map(c)) e = cudaErrorInvalidValue;
    if (e == cudaSuccess && !encode_expert_maps(c)) e = cudaErrorInvalidValue;
    if (e == cudaSuccess && !encode_dense_maps(c)) e = cudaErrorInvalidValue;
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) {
        fprintf(stderr, "dm_ctx_create: %s\n", cudaGetErrorString(e));
        if (c->h_io) cudaFreeHost(c->h_io);
        if (c->h_bio) cudaFreeHost(c->h_bio);
        if (c->host_pool) cudaFreeHost(c->host_pool);
        if (c->h_slot_of) cudaFreeHost(c->h_slot_of);
        if (c->h_sids) cudaFreeHost(c->h_sids);
        cudaFree(c->arena);
        delete c;
        return DM_ERR_CUDA;
    }
    c->bgraphs.assign(2 * (c->bb.cap + 1), nullptr);
    c->have_dense.assign(static_cast<size_t>(c->d.L + 1) * DM_T_COUNT, 0);
    c->have_expert.assign(static_cast<size_t>(c->d.L) * (c->d.E + 1) * 3, 0);
    c->slot_len.assign(c->d.max_seqs, 0);
    c->att_len.assign(static_cast<size_t>(c->d.n_att) * c->d.max_seqs, 0);
    c->dev_pos_valid.assign(c->d.max_seqs, 0);
    c->graphs.assign(c->d.max_seqs, nullptr);
    for (int s = 0; s < c->d.max_seqs; ++s) {
        int r2 = dm_seq_reset(c, s);
        if (r2 != DM_OK) {
            fprintf(stderr, "dm_ctx_create: %s\n", c->last_error.c_str());
            dm_ctx_destroy(c);
            return r2;
        }
    }
    *out_ctx = c;
    return DM_OK;
}

int32_t dm_ctx_destroy(dm_ctx* c) {
    if (!c) return DM_ERR_INVALID_ARG;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (auto& g : c->graphs)
        if (g) cudaGraphExecDestroy(g);
    for (auto& g : c->bgraphs)
        if (g) cudaGraphExecDestroy(g);
    for (uint8_t* pa : c->peer_arena)
        if (pa) cudaIpcCloseMemHandle(pa);
    if (c->h_bio) cudaFreeHost(c->h_bio);
    if (c->arena) cudaFree(c->arena);
    if (c->flush_buf) cudaFree(c->flush_buf);
    if (c->h_io) cudaFreeHost(c->h_io);
    if (c->ld_host) cudaFreeHost(c->ld_host);
    if (c->ld_dev) cudaFree(c->ld_dev);
    if (c->host_pool) cudaFreeHost(c->host_pool);
    if (c->h_slot_of) cudaFreeHost(c->h_slot_of);
    if (c->h_sids) cudaFreeHost(c->h_sids);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    return DM_OK;
}

int32_t dm_ctx_device_bytes(const dm_ctx* c, uint64_t* out) {
    if (!c || !out) return DM_ERR_INVALID_ARG;
    *out = c->arena_bytes;
    return DM_OK;
}

int32_t dm_get_stream(dm_ctx* c, void** s) {
    if (!c || !s) return DM_ERR_INVALID_ARG;
    *s = c->stream;
    return DM_OK;
}

static bool gdn_fused_on(const dm_ctx* c) { return c->gdn_fused; }

int32_t dm_kernels_per_step(dm_ctx* c, int32_t* out) {
    if (!c || !out) return DM_ERR_INVALID_ARG;
    // embed; per block the mixer kernels (attention 3; GDN 2 fused or 3) + 1 MoE kernel; head
    const int gdn_k = gdn_fused_on(c) ? 2 : 3;
    *out = 1 + c->d.n_att * 4 + c->d.n_gdn * (gdn_k + 1) + 1;
    return DM_OK;
}

// ---- weights ------------------------------------------------------------------------
static int tensor_target(dm_ctx* c, int layer, int id, int dtype, uint64_t n, void** dst, size_t* bytes) {
    const Dims& d = c->d;
    const size_t H = d.H;
    auto want = [&](uint64_t expect, int dt, void* p) {
        if (n != expect) return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer,
                                        "tensor %d: expected %llu elements, got %llu", id,
                                        (unsigned long long)expect, (unsigned long long)n);
        if (dtype != dt) return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer,
                                        "tensor %d: wrong dtype", id);
        *dst = p;
        *bytes = expect * (dt == DM_DTYPE_F32 ? 4 : 2);
        return DM_OK;
    };
    if (layer == -1) {
        switch (id) {
            case DM_T_EMBED: return want(static_cast<uint64_t>(d.V) * H, DM_DTYPE_BF16, c->embed);
            case DM_T_FINAL_NORM: return want(H, DM_DTYPE_BF16, c->final_norm);
            case DM_T_LM_HEAD: return want(static_cast<uint64_t>(d.V) * H, DM_DTYPE_BF16, c->lm_head);
            default: return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer, "tensor %d is per-layer", id);
        }
    }
    if (layer < 0 || layer >= d.L) return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer, "layer out of range");
    LayerW& w = c->layers[layer];
    uint16_t* win = const_cast<uint16_t*>(w.w_in);
    switch (id) {
        case DM_T_INPUT_NORM: return want(H, DM_DTYPE_BF16, const_cast<uint16_t*>(w.in_norm));
        case DM_T_POST_NORM: return want(H, DM_DTYPE_BF16, const_cast<uint16_t*>(w.post_norm));
        case DM_T_ROUTER: return want(static_cast<uint64_t>(d.E) * H, DM_DTYPE_BF16, const_cast<uint16_t*>(w.w_router));
        case DM_T_SHARED_GATE: return want(H, DM_DTYPE_BF16, const_cast<uint16_t*>(w.w_router) + static_cast<size_t>(d.E) * H);
        default: break;
    }
    if (w.is_attn) {
        switch (id) {
            case DM_T_ATTN_Q: return want(static_cast<uint64_t>(2) * d.Hq * d.D * H, DM_DTYPE_BF16, win);
            case DM_T_ATTN_K: return want(static_cast<uint64_t>(d.Hkv) * d.D * H, DM_DTYPE_BF16, win + static_cast<size_t>(2) * d.Hq * d.D * H);
            case DM_T_ATTN_V: return want(static_cast<uint64_t>(d.Hkv) * d.D * H, DM_DTYPE_BF16, win + static_cast<size_t>(2 * d.Hq * d.D + d.Hkv * d.D) * H);
            case DM_T_ATTN_Q_NORM: return want(d.D, DM_DTYPE_BF16, const_cast<uint16_t*>(w.q_norm));
            case DM_T_ATTN_K_NORM: return want(d.D, DM_DTYPE_BF16, const_cast<uint16_t*>(w.k_norm));
            case DM_T_ATTN_O: return want(H * d.Hq * d.D, DM_DTYPE_BF16, const_cast<uint16_t*>(w.w_out));
            default: break;
        }
    } else {
        switch (id) {
            case DM_T_GDN_QKV: return want(static_cast<uint64_t>(d.qkv_dim) * H, DM_DTYPE_BF16, win);
            case DM_T_GDN_Z: return want(static_cast<uint64_t>(d.z_dim) * H, DM_DTYPE_BF16, win + static_cast<size_t>(d.qkv_dim) * H);
            case DM_T_GDN_A: return want(static_cast<uint64_t>(d.nv) * H, DM_DTYPE_BF16, win + static_cast<size_t>(d.qkv_dim + d.z_dim) * H);
            case DM_T_GDN_B: return want(static_cast<uint64_t>(d.nv) * H, DM_DTYPE_BF16, win + static_cast<size_t>(d.qkv_dim + d.z_dim + d.nv) * H);
            case DM_T_GDN_CONV: return want(static_cast<uint64_t>(d.qkv_dim) * 4, DM_DTYPE_BF16, const_cast<uint16_t*>(w.conv_w));
            case DM_T_GDN_DT_BIAS: return want(d.nv, DM_DTYPE_F32, const_cast<float*>(w.dt_bias));
            case DM_T_GDN_A_LOG: return want(d.nv, DM_DTYPE_F32, const_cast<float*>(w.a_log));
            case DM_T_GDN_NORM: return want(d.dv, DM_DTYPE_BF16, const_cast<uint16_t*>(w.gdn_norm));
            case DM_T_GDN_OUT: return want(H * d.z_dim, DM_DTYPE_BF16, const_cast<uint16_t*>(w.w_out));
            default: break;
        }
    }
    return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer,
                   "tensor %d does not belong to a %s layer", id, w.is_attn ? "gated-attention" : "GDN");
}

int32_t dm_upload_tensor(dm_ctx* c, int32_t layer, int32_t id, int32_t dtype, const void* data, uint64_t n) {
    if (!c || !data) return DM_ERR_INVALID_ARG;
    void* dst = nullptr;
    size_t bytes = 0;
    int rc = tensor_target(c, layer, id, dtype, n, &dst, &bytes);
    if (rc != DM_OK) return rc;
    cudaSetDevice(c->device);
    DM_CUDA(c, cudaMemcpy(dst, data, bytes, cudaMemcpyHostToDevice), "loader");
    c->have_dense[static_cast<size_t>(layer + 1) * DM_T_COUNT + id] = 1;
    return DM_OK;
}

static uint8_t* expert_record(dm_ctx* c, int layer, int expert) {
    if (expert >= 0 && c->scratch_rec) return c->scratch_rec;  // a spilling pool stages routed records
    LayerW& w = c->layers[layer];
    return expert < 0 ? const_cast<uint8_t*>(w.shared)
                      : const_cast<uint8_t*>(w.experts) + static_cast<size_t>(expert) * c->d.expert_bytes;
}

// A spilling pool keeps its routed records in pinned host memory: the projection just
// repacked into the staging record is copied there.  Gate and up share chunks (rows 0-7
// and 8-15 of each chunk's nibble, scale and zero arrays), so each copies only its own
// 8-row blocks; the down projection is one contiguous region.
static cudaError_t spill_store(dm_ctx* c, int layer, int expert, int proj) {
    if (!c->scratch_rec || expert < 0) return cudaSuccess;
    const Dims& d = c->d;
    uint8_t* host = c->host_pool + (static_cast<size_t>(layer) * d.E + expert) * d.expert_bytes;
    const uint8_t* dev = c->scratch_rec;
    if (proj == DM_PROJ_DOWN) {
        const size_t off = static_cast<size_t>(d.gu_chunks) * d.gu_chunk_bytes;
        return cudaMemcpyAsync(host + off, dev + off, static_cast<size_t>(d.d_chunks) * d.d_chunk_bytes,
                               cudaMemcpyDeviceToHost, c->stream);
    }
    const size_t ng = d.H / d.G, qb = d.H / 2, sb = ng * 2, zb = ng / 2;
    const size_t r0 = proj == DM_PROJ_UP ? 8 : 0;
    const size_t part[3][2] = {{r0 * qb, 8 * qb}, {16 * qb + r0 * sb, 8 * sb}, {16 * qb + 16 * sb + r0 * zb, 8 * zb}};
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < 3 && e == cudaSuccess; ++i)
        e = cudaMemcpy2DAsync(host + part[i][0], d.gu_chunk_bytes, dev + part[i][0], d.gu_chunk_bytes, part[i][1],
                              d.gu_chunks, cudaMemcpyDeviceToHost, c->stream);
    return e;
}

int32_t dm_expert_upload(dm_ctx* c, int32_t layer, int32_t expert, int32_t proj, const uint8_t* q,
                         const uint16_t* s, const uint8_t* z) {
    if (!c || !q || !s || !z) return DM_ERR_INVALID_ARG;
    const Dims& d = c->d;
    if (layer < 0 || layer >= d.L || expert < -1 || expert >= d.E || proj < 0 || proj > 2)
        return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer, "expert index out of range");
    const int rows = proj == DM_PROJ_DOWN ? d.H : d.I;
    const int cols = proj == DM_PROJ_DOWN ? d.I : d.H;
    const size_t qb = static_cast<size_t>(rows) * cols / 2, sb = static_cast<size_t>(rows) * (cols / d.G) * 2,
                 zb = static_cast<size_t>(rows) * (cols / d.G) / 2;
    cudaSetDevice(c->device);
    DM_CUDA(c, cudaMemcpyAsync(c->stage_q, q, qb, cudaMemcpyHostToDevice, c->stream), "loader");
    DM_CUDA(c, cudaMemcpyAsync(c->stage_s, s, sb, cudaMemcpyHostToDevice, c->stream), "loader");
    DM_CUDA(c, cudaMemcpyAsync(c->stage_z, z, zb, cudaMemcpyHostToDevice, c->stream), "loader");
    uint8_t* rec = expert_record(c, layer, expert);
    uint8_t* dst = proj == DM_PROJ_DOWN ? rec + static_cast<size_t>(d.gu_chunks) * d.gu_chunk_bytes : rec;
    DM_CUDA(c, launch_repack_rows(c->stream, c->stage_q, c->stage_s, c->stage_z, rows, cols, d.G, proj, dst), "loader");
    DM_CUDA(c, spill_store(c, layer, expert, proj), "loader");
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "loader");
    c->have_expert[(static_cast<size_t>(layer) * (d.E + 1) + (expert + 1)) * 3 + proj] = 1;
    return DM_OK;
}

int32_t dm_tensor_download(dm_ctx* c, int32_t layer, int32_t id, int32_t dtype, void* out, uint64_t n) {
    if (!c || !out) return DM_ERR_INVALID_ARG;
    void* src = nullptr;
    size_t bytes = 0;
    int rc = tensor_target(c, layer, id, dtype, n, &src, &bytes);
    if (rc != DM_OK) return rc;
    cudaSetDevice(c->device);
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "loader");
    DM_CUDA(c, cudaMemcpy(out, src, bytes, cudaMemcpyDeviceToHost), "loader");
    return DM_OK;
}

// Inverse of the row repack (repack_rows_kernel): the record's chunks -> canonical rows.
int32_t dm_expert_download(dm_ctx* c, int32_t layer, int32_t expert, int32_t proj, uint8_t* q, uint16_t* s,
                           uint8_t* z) {
    if (!c || !q || !s || !z) return DM_ERR_INVALID_ARG;
    const Dims& d = c->d;
    if (layer < 0 || layer >= d.L || expert < -1 || expert >= d.E || proj < 0 || proj > 2)
        return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer, "expert index out of range");
    const int rows = proj == DM_PROJ_DOWN ? d.H : d.I;
    const int cols = proj == DM_PROJ_DOWN ? d.I : d.H;
    const int ng = cols / d.G;
    const size_t qb = cols / 2, sb = static_cast<size_t>(ng) * 2, zb = ng / 2;
    const size_t chunk_bytes = 16 * (qb + sb + zb);
    const int nchunks = proj == DM_PROJ_DOWN ? rows / 16 : rows / 8;
    uint8_t* rec = expert_record(c, layer, expert);
    const uint8_t* src = proj == DM_PROJ_DOWN ? rec + static_cast<size_t>(d.gu_chunks) * d.gu_chunk_bytes : rec;
    std::vector<uint8_t> h(chunk_bytes * nchunks);
    cudaSetDevice(c->device);
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "loader");
    if (c->scratch_rec && expert >= 0) {  // a spilling pool: the record lives in host memory
        const uint8_t* rec_h = c->host_pool + (static_cast<size_t>(layer) * d.E + expert) * d.expert_bytes;
        memcpy(h.data(), rec_h + (src - rec), h.size());
    } else {
        DM_CUDA(c, cudaMemcpy(h.data(), src, h.size(), cudaMemcpyDeviceToHost), "loader");
    }
    for (int r = 0; r < rows; ++r) {
        const int chunk = proj == DM_PROJ_DOWN ? r / 16 : r / 8;
        const int rin = proj == DM_PROJ_DOWN ? r % 16 : (proj == DM_PROJ_UP ? 8 : 0) + r % 8;
        const uint8_t* cb = h.data() + chunk * chunk_bytes;
        memcpy(q + static_cast<size_t>(r) * qb, cb + rin * qb, qb);
        memcpy(s + static_cast<size_t>(r) * ng, cb + 16 * qb + rin * sb, sb);
        memcpy(z + static_cast<size_t>(r) * zb, cb + 16 * qb + 16 * sb + rin * zb, zb);
    }
    return DM_OK;
}

static const char* tensor_name(int id) {
    static const char* names[DM_T_COUNT] = {
        "input_layernorm.weight", "post_attention_layernorm.weight", "linear_attn.in_proj_qkv.weight",
        "linear_attn.conv1d.weight", "linear_attn.in_proj_z.weight", "linear_attn.in_proj_a.weight",
        "linear_attn.in_proj_b.weight", "linear_attn.dt_bias", "linear_attn.A_log", "linear_attn.norm.weight",
        "linear_attn.out_proj.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
        "self_attn.v_proj.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
        "self_attn.o_proj.weight", "mlp.gate.weight", "mlp.shared_expert_gate.weight",
        "embed_tokens.weight", "norm.weight", "lm_head.weight"};
    return (id >= 0 && id < DM_T_COUNT) ? names[id] : "?";
}

int32_t dm_weights_check(dm_ctx* c) {
    if (!c) return DM_ERR_INVALID_ARG;
    const Dims& d = c->d;
    const int glob[] = {DM_T_EMBED, DM_T_FINAL_NORM, DM_T_LM_HEAD};
    for (int id : glob)
        if (!c->have_dense[id])
            return set_err(c, DM_ERR_NOT_READY, "WEIGHT_LOAD_FAILED", "loader", -1, "missing tensor %s", tensor_name(id));
    const int gdn_ids[] = {DM_T_INPUT_NORM, DM_T_POST_NORM, DM_T_GDN_QKV, DM_T_GDN_CONV, DM_T_GDN_Z, DM_T_GDN_A,
                           DM_T_GDN_B, DM_T_GDN_DT_BIAS, DM_T_GDN_A_LOG, DM_T_GDN_NORM, DM_T_GDN_OUT,
                           DM_T_ROUTER, DM_T_SHARED_GATE};
    const int att_ids[] = {DM_T_INPUT_NORM, DM_T_POST_NORM, DM_T_ATTN_Q, DM_T_ATTN_K, DM_T_ATTN_V,
                           DM_T_ATTN_Q_NORM, DM_T_ATTN_K_NORM, DM_T_ATTN_O, DM_T_ROUTER, DM_T_SHARED_GATE};
    for (int l = 0; l < d.L; ++l) {
        const bool att = c->layers[l].is_attn;
        const int* ids = att ? att_ids : gdn_ids;
        const int n = att ? 10 : 13;
        for (int i = 0; i < n; ++i)
            if (!c->have_dense[static_cast<size_t>(l + 1) * DM_T_COUNT + ids[i]])
                return set_err(c, DM_ERR_NOT_READY, "WEIGHT_LOAD_FAILED", "loader", l, "missing tensor layers.%d.%s", l,
                               tensor_name(ids[i]));
        for (int e = -1; e < d.E; ++e)
            for (int p = 0; p < 3; ++p)
                if (!c->have_expert[(static_cast<size_t>(l) * (d.E + 1) + (e + 1)) * 3 + p])
                    return set_err(c, DM_ERR_NOT_READY, "WEIGHT_LOAD_FAILED", "loader", l,
                                   "missing expert %d projection %d of layer %d", e, p, l);
    }
    return DM_OK;
}

int32_t dm_dequant_q4(dm_ctx* c, const uint8_t* q, const uint16_t* s, const uint8_t* z, int32_t rows,
                      int32_t cols, int32_t group, float* out) {
    if (!c || !q || !s || !z || !out || rows <= 0 || cols <= 0 || group <= 0 || cols % (2 * group) != 0)
        return c ? set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "dequant", -1, "invalid dequant arguments")
                 : DM_ERR_INVALID_ARG;
    cudaSetDevice(c->device);
    const size_t n = static_cast<size_t>(rows) * cols;
    const size_t qb = n / 2, sb = static_cast<size_t>(rows) * (cols / group) * 2, zb = static_cast<size_t>(rows) * (cols / group) / 2;
    uint8_t* tmp = nullptr;
    DM_CUDA(c, cudaMalloc(&tmp, qb + sb + zb + n * 4 + 1024), "dequant");
    uint8_t* dq = tmp;
    uint16_t* ds = reinterpret_cast<uint16_t*>(tmp + ((qb + 255) & ~size_t(255)));
    uint8_t* dz = reinterpret_cast<uint8_t*>(ds) + ((sb + 255) & ~size_t(255));
    float* dout = reinterpret_cast<float*>(dz + ((zb + 255) & ~size_t(255)));
    cudaError_t e = cudaMemcpyAsync(dq, q, qb, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(ds, s, sb, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dz, z, zb, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = launch_dequant_q4_canonical(c->stream, dq, ds, dz, rows, cols, group, dout);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, dout, n * 4, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "dequant", -1, "%s", cudaGetErrorString(e));
    return DM_OK;
}

int32_t dm_dequant_sym4(dm_ctx* c, const uint8_t* packed, const uint16_t* scales, int64_t n, int32_t group,
                        uint16_t* out_bf16, float* out_f32) {
    if (!c) return DM_ERR_INVALID_ARG;
    if (!packed || !scales || (!out_bf16 && !out_f32))
        return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "dequant", -1, "null buffer");
    if (group != 32 && group != 64 && group != 128 && group != 256)
        return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "dequant", -1,
                       "group_size must be in {32, 64, 128, 256}, got %d", group);
    if (n <= 0) return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "dequant", -1, "num_elements must be positive");
    if (n % group != 0)
        return set_err(c, DM_ERR_INVALID_ARG, "M6_ERR_INPUT", "dequant", -1,
                       "N %% G != 0 (tail group not supported): N=%lld, G=%d", static_cast<long long>(n), group);
    const int64_t ng = n / group;
    for (int64_t g = 0; g < ng; ++g) {  // the reference validates every scale before any output
        const uint16_t u = scales[g];
        if (((u >> 10) & 0x1F) == 0x1F)
            return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "dequant", -1, "scale is NaN or Inf at group %lld",
                           static_cast<long long>(g));
        if ((u & 0x8000u) || (u & 0x7FFFu) == 0)
            return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "dequant", -1, "scale is non-positive at group %lld",
                           static_cast<long long>(g));
    }
    cudaSetDevice(c->device);
    const size_t pb = static_cast<size_t>(n / 2), sb = static_cast<size_t>(ng) * 2;
    const size_t o_s = (pb + 255) & ~size_t(255), o_b = o_s + ((sb + 255) & ~size_t(255));
    const size_t o_f = o_b + (out_bf16 ? ((static_cast<size_t>(n) * 2 + 255) & ~size_t(255)) : 0);
    const size_t o_bad = o_f + (out_f32 ? ((static_cast<size_t>(n) * 4 + 255) & ~size_t(255)) : 0);
    uint8_t* tmp = nullptr;
    DM_CUDA(c, cudaMalloc(&tmp, o_bad + 256), "dequant");
    uint16_t* dbf = out_bf16 ? reinterpret_cast<uint16_t*>(tmp + o_b) : nullptr;
    float* df = out_f32 ? reinterpret_cast<float*>(tmp + o_f) : nullptr;
    unsigned* dbad = reinterpret_cast<unsigned*>(tmp + o_bad);
    unsigned bad = 0;
    cudaError_t e = cudaMemcpyAsync(tmp, packed, pb, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(tmp + o_s, scales, sb, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(dbad, 0, 4, c->stream);
    if (e == cudaSuccess)
        e = launch_dequant_sym4(c->stream, tmp, reinterpret_cast<const uint16_t*>(tmp + o_s), n, group, dbf, df, dbad);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&bad, dbad, 4, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e == cudaSuccess && !bad && out_bf16) e = cudaMemcpy(out_bf16, dbf, static_cast<size_t>(n) * 2, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && !bad && out_f32) e = cudaMemcpy(out_f32, df, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost);
    cudaFree(tmp);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "dequant", -1, "%s", cudaGetErrorString(e));
    if (bad)
        return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "dequant", -1,
                       "reserved nibble 0b1000 (-8) encountered");
    return DM_OK;
}

// ---- quant-file loaders ---------------------------------------------------------------
// Chunks of at most kLdBytes go file -> pinned host -> device -> dequant/convert kernel;
// dense tensors land in their weights directly, expert projections go through the stage
// buffers and the row repack of dm_expert_upload.
static constexpr size_t kLdBytes = 32u << 20;
static constexpr size_t kLdScaleOff = 24u << 20;  // scales of a custom-format chunk
static constexpr uint64_t kLdSym4Elems = 32ull << 20;  // elements per custom-format chunk

static int slot_dtype(int id) { return (id == DM_T_GDN_DT_BIAS || id == DM_T_GDN_A_LOG) ? DM_DTYPE_F32 : DM_DTYPE_BF16; }

static int loader_staging(dm_ctx* c) {
    if (c->ld_host) return DM_OK;
    cudaSetDevice(c->device);
    const size_t f32_elems = static_cast<size_t>(c->d.I) * c->d.H;
    void* h = nullptr;
    uint8_t* dv = nullptr;
    DM_CUDA(c, cudaMallocHost(&h, kLdBytes), "loader");
    const cudaError_t e = cudaMalloc(&dv, kLdBytes + f32_elems * 4 + 256);
    if (e != cudaSuccess) {
        cudaFreeHost(h);
        return set_err(c, DM_ERR_OOM, "CUDA_ERROR", "loader", -1, "loader staging: %s", cudaGetErrorString(e));
    }
    c->ld_host = h;
    c->ld_dev = dv;
    c->ld_f32 = reinterpret_cast<float*>(dv + kLdBytes);
    c->ld_word = reinterpret_cast<unsigned*>(dv + kLdBytes + f32_elems * 4);
    return DM_OK;
}

static int expert_geometry(dm_ctx* c, int layer, int expert, int proj, int* rows, int* cols) {
    const Dims& d = c->d;
    if (layer < 0 || layer >= d.L || expert < -1 || expert >= d.E || proj < 0 || proj > 2)
        return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer, "expert index out of range");
    *rows = proj == DM_PROJ_DOWN ? d.H : d.I;
    *cols = proj == DM_PROJ_DOWN ? d.I : d.H;
    if (*cols % (2 * d.G) != 0)
        return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer,
                       "row length %d is not a multiple of two pool groups", *cols);
    return DM_OK;
}

// stage buffers (q, s, z of rows x cols) -> the expert record
static int pool_commit(dm_ctx* c, int rows, int cols, int layer, int expert, int proj) {
    const Dims& d = c->d;
    uint8_t* rec = expert_record(c, layer, expert);
    uint8_t* dst = proj == DM_PROJ_DOWN ? rec + static_cast<size_t>(d.gu_chunks) * d.gu_chunk_bytes : rec;
    DM_CUDA(c, launch_repack_rows(c->stream, c->stage_q, c->stage_s, c->stage_z, rows, cols, d.G, proj, dst), "loader");
    DM_CUDA(c, spill_store(c, layer, expert, proj), "loader");
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "loader");
    c->have_expert[(static_cast<size_t>(layer) * (d.E + 1) + (expert + 1)) * 3 + proj] = 1;
    return DM_OK;
}

// c->ld_f32 (rows x cols fp32) -> re-quantised stage buffers -> the expert record
static int requant_commit(dm_ctx* c, int rows, int cols, int layer, int expert, int proj, float* max_err) {
    unsigned w[2] = {0, 0};
    DM_CUDA(c, cudaMemsetAsync(c->ld_word, 0, 8, c->stream), "loader");
    DM_CUDA(c, launch_requant_pool(c->stream, c->ld_f32, rows, cols, c->d.G, c->stage_q, c->stage_s, c->stage_z,
                                   c->ld_word, c->ld_word + 1), "loader");
    DM_CUDA(c, cudaMemcpyAsync(w, c->ld_word, 8, cudaMemcpyDeviceToHost, c->stream), "loader");
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "loader");
    if (w[0] & 8u)
        return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer,
                       "non-finite weight in expert %d projection %d", expert, proj);
    float e;
    memcpy(&e, &w[1], 4);
    if (max_err) *max_err = e;
    return pool_commit(c, rows, cols, layer, expert, proj);
}

// Elements [first, first + n) of GGUF tensor ti dequantised into out_f32 / out_bf16
// (device pointers), chunk by chunk.
static int gguf_stream(dm_ctx* c, const dm_gguf* g, int64_t ti, const dm_gguf_tensor_info& info, uint64_t first,
                       uint64_t n, float* out_f32, uint16_t* out_bf16, unsigned flags, int layer) {
    int bs, bpb;
    dm_ggml_block_spec(info.ggml_type, &bs, &bpb);
    if (first % bs || n % bs)
        return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer,
                       "tensor %s: range [%llu, +%llu) is not whole %d-element blocks", info.name,
                       (unsigned long long)first, (unsigned long long)n, bs);
    int rc = loader_staging(c);
    if (rc != DM_OK) return rc;
    const uint64_t per = kLdBytes / bpb;
    const uint64_t b_end = (first + n) / bs;
    for (uint64_t b0 = first / bs; b0 < b_end; b0 += per) {
        const uint64_t nb = b_end - b0 < per ? b_end - b0 : per;
        rc = dm_gguf_read(g, ti, b0 * bpb, c->ld_host, nb * bpb);
        if (rc != DM_OK)
            return set_err(c, DM_ERR_IO, "GGUF_READ_ERROR", "loader", layer, "truncated read for tensor %s", info.name);
        DM_CUDA(c, cudaMemcpyAsync(c->ld_dev, c->ld_host, nb * bpb, cudaMemcpyHostToDevice, c->stream), "loader");
        const uint64_t o = b0 * bs - first;
        DM_CUDA(c, launch_gguf_dequant(c->stream, info.ggml_type, c->ld_dev, static_cast<int64_t>(nb * bs), flags,
                                       out_f32 ? out_f32 + o : nullptr, out_bf16 ? out_bf16 + o : nullptr), "loader");
        DM_CUDA(c, cudaStreamSynchronize(c->stream), "loader");
    }
    return DM_OK;
}

static int gguf_lookup(dm_ctx* c, const dm_gguf* g, const char* name, int layer, int64_t* ti,
                       dm_gguf_tensor_info* info) {
    if (!g || !name) return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer, "null argument");
    *ti = dm_gguf_find(g, name);
    if (*ti < 0)
        return set_err(c, DM_ERR_NOT_READY, "WEIGHT_LOAD_FAILED", "loader", layer, "tensor not found in GGUF index: %s", name);
    dm_gguf_tensor(g, *ti, info);
    if (!gguf_type_supported(info->ggml_type))
        return set_err(c, DM_ERR_INVALID_ARG, "GGUF_UNSUPPORTED_DTYPE", "loader", layer,
                       "unsupported GGML type %d for tensor %s", info->ggml_type, name);
    return DM_OK;
}

int32_t dm_gguf_dequant(dm_ctx* c, int32_t type, const void* raw, uint64_t raw_bytes, uint64_t n, uint32_t flags,
                        float* out_f32, uint16_t* out_bf16) {
    if (!c) return DM_ERR_INVALID_ARG;
    if (!raw || (!out_f32 && !out_bf16))
        return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "dequant", -1, "null buffer");
    if (!gguf_type_supported(type))
        return set_err(c, DM_ERR_INVALID_ARG, "GGUF_UNSUPPORTED_DTYPE", "dequant", -1, "unsupported GGML type %d", type);
    int bs, bpb;
    dm_ggml_block_spec(type, &bs, &bpb);
    if (n == 0 || n % bs)
        return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "dequant", -1,
                       "%llu elements is not a positive multiple of the %d-element block", (unsigned long long)n, bs);
    const uint64_t need = n / bs * bpb;
    if (raw_bytes < need)
        return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "dequant", -1, "%llu raw bytes, %llu needed",
                       (unsigned long long)raw_bytes, (unsigned long long)need);
    cudaSetDevice(c->device);
    const size_t o_f = (need + 255) & ~size_t(255);
    const size_t o_b = o_f + (out_f32 ? ((n * 4 + 255) & ~size_t(255)) : 0);
    const size_t total = o_b + (out_bf16 ? n * 2 : 0) + 256;
    uint8_t* tmp = nullptr;
    DM_CUDA(c, cudaMalloc(&tmp, total), "dequant");
    float* df = out_f32 ? reinterpret_cast<float*>(tmp + o_f) : nullptr;
    uint16_t* db = out_bf16 ? reinterpret_cast<uint16_t*>(tmp + o_b) : nullptr;
    cudaError_t e = cudaMemcpyAsync(tmp, raw, need, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = launch_gguf_dequant(c->stream, type, tmp, static_cast<int64_t>(n), flags, df, db);
    if (e == cudaSuccess && df) e = cudaMemcpyAsync(out_f32, df, n * 4, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess && db) e = cudaMemcpyAsync(out_bf16, db, n * 2, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "dequant", -1, "%s", cudaGetErrorString(e));
    return DM_OK;
}

int32_t dm_gguf_load_tensor(dm_ctx* c, const dm_gguf* g, const char* name, int32_t layer, int32_t id, uint32_t flags) {
    if (!c) return DM_ERR_INVALID_ARG;
    int64_t ti;
    dm_gguf_tensor_info info;
    int rc = gguf_lookup(c, g, name, layer, &ti, &info);
    if (rc != DM_OK) return rc;
    const int dt = slot_dtype(id);
    void* dst = nullptr;
    size_t bytes = 0;
    rc = tensor_target(c, layer, id, dt, info.num_elements, &dst, &bytes);
    if (rc != DM_OK) return rc;
    cudaSetDevice(c->device);
    rc = gguf_stream(c, g, ti, info, 0, info.num_elements, dt == DM_DTYPE_F32 ? static_cast<float*>(dst) : nullptr,
                     dt == DM_DTYPE_BF16 ? static_cast<uint16_t*>(dst) : nullptr, flags, layer);
    if (rc != DM_OK) return rc;
    c->have_dense[static_cast<size_t>(layer + 1) * DM_T_COUNT + id] = 1;
    return DM_OK;
}

// first element of a (slab, row0) slice of a tensor whose innermost length is `inner`
// and whose slabs hold `slab_elems` elements
static int slice_start(dm_ctx* c, const char* name, int layer, uint64_t inner, uint64_t slab_elems, uint64_t total,
                       int64_t slab, int64_t row0, int rows, int cols, uint64_t* first) {
    if (inner != static_cast<uint64_t>(cols))
        return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer,
                       "tensor %s: rows of %llu elements, the projection has %d", name, (unsigned long long)inner, cols);
    if (slab < 0 || row0 < 0)
        return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer, "negative slab or row");
    const uint64_t f = static_cast<uint64_t>(slab) * slab_elems + static_cast<uint64_t>(row0) * cols;
    const uint64_t n = static_cast<uint64_t>(rows) * cols;
    if (static_cast<uint64_t>(row0) * cols + n > slab_elems || f + n > total)
        return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer,
                       "tensor %s: slice (slab %lld, row %lld, %d rows) is outside the tensor", name,
                       (long long)slab, (long long)row0, rows);
    *first = f;
    return DM_OK;
}

int32_t dm_gguf_load_expert(dm_ctx* c, const dm_gguf* g, const char* name, int64_t slab, int64_t row0, int32_t layer,
                            int32_t expert, int32_t proj, uint32_t flags, float* max_err) {
    if (!c) return DM_ERR_INVALID_ARG;
    int rows, cols;
    int rc = expert_geometry(c, layer, expert, proj, &rows, &cols);
    if (rc != DM_OK) return rc;
    int64_t ti;
    dm_gguf_tensor_info info;
    rc = gguf_lookup(c, g, name, layer, &ti, &info);
    if (rc != DM_OK) return rc;
    const uint64_t slab_elems = info.ndim >= 2 ? info.dims[0] * info.dims[1] : info.num_elements;
    uint64_t first;
    rc = slice_start(c, name, layer, info.dims[0], slab_elems, info.num_elements, slab, row0, rows, cols, &first);
    if (rc != DM_OK) return rc;
    if (!(flags & DM_LOAD_REQUANT))
        return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer,
                       "tensor %s: GGML type %d is not representable exactly in the 4-bit g%d expert pool "
                       "(re-quantisation needs DM_LOAD_REQUANT)", name, info.ggml_type, c->d.G);
    cudaSetDevice(c->device);
    if ((rc = loader_staging(c)) != DM_OK) return rc;  // c->ld_f32 exists from here on
    rc = gguf_stream(c, g, ti, info, first, static_cast<uint64_t>(rows) * cols, c->ld_f32, nullptr, flags, layer);
    if (rc != DM_OK) return rc;
    return requant_commit(c, rows, cols, layer, expert, proj, max_err);
}

static int qf_lookup(dm_ctx* c, const dm_quant_file* q, const char* name, int layer, int64_t* ti,
                     dm_quant_tensor_info* info) {
    if (!q || !name) return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer, "null argument");
    *ti = dm_quant_file_find(q, name);
    if (*ti < 0)
        return set_err(c, DM_ERR_NOT_READY, "WEIGHT_LOAD_FAILED", "loader", layer, "tensor not found in quant model: %s",
                       name);
    dm_quant_file_tensor(q, *ti, info);
    return DM_OK;
}

// Elements [first, first + n) of a custom-format tensor (first, n multiples of its group)
// into ld_host: the scales at kLdScaleOff, the nibbles at 0; then onto the device at the
// same offsets.  Every scale is checked first (validate_quant_payload,
// quant_reader.mojo:464-494).
static int qf_stage(dm_ctx* c, const dm_quant_file* q, int64_t ti, const dm_quant_tensor_info& info, uint64_t first,
                    uint64_t n, int layer) {
    const uint64_t G = static_cast<uint64_t>(info.group_size);
    auto* h = static_cast<uint8_t*>(c->ld_host);
    if (dm_quant_file_read(q, ti, 0, first / G * 2, h + kLdScaleOff, n / G * 2) != DM_OK ||
        dm_quant_file_read(q, ti, 1, first / 2, h, n / 2) != DM_OK)
        return set_err(c, DM_ERR_IO, "WEIGHT_LOAD_FAILED", "loader", layer, "short read of tensor %s", info.name);
    const uint16_t* s = reinterpret_cast<const uint16_t*>(h + kLdScaleOff);
    for (uint64_t i = 0; i < n / G; ++i) {
        if (((s[i] >> 10) & 0x1F) == 0x1F)
            return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "loader", layer, "scale is NaN or Inf in tensor: %s",
                           info.name);
        if ((s[i] & 0x8000u) || (s[i] & 0x7FFFu) == 0)
            return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "loader", layer, "scale is non-positive in tensor: %s",
                           info.name);
    }
    DM_CUDA(c, cudaMemcpyAsync(c->ld_dev, h, n / 2, cudaMemcpyHostToDevice, c->stream), "loader");
    DM_CUDA(c, cudaMemcpyAsync(c->ld_dev + kLdScaleOff, h + kLdScaleOff, n / G * 2, cudaMemcpyHostToDevice, c->stream),
            "loader");
    return DM_OK;
}

int32_t dm_quant_file_load_tensor(dm_ctx* c, const dm_quant_file* q, const char* name, int32_t layer, int32_t id) {
    if (!c) return DM_ERR_INVALID_ARG;
    int64_t ti;
    dm_quant_tensor_info info;
    int rc = qf_lookup(c, q, name, layer, &ti, &info);
    if (rc != DM_OK) return rc;
    const int dt = slot_dtype(id);
    void* dst = nullptr;
    size_t bytes = 0;
    rc = tensor_target(c, layer, id, dt, info.num_elements, &dst, &bytes);
    if (rc != DM_OK) return rc;
    cudaSetDevice(c->device);
    if ((rc = loader_staging(c)) != DM_OK) return rc;
    const uint64_t N = info.num_elements;
    for (uint64_t e0 = 0; e0 < N; e0 += kLdSym4Elems) {
        const uint64_t n = N - e0 < kLdSym4Elems ? N - e0 : kLdSym4Elems;
        if ((rc = qf_stage(c, q, ti, info, e0, n, layer)) != DM_OK) return rc;
        DM_CUDA(c, cudaMemsetAsync(c->ld_word, 0, 4, c->stream), "loader");
        DM_CUDA(c, launch_dequant_sym4(c->stream, c->ld_dev, reinterpret_cast<const uint16_t*>(c->ld_dev + kLdScaleOff),
                                       static_cast<int64_t>(n), info.group_size,
                                       dt == DM_DTYPE_BF16 ? static_cast<uint16_t*>(dst) + e0 : nullptr,
                                       dt == DM_DTYPE_F32 ? static_cast<float*>(dst) + e0 : nullptr, c->ld_word),
                "loader");
        unsigned badw = 0;
        DM_CUDA(c, cudaMemcpyAsync(&badw, c->ld_word, 4, cudaMemcpyDeviceToHost, c->stream), "loader");
        DM_CUDA(c, cudaStreamSynchronize(c->stream), "loader");
        if (badw)
            return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "loader", layer,
                           "reserved nibble 0x8 (-8) in tensor: %s", info.name);
    }
    c->have_dense[static_cast<size_t>(layer + 1) * DM_T_COUNT + id] = 1;
    return DM_OK;
}

int32_t dm_quant_file_load_expert(dm_ctx* c, const dm_quant_file* q, const char* name, int64_t slab, int64_t row0,
                                  int32_t layer, int32_t expert, int32_t proj, uint32_t flags, float* max_err) {
    if (!c) return DM_ERR_INVALID_ARG;
    int rows, cols;
    int rc = expert_geometry(c, layer, expert, proj, &rows, &cols);
    if (rc != DM_OK) return rc;
    int64_t ti;
    dm_quant_tensor_info info;
    rc = qf_lookup(c, q, name, layer, &ti, &info);
    if (rc != DM_OK) return rc;
    const int nd = info.ndim;
    const uint64_t inner = info.shape[nd - 1];
    const uint64_t slab_elems = nd >= 2 ? info.shape[nd - 1] * info.shape[nd - 2] : info.num_elements;
    uint64_t first;
    rc = slice_start(c, name, layer, inner, slab_elems, info.num_elements, slab, row0, rows, cols, &first);
    if (rc != DM_OK) return rc;
    const uint64_t n = static_cast<uint64_t>(rows) * cols;
    if (first % info.group_size || n % info.group_size)
        return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer,
                       "tensor %s: the slice does not start on a group boundary", name);
    cudaSetDevice(c->device);
    if ((rc = loader_staging(c)) != DM_OK) return rc;
    if ((rc = qf_stage(c, q, ti, info, first, n, layer)) != DM_OK) return rc;
    const uint16_t* ds = reinterpret_cast<const uint16_t*>(c->ld_dev + kLdScaleOff);
    unsigned w = 0;
    DM_CUDA(c, cudaMemsetAsync(c->ld_word, 0, 4, c->stream), "loader");
    DM_CUDA(c, launch_sym4_to_pool(c->stream, c->ld_dev, ds, 0, rows, cols, info.group_size, c->d.G, c->stage_q,
                                   c->stage_s, c->stage_z, c->ld_word), "loader");
    DM_CUDA(c, cudaMemcpyAsync(&w, c->ld_word, 4, cudaMemcpyDeviceToHost, c->stream), "loader");
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "loader");
    if (w & 1u)
        return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "loader", layer, "reserved nibble 0x8 (-8) in tensor: %s",
                       name);
    if (w & 2u)
        return set_err(c, DM_ERR_INVALID_ARG, "DEQUANT_ERROR", "loader", layer, "invalid scale in tensor: %s", name);
    if (!(w & 4u)) {
        if (max_err) *max_err = 0.0f;
        return pool_commit(c, rows, cols, layer, expert, proj);
    }
    if (!(flags & DM_LOAD_REQUANT))
        return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", layer,
                       "tensor %s: groups of %d with different scales inside one pool group of %d are not "
                       "representable exactly (re-quantisation needs DM_LOAD_REQUANT)", name, info.group_size, c->d.G);
    DM_CUDA(c, cudaMemsetAsync(c->ld_word, 0, 4, c->stream), "loader");
    DM_CUDA(c, launch_dequant_sym4(c->stream, c->ld_dev, ds, static_cast<int64_t>(n), info.group_size, nullptr,
                                   c->ld_f32, c->ld_word), "loader");
    return requant_commit(c, rows, cols, layer, expert, proj, max_err);
}

int32_t dm_quant_file_load(dm_ctx* c, const dm_quant_file* q, uint32_t flags) {
    if (!c) return DM_ERR_INVALID_ARG;
    if (!q) return set_err(c, DM_ERR_INVALID_ARG, "WEIGHT_LOAD_FAILED", "loader", -1, "null quant file");
    const Dims& d = c->d;
    auto has = [&](const std::string& s) { return dm_quant_file_find(q, s.c_str()) >= 0; };
    auto pick = [&](std::initializer_list<std::string> names) -> std::string {
        for (const std::string& s : names)
            if (has(s)) return s;
        return std::string();
    };
    auto missing = [&](int layer, const std::string& what) {
        return set_err(c, DM_ERR_NOT_READY, "WEIGHT_LOAD_FAILED", "loader", layer, "tensor not found in quant model: %s",
                       what.c_str());
    };
    struct G { int id; const char* a; const char* b; };
    const G globals[] = {{DM_T_EMBED, "model.language_model.embed_tokens.weight", "model.embed_tokens.weight"},
                         {DM_T_FINAL_NORM, "model.language_model.norm.weight", "model.norm.weight"},
                         {DM_T_LM_HEAD, "lm_head.weight", "lm_head.weight"}};
    // a weight the file lacks may have been uploaded before (e.g. tensors too small for the
    // format's groups); only what is still missing is an error
    auto have_dense = [&](int layer, int id) { return c->have_dense[static_cast<size_t>(layer + 1) * DM_T_COUNT + id] != 0; };
    auto have_expert = [&](int layer, int e, int p) {
        return c->have_expert[(static_cast<size_t>(layer) * (d.E + 1) + (e + 1)) * 3 + p] != 0;
    };
    int rc;
    for (const G& gl : globals) {
        const std::string nm = pick({gl.a, gl.b});
        if (nm.empty() && have_dense(-1, gl.id)) continue;
        if (nm.empty()) return missing(-1, gl.a);
        if ((rc = dm_quant_file_load_tensor(c, q, nm.c_str(), -1, gl.id)) != DM_OK) return rc;
    }
    const int gdn_ids[] = {DM_T_INPUT_NORM, DM_T_POST_NORM, DM_T_GDN_QKV, DM_T_GDN_CONV, DM_T_GDN_Z, DM_T_GDN_A,
                           DM_T_GDN_B, DM_T_GDN_DT_BIAS, DM_T_GDN_A_LOG, DM_T_GDN_NORM, DM_T_GDN_OUT,
                           DM_T_ROUTER, DM_T_SHARED_GATE};
    const int att_ids[] = {DM_T_INPUT_NORM, DM_T_POST_NORM, DM_T_ATTN_Q, DM_T_ATTN_K, DM_T_ATTN_V,
                           DM_T_ATTN_Q_NORM, DM_T_ATTN_K_NORM, DM_T_ATTN_O, DM_T_ROUTER, DM_T_SHARED_GATE};
    static const char* proj_names[3] = {"gate_proj.weight", "up_proj.weight", "down_proj.weight"};
    for (int l = 0; l < d.L; ++l) {
        const std::string p1 = "model.language_model.layers." + std::to_string(l) + ".";
        const std::string p2 = "model.layers." + std::to_string(l) + ".";
        const bool att = c->layers[l].is_attn;
        const int* ids = att ? att_ids : gdn_ids;
        const int nids = att ? 10 : 13;
        for (int i = 0; i < nids; ++i) {
            const std::string nm = pick({p1 + tensor_name(ids[i]), p2 + tensor_name(ids[i])});
            if (nm.empty() && have_dense(l, ids[i])) continue;
            if (nm.empty()) return missing(l, p2 + tensor_name(ids[i]));
            if ((rc = dm_quant_file_load_tensor(c, q, nm.c_str(), l, ids[i])) != DM_OK) return rc;
        }
        for (int p = 0; p < 3; ++p) {
            const std::string nm = pick({p1 + "mlp.shared_expert." + proj_names[p], p2 + "mlp.shared_expert." + proj_names[p]});
            if (nm.empty() && have_expert(l, -1, p)) continue;
            if (nm.empty()) return missing(l, p2 + "mlp.shared_expert." + proj_names[p]);
            if ((rc = dm_quant_file_load_expert(c, q, nm.c_str(), 0, 0, l, -1, p, flags, nullptr)) != DM_OK) return rc;
        }
        const std::string gu = pick({p1 + "mlp.experts.gate_up_proj", p2 + "mlp.experts.gate_up_proj",
                                     p1 + "mlp.experts.gate_up_proj.weight", p2 + "mlp.experts.gate_up_proj.weight"});
        const std::string dn = pick({p1 + "mlp.experts.down_proj", p2 + "mlp.experts.down_proj",
                                     p1 + "mlp.experts.down_proj.weight", p2 + "mlp.experts.down_proj.weight"});
        for (int e = 0; e < d.E; ++e) {
            const std::string pe = "mlp.experts." + std::to_string(e) + ".";
            for (int p = 0; p < 3; ++p) {
                const std::string nm = pick({p1 + pe + proj_names[p], p2 + pe + proj_names[p]});
                if (!nm.empty()) {
                    rc = dm_quant_file_load_expert(c, q, nm.c_str(), 0, 0, l, e, p, flags, nullptr);
                } else if (p < 2 && !gu.empty()) {
                    rc = dm_quant_file_load_expert(c, q, gu.c_str(), e, p == DM_PROJ_UP ? d.I : 0, l, e, p, flags, nullptr);
                } else if (p == 2 && !dn.empty()) {
                    rc = dm_quant_file_load_expert(c, q, dn.c_str(), e, 0, l, e, p, flags, nullptr);
                } else if (have_expert(l, e, p)) {
                    rc = DM_OK;
                } else {
                    return missing(l, p2 + pe + proj_names[p]);
                }
                if (rc != DM_OK) return rc;
            }
        }
    }
    return DM_OK;
}

// ---- sequence state -------------------------------------------------------------------
static int check_slot(dm_ctx* c, int slot) {
    if (!c) return DM_ERR_INVALID_ARG;
    if (slot < 0 || slot >= c->d.max_seqs)
        return set_err(c, DM_ERR_INVALID_ARG, "M5_ERR_INPUT", "kv_alloc", -1, "slot %d out of range", slot);
    return DM_OK;
}

int32_t dm_seq_reset(dm_ctx* c, int32_t slot) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    const Dims& d = c->d;
    cudaSetDevice(c->device);
    for (int g = 0; g < d.n_gdn; ++g) {
        const size_t ls = static_cast<size_t>(g) * d.max_seqs + slot;
        DM_CUDA(c, cudaMemsetAsync(c->b.ring + ls * kConvRing * d.qkv_dim, 0, sizeof(float) * kConvRing * d.qkv_dim, c->stream), "kv_alloc");
        DM_CUDA(c, cudaMemsetAsync(c->b.S + ls * d.nv * d.dv * d.dk, 0, sizeof(float) * d.nv * d.dv * d.dk, c->stream), "kv_alloc");
    }
    // identity page table when the pool holds max_pages per slot
    std::vector<int> pt(d.max_pages, -1);
    if (static_cast<int64_t>(d.max_seqs) * d.max_pages <= d.num_pages)
        for (int p = 0; p < d.max_pages; ++p) pt[p] = slot * d.max_pages + p;
    DM_CUDA(c, cudaMemcpyAsync(c->b.page_table + static_cast<size_t>(slot) * d.max_pages, pt.data(), pt.size() * 4,
                               cudaMemcpyHostToDevice, c->stream), "kv_alloc");
    DM_CUDA(c, cudaMemsetAsync(c->b.pos + slot, 0, 4, c->stream), "kv_alloc");
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "kv_alloc");
    c->slot_len[slot] = 0;
    for (int a = 0; a < d.n_att; ++a) c->att_len[static_cast<size_t>(a) * d.max_seqs + slot] = 0;
    c->dev_pos_valid[slot] = 1;
    return DM_OK;
}

int32_t dm_seq_set_page_table(dm_ctx* c, int32_t slot, const int32_t* pages, int32_t n) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    const Dims& d = c->d;
    if (!pages || n < 0 || n > d.max_pages)
        return set_err(c, DM_ERR_INVALID_ARG, "M5_ERR_INPUT", "kv_alloc", -1, "page count %d outside [0, %d]", n, d.max_pages);
    std::vector<int> pt(d.max_pages, -1);
    for (int i = 0; i < n; ++i) {
        if (pages[i] < 0 || pages[i] >= d.num_pages)
            return set_err(c, DM_ERR_INVALID_ARG, "KV_PAGE_ERROR", "kv_alloc", -1, "page %d outside the pool", pages[i]);
        pt[i] = pages[i];
    }
    cudaSetDevice(c->device);
    DM_CUDA(c, cudaMemcpy(c->b.page_table + static_cast<size_t>(slot) * d.max_pages, pt.data(), pt.size() * 4,
                          cudaMemcpyHostToDevice), "kv_alloc");
    return DM_OK;
}

int32_t dm_seq_get_len(dm_ctx* c, int32_t slot, int32_t* len) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    if (!len) return DM_ERR_INVALID_ARG;
    *len = c->slot_len[slot];
    return DM_OK;
}

int32_t dm_seq_set_len(dm_ctx* c, int32_t slot, int32_t len) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    if (len < 0 || len > c->d.max_pages * kPageTokens)
        return set_err(c, DM_ERR_CAPACITY, "M5_ERR_CONTEXT_SIZE", "kv_alloc", -1, "length %d exceeds capacity", len);
    c->slot_len[slot] = len;
    c->dev_pos_valid[slot] = 0;
    return DM_OK;
}

int32_t dm_kv_import(dm_ctx* c, int32_t att, int32_t slot, const uint16_t* k, const uint16_t* v, int32_t n) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    const Dims& d = c->d;
    if (att < 0 || att >= d.n_att || !k || !v || n < 0 || n > d.max_pages * kPageTokens)
        return set_err(c, DM_ERR_INVALID_ARG, "M5_ERR_INPUT", "kv_import", -1, "invalid kv import arguments");
    cudaSetDevice(c->device);
    if (n > 0) {
        const size_t bytes = static_cast<size_t>(n) * d.Hkv * d.D * 2;
        uint16_t* tmp = nullptr;
        DM_CUDA(c, cudaMalloc(&tmp, 2 * bytes), "kv_import");
        cudaError_t e = cudaMemcpyAsync(tmp, k, bytes, cudaMemcpyHostToDevice, c->stream);
        if (e == cudaSuccess) e = cudaMemcpyAsync(tmp + bytes / 2, v, bytes, cudaMemcpyHostToDevice, c->stream);
        uint16_t* kvl = c->b.kv + static_cast<size_t>(att) * d.num_pages * 2 * d.Hkv * kPageTokens * d.D;
        if (e == cudaSuccess)
            e = launch_kv_copy(c->stream, kvl, c->b.page_table + static_cast<size_t>(slot) * d.max_pages, d.Hkv, d.D,
                               tmp, tmp + bytes / 2, n, 1);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
        cudaFree(tmp);
        if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "kv_import", -1, "%s", cudaGetErrorString(e));
        rc = check_device_error(c, "kv_import");
        if (rc != DM_OK) return rc;
    }
    c->att_len[static_cast<size_t>(att) * d.max_seqs + slot] = n;
    return DM_OK;
}

int32_t dm_kv_export(dm_ctx* c, int32_t att, int32_t slot, uint16_t* k, uint16_t* v, int32_t n) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    const Dims& d = c->d;
    if (att < 0 || att >= d.n_att || !k || !v || n < 0 || n > c->att_len[static_cast<size_t>(att) * d.max_seqs + slot])
        return set_err(c, DM_ERR_INVALID_ARG, "M5_ERR_DECODE", "kv_export", -1, "invalid slice length %d", n);
    if (n == 0) return DM_OK;
    cudaSetDevice(c->device);
    const size_t bytes = static_cast<size_t>(n) * d.Hkv * d.D * 2;
    uint16_t* tmp = nullptr;
    DM_CUDA(c, cudaMalloc(&tmp, 2 * bytes), "kv_export");
    uint16_t* kvl = c->b.kv + static_cast<size_t>(att) * d.num_pages * 2 * d.Hkv * kPageTokens * d.D;
    cudaError_t e = launch_kv_copy(c->stream, kvl, c->b.page_table + static_cast<size_t>(slot) * d.max_pages, d.Hkv,
                                   d.D, tmp, tmp + bytes / 2, n, 0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(k, tmp, bytes, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(v, tmp + bytes / 2, bytes, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "kv_export", -1, "%s", cudaGetErrorString(e));
    return check_device_error(c, "kv_export");
}

static int gdn_state_ptrs(dm_ctx* c, int g, int slot, float** S, float** ring) {
    const Dims& d = c->d;
    if (g < 0 || g >= d.n_gdn) return set_err(c, DM_ERR_INVALID_ARG, "GDN_ERROR", "gdn_state", -1, "gdn layer %d out of range", g);
    const size_t ls = static_cast<size_t>(g) * d.max_seqs + slot;
    *S = c->b.S + ls * d.nv * d.dv * d.dk;
    *ring = c->b.ring + ls * kConvRing * d.qkv_dim;
    return DM_OK;
}

int32_t dm_gdn_state_import(dm_ctx* c, int32_t g, int32_t slot, const float* S_host, const float* conv_host) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    float *S, *ring;
    if ((rc = gdn_state_ptrs(c, g, slot, &S, &ring)) != DM_OK) return rc;
    const Dims& d = c->d;
    cudaSetDevice(c->device);
    if (S_host) DM_CUDA(c, cudaMemcpy(S, S_host, sizeof(float) * d.nv * d.dv * d.dk, cudaMemcpyHostToDevice), "gdn_state");
    DM_CUDA(c, cudaMemset(ring, 0, sizeof(float) * kConvRing * d.qkv_dim), "gdn_state");
    if (conv_host) {
        const int L = c->slot_len[slot];
        for (int j = 0; j < 3; ++j) {
            const int p = L - 3 + j;
            if (p < 0) continue;
            DM_CUDA(c, cudaMemcpy(ring + static_cast<size_t>(p & 3) * d.qkv_dim, conv_host + static_cast<size_t>(j) * d.qkv_dim,
                                  sizeof(float) * d.qkv_dim, cudaMemcpyHostToDevice), "gdn_state");
        }
    }
    return DM_OK;
}

// The conv window alone (positions len-3 .. len-1 from conv_host [3][qkv_dim]); S untouched.
static int dm_gdn_state_import_conv(dm_ctx* c, int g, int slot, const float* conv_host) {
    return dm_gdn_state_import(c, g, slot, nullptr, conv_host);
}

int32_t dm_gdn_state_export(dm_ctx* c, int32_t g, int32_t slot, float* S_host, float* conv_host) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    float *S, *ring;
    if ((rc = gdn_state_ptrs(c, g, slot, &S, &ring)) != DM_OK) return rc;
    const Dims& d = c->d;
    cudaSetDevice(c->device);
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "gdn_state");
    if (S_host) DM_CUDA(c, cudaMemcpy(S_host, S, sizeof(float) * d.nv * d.dv * d.dk, cudaMemcpyDeviceToHost), "gdn_state");
    if (conv_host) {
        const int L = c->slot_len[slot];
        for (int j = 0; j < 3; ++j) {
            const int p = L - 3 + j;
            float* dst = conv_host + static_cast<size_t>(j) * d.qkv_dim;
            if (p < 0) {
                memset(dst, 0, sizeof(float) * d.qkv_dim);
                continue;
            }
            DM_CUDA(c, cudaMemcpy(dst, ring + static_cast<size_t>(p & 3) * d.qkv_dim, sizeof(float) * d.qkv_dim,
                                  cudaMemcpyDeviceToHost), "gdn_state");
        }
    }
    return DM_OK;
}

// ---- session files (KMSS v1) ------------------------------------------------------------
// Byte layout of reference src/format/kmss.mojo: header :6-27 / write_kmss_v1 :90-170,
// payload order :172-215 (KV: kv index, position, attention layer, head, dim), token
// prefix :217-224, SHA-256 over header || payload :226-240, tmp + rename :242-277; checks
// of read_kmss_v1 :280-360 in the same order with the same error types.

static void put_u32(uint8_t* b, uint32_t v) {
    for (int i = 0; i < 4; ++i) b[i] = static_cast<uint8_t>(v >> (8 * i));
}
static void put_u64(uint8_t* b, uint64_t v) {
    for (int i = 0; i < 8; ++i) b[i] = static_cast<uint8_t>(v >> (8 * i));
}
static uint32_t get_u32(const uint8_t* b) {
    return uint32_t(b[0]) | (uint32_t(b[1]) << 8) | (uint32_t(b[2]) << 16) | (uint32_t(b[3]) << 24);
}
static uint64_t get_u64(const uint8_t* b) {
    uint64_t v = 0;
    for (int i = 0; i < 8; ++i) v |= uint64_t(b[i]) << (8 * i);
    return v;
}
static float bf16_bits_to_f32(uint16_t h) {
    uint32_t u = static_cast<uint32_t>(h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}
static uint16_t f32_to_bf16_rne(float f) {  // round to nearest even; NaN stays NaN
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return static_cast<uint16_t>((u >> 16) | 0x40);
    const uint32_t r = u + 0x7FFFu + ((u >> 16) & 1u);
    return static_cast<uint16_t>(r >> 16);
}

int32_t dm_seq_copy(dm_ctx* c, int32_t src, int32_t dst) {
    int rc = check_slot(c, src);
    if (rc == DM_OK) rc = check_slot(c, dst);
    if (rc != DM_OK) return rc;
    if (src == dst) return DM_OK;
    const Dims& d = c->d;
    const int L = c->slot_len[src];
    for (int a = 0; a < d.n_att; ++a)
        if (c->att_len[static_cast<size_t>(a) * d.max_seqs + src] != L)
            return set_err(c, DM_ERR_POSITION, "M5_ERR_DECODE", "seq_copy", -1,
                           "source slot %d: attention layer %d holds %d positions, the sequence %d", src, a,
                           c->att_len[static_cast<size_t>(a) * d.max_seqs + src], L);
    cudaSetDevice(c->device);
    const size_t kv_layer = static_cast<size_t>(d.num_pages) * 2 * d.Hkv * kPageTokens * d.D;
    cudaError_t e = cudaSuccess;
    for (int a = 0; a < d.n_att && e == cudaSuccess; ++a)
        e = launch_kv_seq_copy(c->stream, c->b.kv + a * kv_layer, c->b.page_table + static_cast<size_t>(src) * d.max_pages,
                               c->b.page_table + static_cast<size_t>(dst) * d.max_pages, d.Hkv, d.D, d.num_pages, L,
                               c->b.err);
    const size_t s_bytes = sizeof(float) * d.nv * d.dv * d.dk, r_bytes = sizeof(float) * kConvRing * d.qkv_dim;
    if (e == cudaSuccess && d.n_gdn > 0)
        e = cudaMemcpy2DAsync(reinterpret_cast<uint8_t*>(c->b.S) + dst * s_bytes, d.max_seqs * s_bytes,
                              reinterpret_cast<uint8_t*>(c->b.S) + src * s_bytes, d.max_seqs * s_bytes, s_bytes, d.n_gdn,
                              cudaMemcpyDeviceToDevice, c->stream);
    if (e == cudaSuccess && d.n_gdn > 0)
        e = cudaMemcpy2DAsync(reinterpret_cast<uint8_t*>(c->b.ring) + dst * r_bytes, d.max_seqs * r_bytes,
                              reinterpret_cast<uint8_t*>(c->b.ring) + src * r_bytes, d.max_seqs * r_bytes, r_bytes, d.n_gdn,
                              cudaMemcpyDeviceToDevice, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(c->b.token + dst, c->b.token + src, 4, cudaMemcpyDeviceToDevice, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "seq_copy", -1, "%s", cudaGetErrorString(e));
    if ((rc = check_device_error(c, "seq_copy")) != DM_OK) return rc;
    c->slot_len[dst] = L;
    for (int a = 0; a < d.n_att; ++a) c->att_len[static_cast<size_t>(a) * d.max_seqs + dst] = L;
    c->dev_pos_valid[dst] = 0;
    return DM_OK;
}

// ---- GDN conv-window sidecar of a session file -----------------------------------------
// KMSS v1 carries the recurrent states but not the causal-conv window (the last 3 pre-conv
// projections of every GDN layer), so a resumed full-shape sequence would start from a zero
// window.  The sidecar holds that window, bound to one KMSS file by its SHA-256 trailer:
//   "KMCV" | u32 version 1 | u32 gdn layers | u32 qkv_dim | u32 sequence length |
//   32-byte trailer of the KMSS file | fp32 [layers][3][qkv_dim] | SHA-256 of all the above
static bool read_file(const char* path, std::vector<uint8_t>* out) {
    FILE* f = fopen(path, "rb");
    if (!f) return false;
    fseek(f, 0, SEEK_END);
    const long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    out->resize(n > 0 ? static_cast<size_t>(n) : 0);
    const bool ok = n >= 0 && fread(out->data(), 1, out->size(), f) == out->size();
    fclose(f);
    return ok;
}

static void push_u32(std::vector<uint8_t>& b, uint32_t v) {
    for (int i = 0; i < 4; ++i) b.push_back(static_cast<uint8_t>(v >> (8 * i)));
}

int32_t dm_kmss_save_conv(dm_ctx* c, int32_t slot, const char* kmss_path, const char* conv_path) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    if (!kmss_path || !conv_path) return DM_ERR_INVALID_ARG;
    std::vector<uint8_t> kmss;
    if (!read_file(kmss_path, &kmss) || kmss.size() < 32)
        return set_err(c, DM_ERR_IO, "SESSION_NOT_FOUND", "session", -1, "session file not found: %s", kmss_path);
    const Dims& d = c->d;
    std::vector<uint8_t> b;
    b.insert(b.end(), {'K', 'M', 'C', 'V'});
    push_u32(b, 1);
    push_u32(b, static_cast<uint32_t>(d.n_gdn));
    push_u32(b, static_cast<uint32_t>(d.qkv_dim));
    push_u32(b, static_cast<uint32_t>(c->slot_len[slot]));
    b.insert(b.end(), kmss.end() - 32, kmss.end());
    std::vector<float> conv(static_cast<size_t>(3) * d.qkv_dim);
    for (int g = 0; g < d.n_gdn; ++g) {
        if ((rc = dm_gdn_state_export(c, g, slot, nullptr, conv.data())) != DM_OK) return rc;
        const uint8_t* p = reinterpret_cast<const uint8_t*>(conv.data());
        b.insert(b.end(), p, p + conv.size() * 4);
    }
    uint8_t digest[32];
    const uint8_t* parts[1] = {b.data()};
    const size_t sizes[1] = {b.size()};
    dm::sha256_parts(parts, sizes, 1, digest);
    b.insert(b.end(), digest, digest + 32);
    FILE* f = fopen(conv_path, "wb");
    if (!f) return set_err(c, DM_ERR_IO, "IO_ERROR", "session", -1, "cannot write %s", conv_path);
    const bool ok = fwrite(b.data(), 1, b.size(), f) == b.size();
    fclose(f);
    return ok ? DM_OK : set_err(c, DM_ERR_IO, "IO_ERROR", "session", -1, "short write to %s", conv_path);
}

int32_t dm_kmss_load_conv(dm_ctx* c, int32_t slot, const char* kmss_path, const char* conv_path) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    if (!kmss_path || !conv_path) return DM_ERR_INVALID_ARG;
    const Dims& d = c->d;
    std::vector<uint8_t> kmss, b;
    if (!read_file(kmss_path, &kmss) || kmss.size() < 32)
        return set_err(c, DM_ERR_IO, "SESSION_NOT_FOUND", "session", -1, "session file not found: %s", kmss_path);
    if (!read_file(conv_path, &b))
        return set_err(c, DM_ERR_IO, "SESSION_NOT_FOUND", "session", -1, "conv-window file not found: %s", conv_path);
    const size_t body = static_cast<size_t>(d.n_gdn) * 3 * d.qkv_dim * 4;
    auto fail = [&](const char* type, const char* what) {
        return set_err(c, DM_ERR_FORMAT, type, "session", -1, "%s", what);
    };
    if (b.size() != 52 + body + 32) return fail("LAYOUT_MISMATCH", "conv-window file size does not match the model");
    if (memcmp(b.data(), "KMCV", 4) != 0) return fail("FORMAT_MISMATCH", "invalid conv-window magic bytes");
    auto u32 = [&](size_t o) { return b[o] | (b[o + 1] << 8) | (b[o + 2] << 16) | (static_cast<uint32_t>(b[o + 3]) << 24); };
    if (u32(4) != 1) return fail("VERSION_MISMATCH", "unsupported conv-window version");
    if (u32(8) != static_cast<uint32_t>(d.n_gdn) || u32(12) != static_cast<uint32_t>(d.qkv_dim))
        return fail("CONFIG_MISMATCH", "conv-window dimensions do not match the model of this context");
    uint8_t digest[32];
    const uint8_t* parts[1] = {b.data()};
    const size_t sizes[1] = {52 + body};
    dm::sha256_parts(parts, sizes, 1, digest);
    if (memcmp(digest, b.data() + 52 + body, 32) != 0) return fail("CORRUPT_SESSION_CHECKSUM", "checksum mismatch in conv-window file");
    if (memcmp(b.data() + 20, kmss.data() + kmss.size() - 32, 32) != 0)
        return fail("SESSION_MISMATCH", "conv-window file belongs to another session file");
    if (u32(16) != static_cast<uint32_t>(c->slot_len[slot]))
        return fail("SESSION_MISMATCH", "conv-window sequence length differs from the slot's");
    for (int g = 0; g < d.n_gdn; ++g) {
        const float* conv = reinterpret_cast<const float*>(b.data() + 52 + static_cast<size_t>(g) * 3 * d.qkv_dim * 4);
        std::vector<float> tmp(conv, conv + static_cast<size_t>(3) * d.qkv_dim);  // aligned copy
        if ((rc = dm_gdn_state_import_conv(c, g, slot, tmp.data())) != DM_OK) return rc;
    }
    return DM_OK;
}

int32_t dm_kmss_save(dm_ctx* c, int32_t slot, const char* path, const int32_t* tokens, int32_t n_tokens,
                     int32_t kv_dtype, const uint8_t* manifest_hash32) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    if (!path || n_tokens < 0 || (n_tokens > 0 && !tokens) || (kv_dtype != 1 && kv_dtype != 2))
        return set_err(c, DM_ERR_INVALID_ARG, "M5_ERR_INPUT", "session", -1, "invalid session arguments");
    const Dims& d = c->d;
    const int len = c->slot_len[slot];
    for (int a = 0; a < d.n_att; ++a)
        if (c->att_len[static_cast<size_t>(a) * d.max_seqs + slot] != len)
            return set_err(c, DM_ERR_POSITION, "M5_ERR_DECODE", "session", -1, "attention layer %d not at the slot length", a);
    const int seq = std::max(len, static_cast<int>(n_tokens));
    const int b_kv = kv_dtype == 1 ? 4 : 2;
    const size_t row = static_cast<size_t>(d.Hkv) * d.D;  // one position of one layer
    const uint64_t kv_bytes = 2ull * seq * d.n_att * row * b_kv;
    const uint64_t gdn_dv = static_cast<uint64_t>(d.nv) * d.dv;
    const uint64_t gdn_bytes = static_cast<uint64_t>(d.n_gdn) * gdn_dv * d.dk * 4;
    const uint64_t tok_bytes = static_cast<uint64_t>(seq) * 4;
    uint8_t hdr[128] = {0};
    memcpy(hdr, "KMSS", 4);
    put_u32(hdr + 4, 1);
    put_u32(hdr + 8, 2);
    if (manifest_hash32) memcpy(hdr + 12, manifest_hash32, 32);
    put_u32(hdr + 44, seq);
    put_u32(hdr + 48, d.V);
    put_u32(hdr + 52, d.n_att);
    put_u32(hdr + 56, d.Hkv);
    put_u32(hdr + 60, d.D);
    put_u32(hdr + 64, kv_dtype);
    put_u32(hdr + 68, d.n_gdn);
    put_u32(hdr + 72, static_cast<uint32_t>(gdn_dv));
    put_u32(hdr + 76, d.dk);
    put_u32(hdr + 80, 1);
    put_u64(hdr + 84, kv_bytes);
    put_u64(hdr + 92, gdn_bytes);
    put_u64(hdr + 100, tok_bytes);
    // KV: per attention layer the slot's len positions; positions >= len stay zero
    std::vector<uint8_t> kv(kv_bytes, 0);
    std::vector<uint16_t> kb(static_cast<size_t>(len) * row), vb(kb.size());
    for (int a = 0; a < d.n_att && len > 0; ++a) {
        if ((rc = dm_kv_export(c, a, slot, kb.data(), vb.data(), len)) != DM_OK) return rc;
        for (int kvi = 0; kvi < 2; ++kvi) {
            const uint16_t* src = kvi == 0 ? kb.data() : vb.data();
            for (int p = 0; p < len; ++p) {
                const size_t e0 = ((static_cast<size_t>(kvi) * seq + p) * d.n_att + a) * row;
                for (size_t i = 0; i < row; ++i) {
                    const uint16_t h = src[static_cast<size_t>(p) * row + i];
                    if (kv_dtype == 2) {
                        memcpy(kv.data() + (e0 + i) * 2, &h, 2);
                    } else {
                        const float f = bf16_bits_to_f32(h);
                        memcpy(kv.data() + (e0 + i) * 4, &f, 4);
                    }
                }
            }
        }
    }
    std::vector<uint8_t> gdn(gdn_bytes);
    for (int g = 0; g < d.n_gdn; ++g)
        if ((rc = dm_gdn_state_export(c, g, slot, reinterpret_cast<float*>(gdn.data() + static_cast<size_t>(g) * gdn_dv * d.dk * 4),
                                      nullptr)) != DM_OK)
            return rc;
    std::vector<uint8_t> tok(tok_bytes, 0);
    for (int i = 0; i < seq; ++i) put_u32(tok.data() + 4 * i, i < n_tokens ? static_cast<uint32_t>(tokens[i]) : 0u);
    uint8_t digest[32];
    const uint8_t* parts[4] = {hdr, kv.data(), gdn.data(), tok.data()};
    const size_t sizes[4] = {128, kv.size(), gdn.size(), tok.size()};
    dm::sha256_parts(parts, sizes, 4, digest);
    const std::string tmp = std::string(path) + ".tmp";
    FILE* f = fopen(tmp.c_str(), "wb");
    if (!f) return set_err(c, DM_ERR_IO, "OUTPUT_WRITE_FAILED", "session", -1, "cannot write temp KMSS file: %s", tmp.c_str());
    bool ok = true;
    for (int i = 0; i < 4; ++i) ok = ok && (sizes[i] == 0 || fwrite(parts[i], 1, sizes[i], f) == sizes[i]);
    ok = ok && fwrite(digest, 1, 32, f) == 32;
    ok = (fclose(f) == 0) && ok;
    if (!ok) return set_err(c, DM_ERR_IO, "OUTPUT_WRITE_FAILED", "session", -1, "cannot write temp KMSS file: %s", tmp.c_str());
    if (rename(tmp.c_str(), path) != 0)
        return set_err(c, DM_ERR_IO, "OUTPUT_WRITE_FAILED", "session", -1, "atomic rename failed for KMSS: %s", path);
    return DM_OK;
}

int32_t dm_kmss_load(dm_ctx* c, int32_t slot, const char* path, int32_t* tokens_out, int32_t cap, int32_t* n_tokens) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    if (!path || cap < 0 || (cap > 0 && !tokens_out))
        return set_err(c, DM_ERR_INVALID_ARG, "M5_ERR_INPUT", "session", -1, "invalid session arguments");
    const Dims& d = c->d;
    FILE* f = fopen(path, "rb");
    if (!f) return set_err(c, DM_ERR_IO, "SESSION_NOT_FOUND", "session", -1, "session file not found: %s", path);
    fseek(f, 0, SEEK_END);
    const long total = ftell(f);
    fseek(f, 0, SEEK_SET);
    std::vector<uint8_t> all(total > 0 ? static_cast<size_t>(total) : 0);
    const bool read_ok = total >= 0 && fread(all.data(), 1, all.size(), f) == all.size();
    fclose(f);
    auto fail = [&](const char* type, const char* what) {
        return set_err(c, DM_ERR_FORMAT, type, "session", -1, "%s", what);
    };
    if (!read_ok || all.size() < 160) return fail("CORRUPT_SESSION_CHECKSUM", "file too small for KMSS v1");
    const uint8_t* h = all.data();
    if (memcmp(h, "KMSS", 4) != 0) return fail("FORMAT_MISMATCH", "invalid KMSS magic bytes");
    if (get_u32(h + 4) != 1) return fail("VERSION_MISMATCH", "unsupported KMSS version");
    if (get_u32(h + 8) != 2) return fail("CONFIG_MISMATCH", "unsupported KMSS architecture_id, expected 2");
    const uint64_t seq = get_u32(h + 44), kv_layers = get_u32(h + 52), kv_heads = get_u32(h + 56),
                   head_dim = get_u32(h + 60), kv_dtype = get_u32(h + 64), gdn_layers = get_u32(h + 68),
                   gdn_dv = get_u32(h + 72), gdn_dk = get_u32(h + 76);
    const uint64_t kv_bytes = get_u64(h + 84), gdn_bytes = get_u64(h + 92), tok_bytes = get_u64(h + 100);
    const uint64_t b_kv = kv_dtype == 1 ? 4 : 2;
    if (kv_bytes != 2 * seq * kv_layers * kv_heads * head_dim * b_kv) return fail("LAYOUT_MISMATCH", "header kv_bytes mismatch dimensions");
    if (gdn_bytes != gdn_layers * gdn_dv * gdn_dk * 4) return fail("LAYOUT_MISMATCH", "header gdn_bytes mismatch dimensions");
    if (tok_bytes != seq * 4) return fail("LAYOUT_MISMATCH", "header token_bytes mismatch dimensions");
    if (all.size() != 128 + kv_bytes + gdn_bytes + tok_bytes + 32)
        return fail("LAYOUT_MISMATCH", "total file size mismatch expected 160 + payload");
    uint8_t digest[32];
    const uint8_t* parts[1] = {all.data()};
    const size_t sizes[1] = {static_cast<size_t>(128 + kv_bytes + gdn_bytes + tok_bytes)};
    dm::sha256_parts(parts, sizes, 1, digest);
    if (memcmp(digest, all.data() + sizes[0], 32) != 0) return fail("CORRUPT_SESSION_CHECKSUM", "checksum mismatch in KMSS file");
    // this context's model
    if (kv_layers != static_cast<uint64_t>(d.n_att) || kv_heads != static_cast<uint64_t>(d.Hkv) ||
        head_dim != static_cast<uint64_t>(d.D) || gdn_layers != static_cast<uint64_t>(d.n_gdn) ||
        gdn_dv != static_cast<uint64_t>(d.nv) * d.dv || gdn_dk != static_cast<uint64_t>(d.dk) ||
        (kv_dtype != 1 && kv_dtype != 2))
        return fail("CONFIG_MISMATCH", "KMSS dimensions do not match the model of this context");
    if (seq > static_cast<uint64_t>(d.max_pages) * kPageTokens)
        return set_err(c, DM_ERR_CAPACITY, "M5_ERR_CONTEXT_SIZE", "session", -1, "session of %llu tokens exceeds the slot capacity",
                       static_cast<unsigned long long>(seq));
    const uint8_t* kvp = all.data() + 128;
    const uint8_t* gdp = kvp + kv_bytes;
    const uint8_t* tkp = gdp + gdn_bytes;
    if ((rc = dm_seq_reset(c, slot)) != DM_OK) return rc;
    const size_t row = static_cast<size_t>(d.Hkv) * d.D;
    std::vector<uint16_t> kb(seq * row), vb(seq * row);
    for (int a = 0; a < d.n_att && seq > 0; ++a) {
        for (int kvi = 0; kvi < 2; ++kvi) {
            uint16_t* dst = kvi == 0 ? kb.data() : vb.data();
            for (uint64_t p = 0; p < seq; ++p) {
                const size_t e0 = ((static_cast<size_t>(kvi) * seq + p) * d.n_att + a) * row;
                for (size_t i = 0; i < row; ++i) {
                    uint16_t hb;
                    if (kv_dtype == 2) {
                        memcpy(&hb, kvp + (e0 + i) * 2, 2);
                    } else {
                        float fv;
                        memcpy(&fv, kvp + (e0 + i) * 4, 4);
                        hb = f32_to_bf16_rne(fv);  // the cache's single rounding to bf16
                    }
                    dst[p * row + i] = hb;
                }
            }
        }
        if ((rc = dm_kv_import(c, a, slot, kb.data(), vb.data(), static_cast<int32_t>(seq))) != DM_OK) return rc;
    }
    c->slot_len[slot] = static_cast<int>(seq);
    c->dev_pos_valid[slot] = 0;
    std::vector<float> S(static_cast<size_t>(gdn_dv) * gdn_dk);
    for (int g = 0; g < d.n_gdn; ++g) {
        memcpy(S.data(), gdp + static_cast<size_t>(g) * S.size() * 4, S.size() * 4);
        if ((rc = dm_gdn_state_import(c, g, slot, S.data(), nullptr)) != DM_OK) return rc;  // conv window: zero
    }
    for (uint64_t i = 0; i < seq && static_cast<int64_t>(i) < cap; ++i) tokens_out[i] = static_cast<int32_t>(get_u32(tkp + 4 * i));
    if (n_tokens) *n_tokens = static_cast<int32_t>(seq);
    return DM_OK;
}

// ---- compute ------------------------------------------------------------------------
static cudaError_t enqueue_mixer(dm_ctx* c, int layer, int slot) {
    const LayerW& w = c->layers[layer];
    cudaError_t e;
    if (w.is_attn) {
        if ((e = launch_attn_in(lcfg_traced(c, TK_ATTN_IN, layer), c->d, w, c->b, slot)) != cudaSuccess) return e;
        if ((e = launch_attn_decode(lcfg_traced(c, TK_ATTN, layer), c->d, w, c->b, slot)) != cudaSuccess) return e;
        return launch_attn_out(lcfg_traced(c, TK_ATTN_OUT, layer), c->d, w, c->b, slot);
    }
    if ((e = launch_gdn_in(lcfg_traced(c, TK_GDN_IN, layer), c->d, w, c->b, slot)) != cudaSuccess) return e;
    if (gdn_fused_on(c)) return launch_gdn_core_out(lcfg_traced(c, TK_GDN_CORE_OUT, layer), c->d, w, c->b, slot);
    if ((e = launch_gdn_rec(lcfg_traced(c, TK_GDN_REC, layer), c->d, w, c->b, slot)) != cudaSuccess) return e;
    return launch_gdn_out(lcfg_traced(c, TK_GDN_OUT, layer), c->d, w, c->b, slot);
}

// The MoE kernel prefetches into L2 the weights of the kernel after it: the next layer's
// input projection, or (after the last layer) the head's first rows, as much of it as the
// L2 can keep beside the step's other traffic.
static cudaError_t enqueue_moe(dm_ctx* c, int layer, int slot) {
    const LayerW& w = c->layers[layer];
    const Dims& d = c->d;
    const void* next = nullptr;
    uint64_t bytes = 0;
    if (layer + 1 < d.L) {
        const LayerW& n = c->layers[layer + 1];
        next = n.w_in;
        bytes = static_cast<uint64_t>(n.is_attn ? d.attn_in_rows : d.gdn_in_rows) * d.H * 2;
    } else {
        next = c->lm_head;
        bytes = std::min<uint64_t>(static_cast<uint64_t>(d.V) * d.H * 2, 48ull << 20);
    }
    return launch_moe_fused(lcfg_traced(c, TK_MOE, layer), d, w, c->b, slot, next, bytes);
}

static cudaError_t enqueue_step(dm_ctx* c, int slot) {
    c->trace_n = 0;
    c->trace_kinds.clear();
    cudaError_t e = launch_embed(lcfg_traced(c, TK_EMBED, 0), c->d, c->embed, c->b, slot);
    for (int l = 0; l < c->d.L && e == cudaSuccess; ++l) {
        e = enqueue_mixer(c, l, slot);
        if (e == cudaSuccess) e = enqueue_moe(c, l, slot);
    }
    if (e == cudaSuccess)
        e = launch_head(lcfg_traced(c, TK_HEAD, c->d.L), c->d, c->final_norm, c->lm_head, c->b, slot, 1, 1);
    return e;
}

static int ensure_graph(dm_ctx* c, int slot) {
    if (c->graphs[slot]) return DM_OK;
    cudaGraph_t g = nullptr;
    DM_CUDA(c, cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "decode");
    cudaError_t e = enqueue_step(c, slot);
    cudaError_t e2 = cudaStreamEndCapture(c->stream, &g);
    if (e != cudaSuccess || e2 != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "decode", -1, "graph capture failed: %s",
                       cudaGetErrorString(e != cudaSuccess ? e : e2));
    }
    cudaGraphExec_t ge = nullptr;
    e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "decode", -1, "graph instantiate: %s", cudaGetErrorString(e));
    c->graphs[slot] = ge;
    return DM_OK;
}

// Decode-step preconditions: weights present, every attention layer at the slot length,
// room for the new tokens, device position in sync.
static int prepare_decode(dm_ctx* c, int slot, int n_steps) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    const Dims& d = c->d;
    for (int a = 0; a < d.n_att; ++a) {
        const int al = c->att_len[static_cast<size_t>(a) * d.max_seqs + slot];
        if (al != c->slot_len[slot])
            return set_err(c, DM_ERR_POSITION, "M5_ERR_DECODE", "decode", -1,
                           "Position mismatch on KV append: expected current_len %d, actual_pos %d (attention layer %d)",
                           al, c->slot_len[slot], a);
    }
    if (c->slot_len[slot] + n_steps > d.max_pages * kPageTokens)
        return set_err(c, DM_ERR_CAPACITY, "M5_ERR_CONTEXT_SIZE", "kv_alloc", -1,
                       "KV cache capacity exceeded on token append: current_len %d + %d > capacity %d",
                       c->slot_len[slot], n_steps, d.max_pages * kPageTokens);
    cudaSetDevice(c->device);
    if (!c->dev_pos_valid[slot]) {
        c->h_io[3] = c->slot_len[slot];
        DM_CUDA(c, cudaMemcpyAsync(c->b.pos + slot, &c->h_io[3], 4, cudaMemcpyHostToDevice, c->stream), "decode");
        DM_CUDA(c, cudaStreamSynchronize(c->stream), "decode");
        c->dev_pos_valid[slot] = 1;
    }
    return ensure_graph(c, slot);
}

static void advance_lens(dm_ctx* c, int slot, int n) {
    c->slot_len[slot] += n;
    for (int a = 0; a < c->d.n_att; ++a) c->att_len[static_cast<size_t>(a) * c->d.max_seqs + slot] += n;
}

int32_t dm_set_token(dm_ctx* c, int32_t slot, int32_t token) {
    int rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    if (token < 0 || token >= c->d.V)
        return set_err(c, DM_ERR_INVALID_ARG, "M4_ERR_INPUT", "input", -1, "token %d out of range [0, %d)", token, c->d.V);
    cudaSetDevice(c->device);
    c->h_io[0] = token;
    DM_CUDA(c, cudaMemcpyAsync(c->b.token + slot, &c->h_io[0], 4, cudaMemcpyHostToDevice, c->stream), "input");
    return DM_OK;
}

static bool spilling(const dm_ctx* c);
static int spill_reject(dm_ctx* c, const char* what);
static int spill_decode(dm_ctx* c, const int32_t* slots, const int32_t* tokens, int n, int n_steps,
                        int32_t* tokens_out, float* logits);

int32_t dm_enqueue_decode(dm_ctx* c, int32_t slot, int32_t n_steps) {
    if (n_steps < 0) return DM_ERR_INVALID_ARG;
    if (c && spilling(c)) return spill_reject(c, "dm_enqueue_decode");
    int rc = prepare_decode(c, slot, n_steps);
    if (rc != DM_OK) return rc;
    for (int i = 0; i < n_steps; ++i) DM_CUDA(c, cudaGraphLaunch(c->graphs[slot], c->stream), "decode");
    advance_lens(c, slot, n_steps);
    return DM_OK;
}

int32_t dm_sync(dm_ctx* c) {
    if (!c) return DM_ERR_INVALID_ARG;
    cudaSetDevice(c->device);
    return check_device_error(c, "decode");
}

int32_t dm_decode_step(dm_ctx* c, int32_t slot, int32_t token_in, int32_t* token_out, float* logits) {
    // a spilling pool decodes through the batched step (one row)
    if (c && spilling(c)) return spill_decode(c, &slot, &token_in, 1, 1, token_out, logits);
    int rc = prepare_decode(c, slot, 1);
    if (rc != DM_OK) return rc;
    if ((rc = dm_set_token(c, slot, token_in)) != DM_OK) return rc;
    DM_CUDA(c, cudaGraphLaunch(c->graphs[slot], c->stream), "decode");
    DM_CUDA(c, cudaMemcpyAsync(&c->h_io[1], c->b.token + slot, 4, cudaMemcpyDeviceToHost, c->stream), "decode");
    DM_CUDA(c, cudaMemcpyAsync(&c->h_io[2], c->b.err, 4, cudaMemcpyDeviceToHost, c->stream), "decode");
    if (logits)
        DM_CUDA(c, cudaMemcpyAsync(logits, c->b.logits, sizeof(float) * c->d.V, cudaMemcpyDeviceToHost, c->stream), "decode");
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "decode");
    advance_lens(c, slot, 1);
    if (c->h_io[2] != 0) return check_device_error(c, "decode");
    if (token_out) *token_out = c->h_io[1];
    return DM_OK;
}

int32_t dm_generate(dm_ctx* c, int32_t slot, int32_t token_in, int32_t n_steps, int32_t* out) {
    if (!c || !out || n_steps <= 0 || n_steps > c->b.gen_capacity) return DM_ERR_INVALID_ARG;
    if (spilling(c)) return dm_generate_batch(c, &slot, &token_in, 1, n_steps, out);
    int rc = prepare_decode(c, slot, n_steps);
    if (rc != DM_OK) return rc;
    if ((rc = dm_set_token(c, slot, token_in)) != DM_OK) return rc;
    DM_CUDA(c, cudaMemsetAsync(c->b.gen_idx, 0, 4, c->stream), "decode");
    for (int i = 0; i < n_steps; ++i) DM_CUDA(c, cudaGraphLaunch(c->graphs[slot], c->stream), "decode");
    DM_CUDA(c, cudaMemcpyAsync(out, c->b.gen_out, sizeof(int) * n_steps, cudaMemcpyDeviceToHost, c->stream), "decode");
    advance_lens(c, slot, n_steps);
    return check_device_error(c, "decode");
}

int32_t dm_forward(dm_ctx* c, int32_t slot, const int32_t* tokens, int32_t n, float* logits, int32_t* next) {
    if (!c || !tokens || n <= 0) return DM_ERR_INVALID_ARG;
    if (spilling(c)) {  // one batched step per prompt token
        int32_t nx = 0;
        for (int i = 0; i < n; ++i) {
            const int rc = spill_decode(c, &slot, tokens + i, 1, 1, &nx, i == n - 1 ? logits : nullptr);
            if (rc != DM_OK) return rc;
        }
        if (next) *next = nx;
        return DM_OK;
    }
    int rc = prepare_decode(c, slot, n);
    if (rc != DM_OK) return rc;
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= c->d.V)
            return set_err(c, DM_ERR_INVALID_ARG, "M4_ERR_INPUT", "input", -1, "token %d at index %d out of range [0, %d)",
                           tokens[i], i, c->d.V);
    // stage the prompt on the device, copy one id per step into the slot's token
    if (n > c->b.gen_capacity) return DM_ERR_INVALID_ARG;
    cudaError_t e = cudaMemcpyAsync(c->b.prompt, tokens, sizeof(int) * n, cudaMemcpyHostToDevice, c->stream);
    for (int i = 0; i < n && e == cudaSuccess; ++i) {
        e = cudaMemcpyAsync(c->b.token + slot, c->b.prompt + i, 4, cudaMemcpyDeviceToDevice, c->stream);
        if (e == cudaSuccess) e = cudaGraphLaunch(c->graphs[slot], c->stream);
    }
    if (e == cudaSuccess && logits) e = cudaMemcpyAsync(logits, c->b.logits, sizeof(float) * c->d.V, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&c->h_io[1], c->b.token + slot, 4, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "decode", -1, "%s", cudaGetErrorString(e));
    advance_lens(c, slot, n);
    rc = check_device_error(c, "decode");
    if (rc == DM_OK && next) *next = c->h_io[1];
    return rc;
}

static cudaError_t enqueue_pf_chunk(dm_ctx* c, int slot, int pos0, int n, bool head, int write_logits);
static int pf_kernels_per_chunk(const Dims& d);

int32_t dm_prefill(dm_ctx* c, int32_t slot, const int32_t* tokens, int32_t n, float* logits, int32_t* next) {
    if (!c || !tokens || n <= 0) return DM_ERR_INVALID_ARG;
    if (spilling(c)) return spill_reject(c, "dm_prefill");
    if (!pf_gdn_supported(c->d))
        return set_err(c, DM_ERR_INVALID_ARG, "PREFILL_UNSUPPORTED", "prefill", -1,
                       "GDN head dimension %d has no prefill kernel (64 or 128)", c->d.dk);
    int rc = prepare_decode(c, slot, n);
    if (rc != DM_OK) return rc;
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= c->d.V)
            return set_err(c, DM_ERR_INVALID_ARG, "M4_ERR_INPUT", "input", -1, "token %d at index %d out of range [0, %d)",
                           tokens[i], i, c->d.V);
    const int R = c->pb.cap;
    const int pos_start = c->slot_len[slot];
    c->h_io[4] = slot;
    c->h_io[5] = pos_start + n;
    cudaError_t e = cudaMemcpyAsync(c->pb.slots, &c->h_io[4], 4, cudaMemcpyHostToDevice, c->stream);
    for (int t0 = 0; t0 < n && e == cudaSuccess; t0 += R) {
        const int m = std::min(R, n - t0);
        e = cudaMemcpyAsync(c->pb.tok, tokens + t0, sizeof(int) * m, cudaMemcpyHostToDevice, c->stream);
        if (e == cudaSuccess) e = enqueue_pf_chunk(c, slot, pos_start + t0, m, t0 + m == n, logits != nullptr);
    }
    // the device position after the prompt (the decode kernels read it)
    if (e == cudaSuccess) e = cudaMemcpyAsync(c->b.pos + slot, &c->h_io[5], 4, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess && logits)
        e = cudaMemcpyAsync(logits, c->pb.head_logits, sizeof(float) * c->d.V, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&c->h_io[1], c->b.token + slot, 4, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "prefill", -1, "%s", cudaGetErrorString(e));
    advance_lens(c, slot, n);
    rc = check_device_error(c, "prefill");
    if (rc == DM_OK && next) *next = c->h_io[1];
    return rc;
}

int32_t dm_prefill_rows(dm_ctx* c, int32_t* rows_out, int32_t* kernels_per_chunk_out) {
    if (!c || !rows_out) return DM_ERR_INVALID_ARG;
    *rows_out = c->pb.cap;
    if (kernels_per_chunk_out) *kernels_per_chunk_out = pf_kernels_per_chunk(c->d);
    return DM_OK;
}

// ---- batched decode ---------------------------------------------------------------------
// One step of n sequences (rows): dense projections on the tensor cores (dm_gemm_tc.cu:
// weights streamed once per step, the rows' hi/lo operand as the MMA's N), the per-row
// kernels of dm_batch.cu, the GDN recurrence and the attention with a row dimension, the
// experts on the tensor cores (dm_expert_tc.cu).
// C = Xcat . W^T for dense matrix `map` ([N][K]) into bb.c as *splits partials (bb: the
// decode step's or the prefill chunk's scratch).
static cudaError_t bgemm(dm_ctx* c, const BatchBuffers& bb, int map, int N, int K, int n, int* splits,
                         int max_splits = 16) {
    CUtensorMap xm;
    if (!encode_operand_map(bb, K, 2 * n, &xm)) return cudaErrorInvalidValue;
    // the partials share the result buffer: S x 2n x N <= c_cap
    const int max_s = static_cast<int>(std::min<size_t>(max_splits, bb.c_cap / (2 * static_cast<size_t>(n) * N)));
    if (max_s < 1) return cudaErrorInvalidValue;
    *splits = tc_gemm_splits(((N + 127) / 128) * ((2 * n + 127) / 128), K, c->num_sms, max_s);
    return launch_tc_gemm(lcfg(c), &c->dmaps[map], &xm, bb.c, N, K, 2 * n, *splits, c->b.err);
}

// The token mixer of layer l for n rows, through its residual: x -> xm.
static cudaError_t enqueue_b_mixer(dm_ctx* c, int l, int n) {
    const Dims& d = c->d;
    BatchBuffers& bb = c->bb;
    const LaunchCfg lc = lcfg(c);
    const LayerW& w = c->layers[l];
    cudaError_t e = cudaSuccess;
    int sp = 1;
    if (w.is_attn) {
        if (e == cudaSuccess) e = launch_b_prep(lc, BPREP_RMS, bb.x, d.H, w.in_norm, d.eps, nullptr, nullptr, 0, bb.xcat, n);
        if (e == cudaSuccess) e = bgemm(c, bb, 2 * l, d.attn_in_rows, d.H, n, &sp);
        if (e == cudaSuccess) e = launch_b_epi_attn_in(lc, d, bb, n, sp);
        if (e == cudaSuccess) e = launch_attn_decode_batch(lc, d, w, bb, c->b, n);
        if (e == cudaSuccess) e = launch_attn_merge_batch(lc, d, bb, n);
        if (e == cudaSuccess) e = bgemm(c, bb, 2 * l + 1, d.H, d.Hq * d.D, n, &sp);
    } else {
        if (e == cudaSuccess) e = launch_b_prep(lc, BPREP_RMS, bb.x, d.H, w.in_norm, d.eps, nullptr, nullptr, 0, bb.xcat, n);
        if (e == cudaSuccess) e = bgemm(c, bb, 2 * l, d.gdn_in_rows, d.H, n, &sp);
        if (e == cudaSuccess) e = launch_b_epi_gdn_in(lc, d, w, bb, c->b, n, sp);
        if (e == cudaSuccess) e = launch_gdn_rec_batch(lc, d, w, bb, c->b, n);
        if (e == cudaSuccess)
            e = launch_b_prep(lc, BPREP_HEADNORM, bb.o, d.z_dim, nullptr, d.eps, bb.z, w.gdn_norm, d.dv, bb.xcat, n);
        if (e == cudaSuccess) e = bgemm(c, bb, 2 * l + 1, d.H, d.z_dim, n, &sp);
    }
    if (e == cudaSuccess) e = launch_b_epi_resid(lc, bb.c, d.H, bb.x, bb.xm, n, sp);
    return e;
}

// The MoE of layer l after its router: top-k + grouping, experts, weighted combine +
// residual (xm -> x).  slot_of: the layer's slot table when the pool spills.
static cudaError_t enqueue_b_moe_tail(dm_ctx* c, int l, int n, const int* slot_of) {
    const Dims& d = c->d;
    BatchBuffers& bb = c->bb;
    const LaunchCfg lc = lcfg(c);
    cudaError_t e = launch_b_topk_group(lc, d, bb, c->b, n, slot_of);
    if (e == cudaSuccess) e = launch_b_experts(lc, d, c->layers[l], bb, c->b, n);
    if (e == cudaSuccess && bb.ep.world > 1) e = launch_ep_barrier(lc, bb, c->b, 1);
    if (e == cudaSuccess) e = launch_b_combine(lc, d, bb, bb.xm, bb.x, n);
    return e;
}

static cudaError_t enqueue_b_head(dm_ctx* c, int n, int write_logits) {
    const Dims& d = c->d;
    BatchBuffers& bb = c->bb;
    const LaunchCfg lc = lcfg(c);
    cudaError_t e = launch_b_prep(lc, BPREP_RMS, bb.x, d.H, c->final_norm, d.eps, nullptr, nullptr, 0, bb.xcat, n);
    int sp = 1;
    if (e == cudaSuccess) e = bgemm(c, bb, 2 * d.L, d.V, d.H, n, &sp, 1);
    if (e == cudaSuccess && sp != 1) e = cudaErrorInvalidValue;  // the argmax reads one product
    if (e == cudaSuccess) e = launch_b_argmax(lc, d, bb, c->b, n, write_logits, 1);
    return e;
}

static cudaError_t enqueue_batch_step(dm_ctx* c, int n, int write_logits) {
    const Dims& d = c->d;
    BatchBuffers& bb = c->bb;
    const LaunchCfg lc = lcfg(c);
    cudaError_t e = launch_b_embed(lc, d, c->embed, bb, c->b, n);
    for (int l = 0; l < d.L && e == cudaSuccess; ++l) {
        e = enqueue_b_mixer(c, l, n);
        // MoE: canonical router, top-k + grouping, experts, weighted combine + residual
        if (e == cudaSuccess) e = launch_b_router(lc, d, c->layers[l], bb, bb.xm, 1, n);
        if (e == cudaSuccess) e = enqueue_b_moe_tail(c, l, n, nullptr);
    }
    if (e == cudaSuccess) e = enqueue_b_head(c, n, write_logits);
    return e;
}

// ---- prefill ---------------------------------------------------------------------------
// A prompt of n tokens for one slot, as chunks of up to pb.cap rows: each chunk runs the
// layers with its tokens as the rows of the batched kernels (dense projections on the
// tcgen05 GEMM, router, grouping and the tcgen05 experts), the GDN recurrence over the
// chunk's tokens (launch_pf_gdn) and the causal attention over the cache plus the chunk
// (launch_pf_attn); the final norm, lm_head and argmax run for the prompt's last token only.
static cudaError_t enqueue_pf_chunk(dm_ctx* c, int slot, int pos0, int n, bool head, int write_logits) {
    const Dims& d = c->d;
    BatchBuffers& pb = c->pb;
    const LaunchCfg lc = lcfg(c);
    cudaError_t e = launch_b_embed(lc, d, c->embed, pb, c->b, n);
    for (int l = 0; l < d.L && e == cudaSuccess; ++l) {
        const LayerW& w = c->layers[l];
        int sp = 1;
        e = launch_b_prep(lc, BPREP_RMS, pb.x, d.H, w.in_norm, d.eps, nullptr, nullptr, 0, pb.xcat, n);
        if (w.is_attn) {
            if (e == cudaSuccess) e = bgemm(c, pb, 2 * l, d.attn_in_rows, d.H, n, &sp);
            if (e == cudaSuccess) e = launch_b_epi_attn_in(lc, d, pb, n, sp);
            if (e == cudaSuccess) e = launch_pf_attn(lc, d, w, pb, c->b, slot, pos0, n);
            if (e == cudaSuccess) e = bgemm(c, pb, 2 * l + 1, d.H, d.Hq * d.D, n, &sp);
        } else {
            if (e == cudaSuccess) e = bgemm(c, pb, 2 * l, d.gdn_in_rows, d.H, n, &sp);
            if (e == cudaSuccess) e = launch_b_epi_gdn_pf(lc, d, w, pb, n, sp);
            if (e == cudaSuccess) e = launch_pf_gdn(lc, d, w, pb, c->b, slot, pos0, n);
            if (e == cudaSuccess)
                e = launch_b_prep(lc, BPREP_HEADNORM, pb.o, d.z_dim, nullptr, d.eps, pb.z, w.gdn_norm, d.dv, pb.xcat, n);
            if (e == cudaSuccess) e = bgemm(c, pb, 2 * l + 1, d.H, d.z_dim, n, &sp);
        }
        if (e == cudaSuccess) e = launch_b_epi_resid(lc, pb.c, d.H, pb.x, pb.xm, n, sp);
        if (e == cudaSuccess) e = launch_b_router(lc, d, w, pb, pb.xm, 1, n);
        if (e == cudaSuccess) e = launch_b_topk_group(lc, d, pb, c->b, n);
        if (e == cudaSuccess) e = launch_b_experts(lc, d, w, pb, c->b, n);
        if (e == cudaSuccess) e = launch_b_combine(lc, d, pb, pb.xm, pb.x, n);
    }
    if (head && e == cudaSuccess) {
        e = launch_b_prep(lc, BPREP_RMS, pb.x + static_cast<size_t>(n - 1) * d.H, d.H, c->final_norm, d.eps, nullptr,
                          nullptr, 0, pb.xcat, 1);
        int sp = 1;
        if (e == cudaSuccess) e = bgemm(c, pb, 2 * d.L, d.V, d.H, 1, &sp, 1);
        if (e == cudaSuccess && sp != 1) e = cudaErrorInvalidValue;  // the argmax reads one product
        if (e == cudaSuccess) e = launch_b_argmax(lc, d, pb, c->b, 1, write_logits, 0, 0);
    }
    return e;
}

// Kernel launches of one prefill chunk (the head excluded).
static int pf_kernels_per_chunk(const Dims& d) {
    // embed + per GDN layer 15 (prep, gemm, epi, conv, scan, ring, prep, gemm, resid,
    // router, group, xstage, 2 experts, combine) + per attention layer 13 (prep, gemm, epi, attn
    // prep, attn, merge, gemm, resid, router, group, xstage, 2 experts, combine)
    return 1 + 15 * d.n_gdn + 13 * d.n_att;
}

// ---- spilling expert pool -----------------------------------------------------------
static int prepare_batch(dm_ctx* c, const int32_t* slots, const int32_t* tokens, int n, int n_steps);
static bool spilling(const dm_ctx* c) { return c->host_pool != nullptr; }

static int spill_reject(dm_ctx* c, const char* what) {
    return set_err(c, DM_ERR_INVALID_ARG, "SPILL_UNSUPPORTED", "decode", -1,
                   "%s needs every expert resident (expert_cache_slots = 0)", what);
}

// Host -> HBM copies of the (expert, slot) loads of layer l, then the layer's slot table.
static cudaError_t spill_apply(dm_ctx* c, int l, const std::vector<std::pair<int, int>>& loads) {
    if (loads.empty()) return cudaSuccess;
    const Dims& d = c->d;
    const size_t eb = d.expert_bytes;
    uint8_t* dev = const_cast<uint8_t*>(c->layers[l].experts);
    cudaError_t e = cudaSuccess;
    for (const auto& ld : loads)
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(dev + static_cast<size_t>(ld.second) * eb,
                                c->host_pool + (static_cast<size_t>(l) * d.E + ld.first) * eb, eb, cudaMemcpyHostToDevice,
                                c->stream);
    int* row = c->h_slot_of + static_cast<size_t>(l) * d.E;
    memcpy(row, c->spill.slot_of.data() + static_cast<size_t>(l) * d.E, sizeof(int) * d.E);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(c->d_slot_of + static_cast<size_t>(l) * d.E, row, sizeof(int) * d.E, cudaMemcpyHostToDevice,
                            c->stream);
    c->spill_bytes += loads.size() * eb;
    c->spill.stats[4] += loads.size();
    return e;
}

// One batched step over a spilling pool (not captured: the host decides residency between
// each layer's router and its experts).  Per layer: mixer and router on the device, the
// routed ids back to the host, the residency policy makes the selected experts resident
// (host -> HBM on the context stream, ordered before the expert kernels), then the rest of
// the MoE.  Earlier copies of a slot table row have completed by the time the row changes
// again: every layer synchronises the stream before its residency decision.
static int spill_step(dm_ctx* c, int n, int write_logits) {
    const Dims& d = c->d;
    BatchBuffers& bb = c->bb;
    const LaunchCfg lc = lcfg(c);
    std::vector<std::pair<int, int>> loads;
    cudaError_t e = launch_b_embed(lc, d, c->embed, bb, c->b, n);
    for (int l = 0; l < d.L && e == cudaSuccess; ++l) {
        e = enqueue_b_mixer(c, l, n);
        if (e == cudaSuccess) e = launch_b_router(lc, d, c->layers[l], bb, bb.xm, 1, n);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(c->h_sids, bb.ids, sizeof(int) * n * d.topk, cudaMemcpyDeviceToHost, c->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
        if (e != cudaSuccess) break;
        for (int i = 0; i < n * d.topk; ++i)
            c->h_sids[i] = std::min(std::max(c->h_sids[i], 0), d.E - 1);
        if (!c->spill.resolve(l, c->h_sids, n * d.topk, loads))
            return set_err(c, DM_ERR_CAPACITY, "SPILL_CAPACITY", "decode", l,
                           "expert cache of %d slots cannot hold the experts of this step", d.E_res);
        e = spill_apply(c, l, loads);
        if (e == cudaSuccess) e = enqueue_b_moe_tail(c, l, n, c->d_slot_of + static_cast<size_t>(l) * d.E);
    }
    if (e == cudaSuccess) e = enqueue_b_head(c, n, write_logits);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "decode", -1, "%s", cudaGetErrorString(e));
    return DM_OK;
}

// n_steps batched steps over a spilling pool; tokens fed back on the device as in the
// captured step.  The cache must be able to hold one step's experts next to the pinned
// ones: n * top-k + pinned <= slots, checked before any work.
static int spill_decode(dm_ctx* c, const int32_t* slots, const int32_t* tokens, int n, int n_steps,
                        int32_t* tokens_out, float* logits) {
    int rc = prepare_batch(c, slots, tokens, n, n_steps);
    if (rc != DM_OK) return rc;
    const Dims& d = c->d;
    int pinned = 0;
    for (int l = 0; l < d.L; ++l) pinned = std::max(pinned, c->spill.pinned_count[l]);
    if (n * d.topk + pinned > d.E_res)
        return set_err(c, DM_ERR_CAPACITY, "SPILL_CAPACITY", "decode", -1,
                       "%d rows x top-%d experts + %d pinned exceed the %d cache slots of a layer", n, d.topk, pinned,
                       d.E_res);
    for (int i = 0; i < n_steps; ++i) {
        rc = spill_step(c, n, (logits && i == n_steps - 1) ? 1 : 0);
        if (rc != DM_OK) return rc;
    }
    DM_CUDA(c, cudaMemcpyAsync(c->h_bio + 2 * kMaxBatch, c->bb.tok, sizeof(int) * n, cudaMemcpyDeviceToHost, c->stream),
            "decode");
    if (logits)
        DM_CUDA(c, cudaMemcpyAsync(logits, c->bb.head_logits, sizeof(float) * n * d.V, cudaMemcpyDeviceToHost, c->stream),
                "decode");
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "decode");
    for (int i = 0; i < n; ++i) advance_lens(c, slots[i], n_steps);
    rc = check_device_error(c, "decode");
    if (rc == DM_OK && tokens_out)
        for (int i = 0; i < n; ++i) tokens_out[i] = c->h_bio[2 * kMaxBatch + i];
    return rc;
}

static int ensure_bgraph(dm_ctx* c, int n, int write_logits) {
    cudaGraphExec_t& ge = c->bgraphs[2 * n + (write_logits ? 1 : 0)];
    if (ge) return DM_OK;
    cudaGraph_t g = nullptr;
    DM_CUDA(c, cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal), "decode");
    cudaError_t e = enqueue_batch_step(c, n, write_logits);
    cudaError_t e2 = cudaStreamEndCapture(c->stream, &g);
    if (e != cudaSuccess || e2 != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "decode", -1, "batched graph capture failed: %s",
                       e == cudaErrorUnknown ? "GEMM launch" : cudaGetErrorString(e != cudaSuccess ? e : e2));
    }
    e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) {
        ge = nullptr;
        return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "decode", -1, "graph instantiate: %s", cudaGetErrorString(e));
    }
    return DM_OK;
}

// Batch preconditions: 1 <= n <= capacity, distinct valid slots, each slot ready to decode
// n_steps tokens (attention layers at the slot length, room in its pages), tokens in range.
// Stages slots and tokens on the device and brings every device position in sync.
static int prepare_batch(dm_ctx* c, const int32_t* slots, const int32_t* tokens, int n, int n_steps) {
    if (!c || !slots || !tokens || n_steps <= 0) return DM_ERR_INVALID_ARG;
    if (n <= 0 || n > c->bb.cap)
        return set_err(c, DM_ERR_INVALID_ARG, "M5_ERR_INPUT", "decode", -1, "batch of %d rows outside [1, %d]", n, c->bb.cap);
    const Dims& d = c->d;
    for (int i = 0; i < n; ++i) {
        int rc = check_slot(c, slots[i]);
        if (rc != DM_OK) return rc;
        for (int j = 0; j < i; ++j)
            if (slots[j] == slots[i])
                return set_err(c, DM_ERR_INVALID_ARG, "M5_ERR_INPUT", "decode", -1, "slot %d appears twice in the batch", slots[i]);
        if (tokens[i] < 0 || tokens[i] >= d.V)
            return set_err(c, DM_ERR_INVALID_ARG, "M4_ERR_INPUT", "input", -1, "token %d at row %d out of range [0, %d)",
                           tokens[i], i, d.V);
        const int s = slots[i];
        for (int a = 0; a < d.n_att; ++a) {
            const int al = c->att_len[static_cast<size_t>(a) * d.max_seqs + s];
            if (al != c->slot_len[s])
                return set_err(c, DM_ERR_POSITION, "M5_ERR_DECODE", "decode", -1,
                               "Position mismatch on KV append: expected current_len %d, actual_pos %d (attention layer %d)",
                               al, c->slot_len[s], a);
        }
        if (c->slot_len[s] + n_steps > d.max_pages * kPageTokens)
            return set_err(c, DM_ERR_CAPACITY, "M5_ERR_CONTEXT_SIZE", "kv_alloc", -1,
                           "KV cache capacity exceeded on token append: current_len %d + %d > capacity %d", c->slot_len[s],
                           n_steps, d.max_pages * kPageTokens);
    }
    if (static_cast<int64_t>(n) * n_steps > c->bb.gen_cap)
        return set_err(c, DM_ERR_INVALID_ARG, "M5_ERR_INPUT", "decode", -1, "n * n_steps above %d", c->bb.gen_cap);
    cudaSetDevice(c->device);
    for (int i = 0; i < n; ++i) {
        const int s = slots[i];
        if (!c->dev_pos_valid[s]) {
            c->h_io[3] = c->slot_len[s];
            DM_CUDA(c, cudaMemcpyAsync(c->b.pos + s, &c->h_io[3], 4, cudaMemcpyHostToDevice, c->stream), "decode");
            DM_CUDA(c, cudaStreamSynchronize(c->stream), "decode");
            c->dev_pos_valid[s] = 1;
        }
    }
    for (int i = 0; i < n; ++i) {
        c->h_bio[i] = slots[i];
        c->h_bio[kMaxBatch + i] = tokens[i];
    }
    DM_CUDA(c, cudaMemcpyAsync(c->bb.slots, c->h_bio, sizeof(int) * n, cudaMemcpyHostToDevice, c->stream), "decode");
    DM_CUDA(c, cudaMemcpyAsync(c->bb.tok, c->h_bio + kMaxBatch, sizeof(int) * n, cudaMemcpyHostToDevice, c->stream), "decode");
    DM_CUDA(c, cudaMemsetAsync(c->bb.gen_idx, 0, 4, c->stream), "decode");
    return DM_OK;
}

static void advance_batch(dm_ctx* c, const int32_t* slots, int n, int n_steps) {
    for (int i = 0; i < n; ++i) advance_lens(c, slots[i], n_steps);
}

// Captured graphs hold kernel arguments by value: drop them when an argument changes.
static void drop_graphs(dm_ctx* c) {
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (auto& g : c->graphs)
        if (g) cudaGraphExecDestroy(g), g = nullptr;
    for (auto& g : c->bgraphs)
        if (g) cudaGraphExecDestroy(g), g = nullptr;
}

int32_t dm_set_router_bias(dm_ctx* c, int32_t layer, const float* bias, int32_t n) {
    if (!c) return DM_ERR_INVALID_ARG;
    if (layer < 0 || layer >= c->d.L) return set_err(c, DM_ERR_INVALID_ARG, "ROUTER_ERROR", "router", layer, "layer out of range");
    if (bias && n != c->d.E)
        return set_err(c, DM_ERR_INVALID_ARG, "ROUTER_ERROR", "router", layer, "bias of %d values, expected %d", n, c->d.E);
    cudaSetDevice(c->device);
    float* dst = c->rbias + static_cast<size_t>(layer) * c->d.E;
    if (bias) DM_CUDA(c, cudaMemcpy(dst, bias, sizeof(float) * n, cudaMemcpyHostToDevice), "router");
    drop_graphs(c);
    c->layers[layer].router_bias = bias ? dst : nullptr;
    return DM_OK;
}

// ---- expert-parallel group ------------------------------------------------------------
int32_t dm_ep_ipc_handle(dm_ctx* c, void* handle_out) {
    if (!c || !handle_out) return DM_ERR_INVALID_ARG;
    cudaSetDevice(c->device);
    cudaIpcMemHandle_t h;
    DM_CUDA(c, cudaIpcGetMemHandle(&h, c->arena), "ep");
    static_assert(sizeof(cudaIpcMemHandle_t) == DM_EP_HANDLE_BYTES, "handle size");
    memcpy(handle_out, &h, sizeof h);
    return DM_OK;
}

static void ep_close(dm_ctx* c) {
    for (uint8_t*& pa : c->peer_arena)
        if (pa) cudaIpcCloseMemHandle(pa), pa = nullptr;
    c->peer_arena.clear();
}

int32_t dm_ep_attach(dm_ctx* c, int32_t rank, int32_t world, const void* handles) {
    if (!c || !handles) return DM_ERR_INVALID_ARG;
    if (spilling(c)) return spill_reject(c, "an expert-parallel group");
    const Dims& d = c->d;
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
        return set_err(c, DM_ERR_INVALID_ARG, "EP_ERROR", "ep", -1, "rank %d of %d outside [0, world <= %d)", rank, world, kMaxRanks);
    if (d.E % world != 0)
        return set_err(c, DM_ERR_INVALID_ARG, "EP_ERROR", "ep", -1, "num_experts %d not divisible by world %d", d.E, world);
    cudaSetDevice(c->device);
    drop_graphs(c);
    ep_close(c);
    c->peer_arena.assign(world, nullptr);
    BatchBuffers& bb = c->bb;
    const uint8_t* A = c->arena;
    auto off = [&](const void* p) { return static_cast<size_t>(static_cast<const uint8_t*>(p) - A); };
    EpView v{};
    v.rank = rank;
    v.world = world;
    for (int q = 0; q < world; ++q) {
        uint8_t* base = c->arena;
        if (q != rank) {
            cudaIpcMemHandle_t h;
            memcpy(&h, static_cast<const uint8_t*>(handles) + static_cast<size_t>(q) * DM_EP_HANDLE_BYTES, sizeof h);
            void* p = nullptr;
            cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                ep_close(c);
                set_local_ep(c);
                return set_err(c, DM_ERR_CUDA, "EP_ERROR", "ep", -1, "opening rank %d's memory: %s", q, cudaGetErrorString(e));
            }
            base = static_cast<uint8_t*>(p);
            c->peer_arena[q] = base;
        }
        v.ids[q] = reinterpret_cast<const int*>(base + off(bb.ids));
        v.xn[q] = reinterpret_cast<const float*>(base + off(bb.xn));
        v.eout[q] = reinterpret_cast<float*>(base + off(bb.eout));
        v.flags[q] = reinterpret_cast<unsigned*>(base + off(bb.ep_flags));
    }
    bb.ep = v;
    // barriers start from zero on every rank (the caller joins the ranks after this call)
    DM_CUDA(c, cudaMemset(bb.ep_flags, 0, 2 * kMaxRanks * 4), "ep");
    DM_CUDA(c, cudaMemset(bb.ep_epoch, 0, 2 * 4), "ep");
    DM_CUDA(c, cudaDeviceSynchronize(), "ep");
    return DM_OK;
}

int32_t dm_ep_detach(dm_ctx* c) {
    if (!c) return DM_ERR_INVALID_ARG;
    cudaSetDevice(c->device);
    drop_graphs(c);
    ep_close(c);
    set_local_ep(c);
    return DM_OK;
}

int32_t dm_batch_capacity(dm_ctx* c, int32_t* cap) {
    if (!c || !cap) return DM_ERR_INVALID_ARG;
    *cap = c->bb.cap;
    return DM_OK;
}

int32_t dm_decode_batch(dm_ctx* c, const int32_t* slots, const int32_t* tokens_in, int32_t n, int32_t* tokens_out,
                        float* logits) {
    if (c && spilling(c)) return spill_decode(c, slots, tokens_in, n, 1, tokens_out, logits);
    int rc = prepare_batch(c, slots, tokens_in, n, 1);
    if (rc != DM_OK) return rc;
    const int wl = logits ? 1 : 0;
    if ((rc = ensure_bgraph(c, n, wl)) != DM_OK) return rc;
    DM_CUDA(c, cudaGraphLaunch(c->bgraphs[2 * n + wl], c->stream), "decode");
    DM_CUDA(c, cudaMemcpyAsync(c->h_bio + 2 * kMaxBatch, c->bb.tok, sizeof(int) * n, cudaMemcpyDeviceToHost, c->stream), "decode");
    if (logits)
        DM_CUDA(c, cudaMemcpyAsync(logits, c->bb.head_logits, sizeof(float) * n * c->d.V, cudaMemcpyDeviceToHost, c->stream),
                "decode");
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "decode");
    advance_batch(c, slots, n, 1);
    rc = check_device_error(c, "decode");
    if (rc == DM_OK && tokens_out)
        for (int i = 0; i < n; ++i) tokens_out[i] = c->h_bio[2 * kMaxBatch + i];
    return rc;
}

int32_t dm_enqueue_decode_batch(dm_ctx* c, const int32_t* slots, const int32_t* tokens_in, int32_t n, int32_t n_steps) {
    // a spilling pool runs the steps here (the host takes part in every layer)
    if (c && spilling(c)) return spill_decode(c, slots, tokens_in, n, n_steps, nullptr, nullptr);
    int rc = prepare_batch(c, slots, tokens_in, n, n_steps);
    if (rc != DM_OK) return rc;
    if ((rc = ensure_bgraph(c, n, 0)) != DM_OK) return rc;
    for (int i = 0; i < n_steps; ++i) DM_CUDA(c, cudaGraphLaunch(c->bgraphs[2 * n], c->stream), "decode");
    advance_batch(c, slots, n, n_steps);
    return DM_OK;
}

int32_t dm_batch_read_generated(dm_ctx* c, int32_t n, int32_t n_steps, int32_t* out) {
    if (!c || !out || n <= 0 || n_steps <= 0 || static_cast<int64_t>(n) * n_steps > c->bb.gen_cap) return DM_ERR_INVALID_ARG;
    cudaSetDevice(c->device);
    DM_CUDA(c, cudaMemcpyAsync(out, c->bb.gen_out, sizeof(int) * n * n_steps, cudaMemcpyDeviceToHost, c->stream), "decode");
    return check_device_error(c, "decode");
}

int32_t dm_generate_batch(dm_ctx* c, const int32_t* slots, const int32_t* tokens_in, int32_t n, int32_t n_steps,
                          int32_t* out) {
    if (!out) return DM_ERR_INVALID_ARG;
    int rc = dm_enqueue_decode_batch(c, slots, tokens_in, n, n_steps);
    if (rc != DM_OK) return rc;
    return dm_batch_read_generated(c, n, n_steps, out);
}

int32_t dm_spill_stats(dm_ctx* c, uint64_t* out8) {
    if (!c || !out8) return DM_ERR_INVALID_ARG;
    memcpy(out8, c->spill.stats, sizeof(uint64_t) * 6);
    out8[6] = c->spill_bytes;
    out8[7] = spilling(c) ? static_cast<uint64_t>(c->d.E_res) : 0;
    return DM_OK;
}

int32_t dm_spill_pin(dm_ctx* c, int32_t layer, int32_t expert, int32_t* pinned) {
    if (!c) return DM_ERR_INVALID_ARG;
    if (!spilling(c)) return set_err(c, DM_ERR_INVALID_ARG, "SPILL_UNSUPPORTED", "loader", layer, "the expert pool does not spill");
    if (layer < 0 || layer >= c->d.L || expert < 0 || expert >= c->d.E)
        return set_err(c, DM_ERR_INVALID_ARG, "SPILL_ERROR", "loader", layer, "expert index out of range");
    std::vector<std::pair<int, int>> loads;
    const int r = c->spill.pin(layer, expert, loads);
    if (r < 0) return set_err(c, DM_ERR_CAPACITY, "SPILL_CAPACITY", "loader", layer, "no slot can hold expert %d", expert);
    cudaSetDevice(c->device);
    DM_CUDA(c, spill_apply(c, layer, loads), "loader");
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "loader");
    if (pinned) *pinned = r;
    return DM_OK;
}

int32_t dm_batch_stats(dm_ctx* c, int32_t reset, uint32_t* out4) {
    if (!c) return DM_ERR_INVALID_ARG;
    cudaSetDevice(c->device);
    if (out4) {
        DM_CUDA(c, cudaMemcpyAsync(c->h_bio + 3 * kMaxBatch, c->bb.stats, 16, cudaMemcpyDeviceToHost, c->stream), "stats");
        DM_CUDA(c, cudaStreamSynchronize(c->stream), "stats");
        memcpy(out4, c->h_bio + 3 * kMaxBatch, 16);
    }
    if (reset) DM_CUDA(c, cudaMemsetAsync(c->bb.stats, 0, 16, c->stream), "stats");
    return DM_OK;
}

int32_t dm_batch_kernels_per_step(dm_ctx* c, int32_t n, int32_t* own, int32_t* gemms) {
    if (!c || !own || !gemms || n <= 0 || n > c->bb.cap) return DM_ERR_INVALID_ARG;
    // embed; per block: prep, input GEMM, epilogue, mixer core (recurrence, or attention +
    // split merge), (head-norm prep,) output GEMM, residual epilogue, router, top-k +
    // grouping, the expert kernels (operand staging; gate/up and down of the small segments;
    // gate/up and down of the large ones when a step can have them), combine; head: prep,
    // GEMM, two argmax kernels.  No library GEMMs.
    *own = 1 + (10 + b_expert_launches(c->d, c->bb, n)) * c->d.L + 4;
    *gemms = 0;
    return DM_OK;
}

// Layer-level entry points: one token at a time, host activations in and out.
static int layer_args_ok(dm_ctx* c, int layer, const float* x, int n, float* y) {
    if (!c || !x || !y || n <= 0) return DM_ERR_INVALID_ARG;
    if (layer < 0 || layer >= c->d.L)
        return set_err(c, DM_ERR_INVALID_ARG, "LAYER_ERROR", "block", layer, "layer out of range");
    return DM_OK;
}

static int mixer_tokens(dm_ctx* c, int layer, int slot, int pos_offset, const float* x, int n, float* y, bool with_moe) {
    const Dims& d = c->d;
    const LayerW& w = c->layers[layer];
    int* alen = w.is_attn ? &c->att_len[static_cast<size_t>(w.sub) * d.max_seqs + slot] : nullptr;
    if (alen && pos_offset != *alen)
        return set_err(c, DM_ERR_POSITION, "M5_ERR_DECODE", "decode", layer,
                       "Position mismatch on KV append: expected current_len %d, actual_pos %d", *alen, pos_offset);
    if (pos_offset < 0 || pos_offset + n > d.max_pages * kPageTokens)
        return set_err(c, DM_ERR_CAPACITY, "M5_ERR_CONTEXT_SIZE", "kv_alloc", layer,
                       "KV cache capacity exceeded on token append");
    cudaSetDevice(c->device);
    const size_t xo = static_cast<size_t>(slot) * d.H;
    for (int t = 0; t < n; ++t) {
        c->h_io[3] = pos_offset + t;
        DM_CUDA(c, cudaMemcpyAsync(c->b.pos + slot, &c->h_io[3], 4, cudaMemcpyHostToDevice, c->stream), "block");
        DM_CUDA(c, cudaMemcpyAsync(c->b.xres + xo, x + static_cast<size_t>(t) * d.H, sizeof(float) * d.H,
                                   cudaMemcpyHostToDevice, c->stream), "block");
        DM_CUDA(c, enqueue_mixer(c, layer, slot), "block");
        const float* src = c->b.xmid + xo;
        if (with_moe) {
            DM_CUDA(c, enqueue_moe(c, layer, slot), "block");
            src = c->b.xres + xo;
        }
        DM_CUDA(c, cudaMemcpyAsync(y + static_cast<size_t>(t) * d.H, src, sizeof(float) * d.H, cudaMemcpyDeviceToHost,
                                   c->stream), "block");
        DM_CUDA(c, cudaStreamSynchronize(c->stream), "block");
        if (alen) *alen += 1;
    }
    c->dev_pos_valid[slot] = 0;
    return check_device_error(c, "block");
}

int32_t dm_mixer_block(dm_ctx* c, int32_t layer, int32_t slot, int32_t pos_offset, const float* x, int32_t n, float* y) {
    int rc = layer_args_ok(c, layer, x, n, y);
    if (rc == DM_OK) rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    return mixer_tokens(c, layer, slot, pos_offset, x, n, y, false);
}

int32_t dm_block_forward(dm_ctx* c, int32_t layer, int32_t slot, int32_t pos_offset, const float* x, int32_t n, float* y) {
    if (c && spilling(c)) return spill_reject(c, "dm_block_forward");
    int rc = layer_args_ok(c, layer, x, n, y);
    if (rc == DM_OK) rc = check_slot(c, slot);
    if (rc != DM_OK) return rc;
    return mixer_tokens(c, layer, slot, pos_offset, x, n, y, true);
}

int32_t dm_moe_block(dm_ctx* c, int32_t layer, const float* x_mid, int32_t n, float* y) {
    if (c && spilling(c)) return spill_reject(c, "dm_moe_block");
    int rc = layer_args_ok(c, layer, x_mid, n, y);
    if (rc != DM_OK) return rc;
    cudaSetDevice(c->device);
    const int H = c->d.H;
    for (int t = 0; t < n; ++t) {
        DM_CUDA(c, cudaMemcpyAsync(c->b.xmid, x_mid + static_cast<size_t>(t) * H, sizeof(float) * H, cudaMemcpyHostToDevice, c->stream), "moe");
        DM_CUDA(c, enqueue_moe(c, layer, 0), "moe");
        DM_CUDA(c, cudaMemcpyAsync(y + static_cast<size_t>(t) * H, c->b.xres, sizeof(float) * H, cudaMemcpyDeviceToHost, c->stream), "moe");
        DM_CUDA(c, cudaStreamSynchronize(c->stream), "moe");
    }
    return check_device_error(c, "moe");
}

int32_t dm_router(dm_ctx* c, int32_t layer, const float* x, int32_t n, int32_t* ids, float* probs, float* sg) {
    if (!c || !x || !ids || !probs || n <= 0) return DM_ERR_INVALID_ARG;
    if (layer < 0 || layer >= c->d.L) return set_err(c, DM_ERR_INVALID_ARG, "ROUTER_ERROR", "router", layer, "layer out of range");
    cudaSetDevice(c->device);
    const Dims& d = c->d;
    const LaunchCfg lc = lcfg(c);
    if (n > 1 && n <= c->bb.cap) {  // several rows: the batched router (same canonical bits)
        BatchBuffers& bb = c->bb;
        DM_CUDA(c, cudaMemcpyAsync(bb.xm, x, sizeof(float) * n * d.H, cudaMemcpyHostToDevice, c->stream), "router");
        DM_CUDA(c, launch_b_router(lc, d, c->layers[layer], bb, bb.xm, 0, n), "router");
        DM_CUDA(c, cudaMemcpyAsync(ids, bb.ids, sizeof(int) * n * d.topk, cudaMemcpyDeviceToHost, c->stream), "router");
        DM_CUDA(c, cudaMemcpyAsync(probs, bb.probs, sizeof(float) * n * d.topk, cudaMemcpyDeviceToHost, c->stream), "router");
        if (sg) DM_CUDA(c, cudaMemcpyAsync(sg, bb.sg, sizeof(float) * n, cudaMemcpyDeviceToHost, c->stream), "router");
        DM_CUDA(c, cudaStreamSynchronize(c->stream), "router");
        return check_device_error(c, "router");
    }
    for (int t = 0; t < n; ++t) {
        DM_CUDA(c, cudaMemcpyAsync(c->b.xn, x + static_cast<size_t>(t) * d.H, sizeof(float) * d.H, cudaMemcpyHostToDevice, c->stream), "router");
        DM_CUDA(c, launch_router(lc, d, c->layers[layer], c->b, 0, 0), "router");
        DM_CUDA(c, cudaMemcpyAsync(ids + static_cast<size_t>(t) * d.topk, c->b.topk_ids, sizeof(int) * d.topk, cudaMemcpyDeviceToHost, c->stream), "router");
        DM_CUDA(c, cudaMemcpyAsync(probs + static_cast<size_t>(t) * d.topk, c->b.topk_p, sizeof(float) * d.topk, cudaMemcpyDeviceToHost, c->stream), "router");
        if (sg) DM_CUDA(c, cudaMemcpyAsync(sg + t, c->b.shared_g, sizeof(float), cudaMemcpyDeviceToHost, c->stream), "router");
        DM_CUDA(c, cudaStreamSynchronize(c->stream), "router");
    }
    return check_device_error(c, "router");
}

// ---- phase tracing --------------------------------------------------------------------
int32_t dm_trace_enable(dm_ctx* c, int32_t on) {
    if (!c) return DM_ERR_INVALID_ARG;
    cudaSetDevice(c->device);
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "trace");
    DM_CUDA(c, cudaMemset(c->trace_buf, 0, kTraceSlots * 8), "trace");
    DM_CUDA(c, cudaMemset(c->ktrace_buf, 0, kMaxTraceKernels * 4 * 8), "trace");
    c->b.trace = on ? c->trace_buf : nullptr;
    c->b.ktrace = on ? c->ktrace_buf : nullptr;
    for (auto& g : c->graphs)  // captured graphs hold the old pointer: recapture lazily
        if (g) {
            cudaGraphExecDestroy(g);
            g = nullptr;
        }
    return DM_OK;
}

int32_t dm_trace_read(dm_ctx* c, uint64_t* out_host, int32_t n) {
    if (!c || !out_host || n <= 0 || n > kTraceSlots) return DM_ERR_INVALID_ARG;
    cudaSetDevice(c->device);
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "trace");
    DM_CUDA(c, cudaMemcpy(out_host, c->trace_buf, static_cast<size_t>(n) * 8, cudaMemcpyDeviceToHost), "trace");
    return DM_OK;
}

int32_t dm_trace_timeline(dm_ctx* c, uint64_t* rec_host, int32_t* kinds_host, int32_t n, int32_t* count) {
    if (!c || !rec_host || !kinds_host || !count || n <= 0) return DM_ERR_INVALID_ARG;
    cudaSetDevice(c->device);
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "trace");
    const int m = std::min(n, c->trace_n);
    DM_CUDA(c, cudaMemcpy(rec_host, c->ktrace_buf, static_cast<size_t>(m) * 4 * 8, cudaMemcpyDeviceToHost), "trace");
    for (int i = 0; i < m; ++i) kinds_host[i] = c->trace_kinds[i];
    *count = m;
    return DM_OK;
}

// ---- kernel timing (roofline measurement) ----------------------------------------------
int32_t dm_time_kernel(dm_ctx* c, int32_t which, int32_t layer, int32_t iters, float* avg_ms, uint64_t* bytes) {
    if (!c || !avg_ms || !bytes || iters <= 0) return DM_ERR_INVALID_ARG;
    if (spilling(c)) return spill_reject(c, "dm_time_kernel");
    const Dims& d = c->d;
    if (layer < 0 || layer >= d.L) return set_err(c, DM_ERR_INVALID_ARG, "PROFILE", "profile", layer, "layer out of range");
    const LayerW& w = c->layers[layer];
    LaunchCfg lc = lcfg(c);
    lc.pdl = false;  // timed alone: nothing to overlap with
    const int slot = 0;
    const uint64_t H = d.H;
    auto launch = [&]() -> cudaError_t {
        switch (which) {
            case DM_KERNEL_MIXER_IN:
                return w.is_attn ? launch_attn_in(lc, d, w, c->b, slot) : launch_gdn_in(lc, d, w, c->b, slot);
            case DM_KERNEL_MIXER_OUT:
                return w.is_attn ? launch_attn_out(lc, d, w, c->b, slot) : launch_gdn_out(lc, d, w, c->b, slot);
            case DM_KERNEL_MIXER_CORE:  // GDN: the recurrence, with the output projection when fused
                if (w.is_attn) return launch_attn_decode(lc, d, w, c->b, slot);
                return gdn_fused_on(c) ? launch_gdn_core_out(lc, d, w, c->b, slot) : launch_gdn_rec(lc, d, w, c->b, slot);
            case DM_KERNEL_ROUTER: return launch_router(lc, d, w, c->b, slot, 1);
            case DM_KERNEL_MOE: return launch_moe_fused(lc, d, w, c->b, slot);
            case DM_KERNEL_HEAD: return launch_head(lc, d, c->final_norm, c->lm_head, c->b, slot, 0, 0);
            default: return cudaErrorInvalidValue;
        }
    };
    // algorithmic bytes per launch (weights + state the kernel must move)
    const uint64_t eb = static_cast<uint64_t>(d.expert_bytes);
    switch (which) {
        case DM_KERNEL_MIXER_IN: *bytes = (w.is_attn ? d.attn_in_rows : d.gdn_in_rows) * H * 2; break;
        case DM_KERNEL_MIXER_OUT: *bytes = H * (w.is_attn ? d.Hq * d.D : d.z_dim) * 2; break;
        case DM_KERNEL_MIXER_CORE: {
            int len = c->slot_len[slot];
            *bytes = w.is_attn ? static_cast<uint64_t>(len + 1) * 2 * d.Hkv * d.D * 2
                               : 2ull * d.nv * d.dv * d.dk * 4 + 4ull * d.qkv_dim * 4 +
                                     (gdn_fused_on(c) ? H * d.z_dim * 2 : 0);
            break;
        }
        case DM_KERNEL_ROUTER: *bytes = (d.E + 1) * H * 2; break;
        case DM_KERNEL_MOE: *bytes = (d.E + 1) * H * 2 + (d.topk + 1) * eb; break;
        case DM_KERNEL_HEAD: *bytes = static_cast<uint64_t>(d.V) * H * 2; break;
        default: return DM_ERR_INVALID_ARG;
    }
    cudaSetDevice(c->device);
    // Each launch is timed alone after a read of kFlushBytes (twice the L2) has evicted
    // what the previous launch left in L2, so every weight byte comes from HBM; a read
    // leaves clean lines, as the weight streams of a decode step do, so the timed kernel
    // pays no write-back for the flush.
    constexpr size_t kFlushBytes = 256ull << 20;
    if (!c->flush_buf) {
        DM_CUDA(c, cudaMalloc(&c->flush_buf, kFlushBytes), "profile");
        DM_CUDA(c, cudaMemsetAsync(c->flush_buf, 0, kFlushBytes, c->stream), "profile");
    }
    cudaEvent_t e0, e1;
    DM_CUDA(c, cudaEventCreate(&e0), "profile");
    DM_CUDA(c, cudaEventCreate(&e1), "profile");
    cudaError_t e = launch();  // warm-up
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    float ms = 0.0f;
    for (int i = 0; i < iters && e == cudaSuccess; ++i) {
        e = launch_l2_flush_read(c->stream, c->flush_buf, kFlushBytes, c->num_sms);
        if (e == cudaSuccess) e = cudaEventRecord(e0, c->stream);
        if (e == cudaSuccess) e = launch();
        if (e == cudaSuccess) e = cudaEventRecord(e1, c->stream);
        if (e == cudaSuccess) e = cudaEventSynchronize(e1);
        float one = 0.0f;
        if (e == cudaSuccess) e = cudaEventElapsedTime(&one, e0, e1);
        ms += one;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "profile", layer, "%s", cudaGetErrorString(e));
    *avg_ms = ms / iters;
    return check_device_error(c, "profile");
}

// Times one kernel of the batched step for the n rows staged by the last batched call,
// on the state that call left (attention and recurrence: a layer's kernel re-run on the
// current positions; experts: gate/up + down of the grouping of the last layer).  Same
// method as dm_time_kernel: each launch alone after an L2-evicting read, CUDA events.
int32_t dm_time_batch_kernel(dm_ctx* c, int32_t n, int32_t which, int32_t layer, int32_t iters, float* avg_ms,
                             uint64_t* bytes) {
    if (!c || !avg_ms || !bytes || iters <= 0 || n <= 0 || n > c->bb.cap) return DM_ERR_INVALID_ARG;
    if (spilling(c)) return spill_reject(c, "dm_time_batch_kernel");
    const Dims& d = c->d;
    if (layer < 0 || layer >= d.L) return set_err(c, DM_ERR_INVALID_ARG, "PROFILE", "profile", layer, "layer out of range");
    const LayerW& w = c->layers[layer];
    LaunchCfg lc = lcfg(c);
    // a single kernel is timed alone; the experts are a sequence of kernels (staging, gate/up,
    // down), launched as the step launches them: each lets the next one start early
    lc.pdl = which == DM_BKERNEL_EXPERTS;
    cudaSetDevice(c->device);
    std::vector<int> slots(n);
    DM_CUDA(c, cudaMemcpy(slots.data(), c->bb.slots, sizeof(int) * n, cudaMemcpyDeviceToHost), "profile");
    uint64_t by = 0;
    if (which == DM_BKERNEL_ATTN) {
        if (!w.is_attn) return set_err(c, DM_ERR_INVALID_ARG, "PROFILE", "profile", layer, "not an attention layer");
        // every row reads its whole history (positions 0..pos) once, K and V
        for (int i = 0; i < n; ++i) by += static_cast<uint64_t>(c->slot_len[slots[i]] + 1) * 2 * d.Hkv * d.D * 2;
    } else if (which == DM_BKERNEL_GDN_REC) {
        if (w.is_attn) return set_err(c, DM_ERR_INVALID_ARG, "PROFILE", "profile", layer, "not a GDN layer");
        by = static_cast<uint64_t>(n) * (2ull * d.nv * d.dv * d.dk * 4 + 4ull * d.qkv_dim * 4);
    } else if (which == DM_BKERNEL_EXPERTS) {
        std::vector<int> ids(static_cast<size_t>(n) * d.topk);
        DM_CUDA(c, cudaMemcpy(ids.data(), c->bb.ids, sizeof(int) * ids.size(), cudaMemcpyDeviceToHost), "profile");
        std::vector<uint8_t> seen(d.E, 0);
        int uniq = 0;
        for (int v : ids)
            if (v >= 0 && v < d.E && !seen[v]) seen[v] = 1, ++uniq;
        by = static_cast<uint64_t>(uniq + 1) * d.expert_bytes;  // + the shared expert
    } else if (which == DM_BKERNEL_ROUTER) {
        by = static_cast<uint64_t>(d.E + 1) * d.H * 2;  // router rows + the shared-expert gate row
    } else if (which == DM_BKERNEL_GEMM_IN) {
        // weights once, the 2n hi/lo operand rows, the fp32 partial products
        const int N = w.is_attn ? d.attn_in_rows : d.gdn_in_rows;
        by = static_cast<uint64_t>(N) * d.H * 2 + 2ull * n * d.H * 2 + 2ull * n * N * 4;
    } else {
        return DM_ERR_INVALID_ARG;
    }
    *bytes = by;
    const LayerW& wl = c->layers[d.L - 1];  // the grouping in the buffers is the last layer's
    auto launch = [&]() -> cudaError_t {
        if (which == DM_BKERNEL_ATTN) return launch_attn_decode_batch(lc, d, w, c->bb, c->b, n);
        if (which == DM_BKERNEL_GDN_REC) return launch_gdn_rec_batch(lc, d, w, c->bb, c->b, n);
        if (which == DM_BKERNEL_ROUTER) return launch_b_router(lc, d, w, c->bb, c->bb.xm, 0, n);
        if (which == DM_BKERNEL_GEMM_IN) {
            int sp = 1;
            return bgemm(c, c->bb, 2 * layer, w.is_attn ? d.attn_in_rows : d.gdn_in_rows, d.H, n, &sp);
        }
        cudaError_t e = cudaMemsetAsync(c->bb.work + 1, 0, 8, c->stream);
        return e == cudaSuccess ? launch_b_experts(lc, d, wl, c->bb, c->b, n) : e;
    };
    constexpr size_t kFlushBytes = 256ull << 20;
    if (!c->flush_buf) {
        DM_CUDA(c, cudaMalloc(&c->flush_buf, kFlushBytes), "profile");
        DM_CUDA(c, cudaMemsetAsync(c->flush_buf, 0, kFlushBytes, c->stream), "profile");
    }
    cudaEvent_t e0, e1;
    DM_CUDA(c, cudaEventCreate(&e0), "profile");
    DM_CUDA(c, cudaEventCreate(&e1), "profile");
    cudaError_t e = launch();
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    float ms = 0.0f;
    for (int i = 0; i < iters && e == cudaSuccess; ++i) {
        e = launch_l2_flush_read(c->stream, c->flush_buf, kFlushBytes, c->num_sms);
        // the experts' work counters are reset before the start event
        if (e == cudaSuccess && which == DM_BKERNEL_EXPERTS) e = cudaMemsetAsync(c->bb.work + 1, 0, 8, c->stream);
        if (e == cudaSuccess) e = cudaEventRecord(e0, c->stream);
        if (e == cudaSuccess)
            e = which == DM_BKERNEL_EXPERTS ? launch_b_experts(lc, d, wl, c->bb, c->b, n) : launch();
        if (e == cudaSuccess) e = cudaEventRecord(e1, c->stream);
        if (e == cudaSuccess) e = cudaEventSynchronize(e1);
        float one = 0.0f;
        if (e == cudaSuccess) e = cudaEventElapsedTime(&one, e0, e1);
        ms += one;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "profile", layer, "%s", cudaGetErrorString(e));
    *avg_ms = ms / iters;
    return check_device_error(c, "profile");
}

// ---- synthetic checkpoint -------------------------------------------------------------
int32_t dm_synth_bf16(uint64_t seed, uint64_t sid, uint64_t n, float mean, float std, uint16_t* out) {
    if (!out) return DM_ERR_INVALID_ARG;
    const uint64_t key = synth_key(seed, sid);
    host_parallel(n, [&](uint64_t a, uint64_t b) {
        for (uint64_t i = a; i < b; ++i) out[i] = synth_f32_to_bf16(mean + std * synth_normal(synth_hash(key, i)));
    });
    return DM_OK;
}

int32_t dm_synth_f32(uint64_t seed, uint64_t sid, uint64_t n, float mean, float std, float* out) {
    if (!out) return DM_ERR_INVALID_ARG;
    const uint64_t key = synth_key(seed, sid);
    host_parallel(n, [&](uint64_t a, uint64_t b) {
        for (uint64_t i = a; i < b; ++i) out[i] = mean + std * synth_normal(synth_hash(key, i));
    });
    return DM_OK;
}

int32_t dm_synth_u8(uint64_t seed, uint64_t sid, uint64_t n, uint8_t* out) {
    if (!out) return DM_ERR_INVALID_ARG;
    const uint64_t key = synth_key(seed, sid);
    host_parallel(n, [&](uint64_t a, uint64_t b) {
        for (uint64_t i = a; i < b; ++i) out[i] = synth_byte(key, i);
    });
    return DM_OK;
}

int32_t dm_synth_f16_absnormal(uint64_t seed, uint64_t sid, uint64_t n, float std, uint16_t* out) {
    if (!out) return DM_ERR_INVALID_ARG;
    const uint64_t key = synth_key(seed, sid);
    host_parallel(n, [&](uint64_t a, uint64_t b) {
        for (uint64_t i = a; i < b; ++i) out[i] = synth_f32_to_f16(fabsf(std * synth_normal(synth_hash(key, i))));
    });
    return DM_OK;
}

// Seeded synthetic sequence state for every slot: the whole KV page pool bf16 N(0, kv_std),
// every GDN recurrent state and conv window fp32 N(0, state_std); every slot's length (and
// each attention layer's) becomes `len`.  Page tables are left as they are.
int32_t dm_synth_state_device(dm_ctx* c, uint64_t seed, float kv_std, float state_std, int32_t len) {
    if (!c) return DM_ERR_INVALID_ARG;
    const Dims& d = c->d;
    if (len < 0 || len > d.max_pages * kPageTokens)
        return set_err(c, DM_ERR_CAPACITY, "M5_ERR_CONTEXT_SIZE", "kv_alloc", -1, "length %d exceeds capacity", len);
    cudaSetDevice(c->device);
    const uint64_t nkv = static_cast<uint64_t>(d.n_att) * d.num_pages * 2 * d.Hkv * kPageTokens * d.D;
    const uint64_t ns = static_cast<uint64_t>(d.n_gdn) * d.max_seqs * d.nv * d.dv * d.dk;
    const uint64_t nr = static_cast<uint64_t>(d.n_gdn) * d.max_seqs * kConvRing * d.qkv_dim;
    cudaError_t e = nkv ? launch_synth_bf16(c->stream, c->b.kv, nkv, seed, 0x5eed0001ull, 0.0f, kv_std) : cudaSuccess;
    if (e == cudaSuccess && ns) e = launch_synth_f32(c->stream, c->b.S, ns, seed, 0x5eed0002ull, 0.0f, state_std);
    if (e == cudaSuccess && nr) e = launch_synth_f32(c->stream, c->b.ring, nr, seed, 0x5eed0003ull, 0.0f, state_std);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "synth", -1, "%s", cudaGetErrorString(e));
    for (int s = 0; s < d.max_seqs; ++s) {
        c->slot_len[s] = len;
        for (int a = 0; a < d.n_att; ++a) c->att_len[static_cast<size_t>(a) * d.max_seqs + s] = len;
        c->dev_pos_valid[s] = 0;
    }
    return DM_OK;
}

// W += beta u^T for a bf16 dense tensor (rows x cols as uploaded): a rank-one change of
// an uploaded weight, used to shape synthetic workloads (e.g. skewed expert load).
int32_t dm_tensor_add_rank1(dm_ctx* c, int32_t layer, int32_t id, const float* beta_host, int64_t rows,
                            const float* u_host, int32_t cols) {
    if (!c || !beta_host || !u_host || rows <= 0 || cols <= 0) return DM_ERR_INVALID_ARG;
    void* dst = nullptr;
    size_t bytes = 0;
    int rc = tensor_target(c, layer, id, DM_DTYPE_BF16, static_cast<uint64_t>(rows) * cols, &dst, &bytes);
    if (rc != DM_OK) return rc;
    cudaSetDevice(c->device);
    float* tmp = nullptr;
    DM_CUDA(c, cudaMalloc(&tmp, sizeof(float) * (rows + cols)), "synth");
    cudaError_t e = cudaMemcpyAsync(tmp, beta_host, sizeof(float) * rows, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(tmp + rows, u_host, sizeof(float) * cols, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = launch_rank1_add_bf16(c->stream, static_cast<uint16_t*>(dst), rows, cols, tmp, tmp + rows);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "synth", layer, "%s", cudaGetErrorString(e));
    return DM_OK;
}

int32_t dm_synth_model_device(dm_ctx* c, uint64_t seed) {
    if (!c) return DM_ERR_INVALID_ARG;
    cudaSetDevice(c->device);
    const Dims& d = c->d;
    const float rstd = 1.0f / sqrtf(static_cast<float>(d.H));
    auto dense = [&](int layer, int id, float mean, float std) -> int {
        void* dst = nullptr;
        size_t bytes = 0;
        const int dt = (id == DM_T_GDN_DT_BIAS || id == DM_T_GDN_A_LOG) ? DM_DTYPE_F32 : DM_DTYPE_BF16;
        // element count from the tensor table
        uint64_t n = 0;
        const size_t H = d.H;
        switch (id) {
            case DM_T_INPUT_NORM: case DM_T_POST_NORM: case DM_T_SHARED_GATE: case DM_T_FINAL_NORM: n = H; break;
            case DM_T_ROUTER: n = static_cast<uint64_t>(d.E) * H; break;
            case DM_T_GDN_QKV: n = static_cast<uint64_t>(d.qkv_dim) * H; break;
            case DM_T_GDN_Z: n = static_cast<uint64_t>(d.z_dim) * H; break;
            case DM_T_GDN_A: case DM_T_GDN_B: n = static_cast<uint64_t>(d.nv) * H; break;
            case DM_T_GDN_CONV: n = static_cast<uint64_t>(d.qkv_dim) * 4; break;
            case DM_T_GDN_DT_BIAS: case DM_T_GDN_A_LOG: n = d.nv; break;
            case DM_T_GDN_NORM: n = d.dv; break;
            case DM_T_GDN_OUT: n = H * d.z_dim; break;
            case DM_T_ATTN_Q: n = static_cast<uint64_t>(2) * d.Hq * d.D * H; break;
            case DM_T_ATTN_K: case DM_T_ATTN_V: n = static_cast<uint64_t>(d.Hkv) * d.D * H; break;
            case DM_T_ATTN_Q_NORM: case DM_T_ATTN_K_NORM: n = d.D; break;
            case DM_T_ATTN_O: n = H * d.Hq * d.D; break;
            case DM_T_EMBED: case DM_T_LM_HEAD: n = static_cast<uint64_t>(d.V) * H; break;
            default: return DM_ERR_INVALID_ARG;
        }
        int rc = tensor_target(c, layer, id, dt, n, &dst, &bytes);
        if (rc != DM_OK) return rc;
        const uint64_t sid = synth_dense_stream(layer, id);
        cudaError_t e = dt == DM_DTYPE_F32 ? launch_synth_f32(c->stream, static_cast<float*>(dst), n, seed, sid, mean, std)
                                           : launch_synth_bf16(c->stream, static_cast<uint16_t*>(dst), n, seed, sid, mean, std);
        if (e != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "synth", layer, "%s", cudaGetErrorString(e));
        c->have_dense[static_cast<size_t>(layer + 1) * DM_T_COUNT + id] = 1;
        return DM_OK;
    };
    int rc;
#define DM_TRY(x) \
    if ((rc = (x)) != DM_OK) return rc;
    DM_TRY(dense(-1, DM_T_EMBED, 0.0f, 0.02f));
    DM_TRY(dense(-1, DM_T_FINAL_NORM, 1.0f, 0.02f));
    DM_TRY(dense(-1, DM_T_LM_HEAD, 0.0f, 0.02f));
    for (int l = 0; l < d.L; ++l) {
        DM_TRY(dense(l, DM_T_INPUT_NORM, 1.0f, 0.02f));
        DM_TRY(dense(l, DM_T_POST_NORM, 1.0f, 0.02f));
        DM_TRY(dense(l, DM_T_ROUTER, 0.0f, rstd));
        DM_TRY(dense(l, DM_T_SHARED_GATE, 0.0f, 0.02f));
        if (c->layers[l].is_attn) {
            DM_TRY(dense(l, DM_T_ATTN_Q, 0.0f, 0.02f));
            DM_TRY(dense(l, DM_T_ATTN_K, 0.0f, 0.02f));
            DM_TRY(dense(l, DM_T_ATTN_V, 0.0f, 0.02f));
            DM_TRY(dense(l, DM_T_ATTN_Q_NORM, 1.0f, 0.02f));
            DM_TRY(dense(l, DM_T_ATTN_K_NORM, 1.0f, 0.02f));
            DM_TRY(dense(l, DM_T_ATTN_O, 0.0f, 0.02f));
        } else {
            DM_TRY(dense(l, DM_T_GDN_QKV, 0.0f, 0.02f));
            DM_TRY(dense(l, DM_T_GDN_Z, 0.0f, 0.02f));
            DM_TRY(dense(l, DM_T_GDN_A, 0.0f, 0.02f));
            DM_TRY(dense(l, DM_T_GDN_B, 0.0f, 0.02f));
            DM_TRY(dense(l, DM_T_GDN_CONV, 0.0f, 0.02f));
            DM_TRY(dense(l, DM_T_GDN_DT_BIAS, 0.0f, 0.02f));
            DM_TRY(dense(l, DM_T_GDN_A_LOG, 0.0f, 0.02f));
            DM_TRY(dense(l, DM_T_GDN_NORM, 1.0f, 0.02f));
            DM_TRY(dense(l, DM_T_GDN_OUT, 0.0f, 0.02f));
        }
        for (int e = -1; e < d.E; ++e) {
            for (int p = 0; p < 3; ++p) {
                const int rows = p == DM_PROJ_DOWN ? d.H : d.I;
                const int cols = p == DM_PROJ_DOWN ? d.I : d.H;
                const uint64_t nq = static_cast<uint64_t>(rows) * cols / 2, ns = static_cast<uint64_t>(rows) * (cols / d.G),
                               nz = ns / 2;
                cudaError_t ce = launch_synth_u8(c->stream, c->stage_q, nq, seed, synth_expert_stream(l, e, p, 0));
                if (ce == cudaSuccess) ce = launch_synth_f16abs(c->stream, c->stage_s, ns, seed, synth_expert_stream(l, e, p, 1), 0.02f);
                if (ce == cudaSuccess) ce = launch_synth_u8(c->stream, c->stage_z, nz, seed, synth_expert_stream(l, e, p, 2));
                uint8_t* rec = expert_record(c, l, e);
                uint8_t* dst = p == DM_PROJ_DOWN ? rec + static_cast<size_t>(d.gu_chunks) * d.gu_chunk_bytes : rec;
                if (ce == cudaSuccess) ce = launch_repack_rows(c->stream, c->stage_q, c->stage_s, c->stage_z, rows, cols, d.G, p, dst);
                if (ce == cudaSuccess) ce = spill_store(c, l, e, p);
                if (ce != cudaSuccess) return set_err(c, DM_ERR_CUDA, "CUDA_ERROR", "synth", l, "%s", cudaGetErrorString(ce));
                c->have_expert[(static_cast<size_t>(l) * (d.E + 1) + (e + 1)) * 3 + p] = 1;
            }
        }
    }
#undef DM_TRY
    DM_CUDA(c, cudaStreamSynchronize(c->stream), "synth");
    return DM_OK;
}

}  // extern "C"
