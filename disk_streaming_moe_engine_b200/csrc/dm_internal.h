// dm_internal.h — device data layout and kernel launch interface of libdismoen_cuda.so.
//
// HBM layout (one context = one model + its sequence slots):
//   dense weights   bf16, row-major [out_rows][in_cols], per layer; the token-mixer input
//                   projections of a layer are one concatenated matrix so that a single
//                   GEMV streams them (GDN: qkv | z | a | b; attention: q+gate | k | v),
//                   and the router rows are followed by the shared-expert gate row.
//   experts         per layer E routed + 1 shared record of the asymmetric 4-bit format in
//                   16-row chunks: [nibbles 16 x cols/2][fp16 scales 16 x cols/g]
//                   [uint4 zeros 16 x cols/2g]; gate_up chunk c holds gate rows 8c..8c+7
//                   then up rows 8c..8c+7 (so one CTA owns both halves of SwiGLU), then the
//                   down projection in chunks of 16 output rows.
//   GDN state       fp32 [gdn_layer][slot][nv][dv][dk]; conv window as a ring of the last
//                   4 pre-convolution projections, slot of position p = p % 4.
//   KV cache        bf16 pages [att_layer][page][K|V][Hkv][16][D], page table per slot.
#pragma once
#include <cstdint>
#include <utility>
#include <vector>
#include <cuda_runtime.h>

// Device error word bits (OR-ed by kernels, read by the host after a step).
#define DM_DEVERR_TIMEOUT 0x1u
#define DM_DEVERR_NONFINITE 0x2u
#define DM_DEVERR_CAPACITY 0x4u
#define DM_DEVERR_PAGE 0x8u
#define DM_DEVERR_TOKEN 0x10u
#define DM_DEVERR_RANGE 0x20u   // a batched expert operand exceeded the fp16 range (|x| > 65504)

namespace dm {

constexpr int kPageTokens = 16;
constexpr int kConvRing = 4;       // ring slots for the causal conv window (kernel 4)
constexpr int kMaxTopK = 16;
constexpr int kMaxSplits = 64;     // split-K partitions of decode attention
constexpr int kPfMaxSplits = 8;    // key-range splits of the prefill attention (partial slots per row and head)
constexpr int kPfMaxRows = 512;    // rows (prompt tokens) of one prefill chunk: the grouping kernel's source-row limit
constexpr int kGemvRowsPerStage = 4;
constexpr int kAttnMaxScoreSmem = 160 * 1024;  // dynamic smem bound of the decode attention

struct Dims {
    int H, L, interval, V;
    float eps;
    int Hq, Hkv, D, rot_dim;
    float theta;
    int nk, nv, dk, dv, conv_k;
    int qkv_dim, z_dim, gdn_in_rows;     // 2*nk*dk + nv*dv, nv*dv, qkv+z+2nv
    int attn_in_rows;                    // 2*Hq*D + 2*Hkv*D
    int E, topk, I, G;
    int E_res;                           // routed expert records resident in HBM per layer
                                         // (E, or the cache slots when the pool spills)
    int max_seqs, num_pages, max_pages;
    int n_gdn, n_att;
    // expert record geometry (bytes)
    int64_t gu_chunk_bytes, d_chunk_bytes, expert_bytes;
    int gu_chunks, d_chunks;
};

struct LayerW {
    int is_attn;
    int sub;                         // index among GDN layers or among attention layers
    const uint16_t* in_norm;
    const uint16_t* post_norm;
    const uint16_t* w_in;            // concatenated input projections
    const uint16_t* conv_w;          // GDN [qkv_dim][conv_k]
    const float* dt_bias;            // GDN [nv]
    const float* a_log;              // GDN [nv]
    const uint16_t* gdn_norm;        // GDN [dv]
    const uint16_t* q_norm;          // attn [D]
    const uint16_t* k_norm;          // attn [D]
    const uint16_t* w_out;           // [H][nv*dv] or [H][Hq*D]
    const uint16_t* w_router;        // [E+1][H]
    const float* router_bias;        // [E] logit offsets of a synthetic workload, or null (none)
    const void* tm_gu;               // host CUtensorMaps of the pool's gate/up and down nibble
    const void* tm_dn;               // rows (4-D: row bytes, 16 rows, chunk, expert), or null
    const uint8_t* experts;          // [E] records
    const uint8_t* shared;           // 1 record
};

// Per-context scratch and state (device pointers).
struct Buffers {
    float* xres;          // [max_seqs][H] residual stream (layer input/output)
    float* xmid;          // [max_seqs][H] after the token mixer
    float* ring;          // [n_gdn][max_seqs][4][qkv_dim]
    float* S;             // [n_gdn][max_seqs][nv][dv][dk]
    uint16_t* kv;         // [n_att][num_pages][2][Hkv][16][D]
    const void* kv_tmap;  // host CUtensorMap: 2-D view of kv (columns D, rows), 16 x 64 boxes
    int* page_table;      // [max_seqs][max_pages]
    int* pos;             // [max_seqs] current length
    int* token;           // [max_seqs] token to embed next
    int* gen_out;         // [gen_capacity] generated tokens (device loop)
    int* gen_idx;         // [1] write index into gen_out
    int gen_capacity;
    int* prompt;          // [gen_capacity] prompt ids staged for dm_forward
    // scratch for one token
    float* z;             // [z_dim]   SiLU(W_z x)
    float* ab;            // [2*nv]    a then b
    float* o;             // [nv*dv]   S q per head
    float* qg;            // [2*Hq*D]  q rows then gate rows
    float* kvnew;         // [2*Hkv*D] k then v (raw projections)
    float* attn_part;     // [Hq][kMaxSplits][D + 2]
    float* attn_out;      // [Hq*D]    gated attention output
    float* xn;            // [H]       post-attention RMSNorm output (MoE input)
    unsigned long long* rslots; // [E+1] router logit words: launch tag << 32 | fp32 bits (zero: empty)
    int* topk_ids;        // [topk]
    float* topk_p;        // [topk]
    float* shared_g;      // [1]
    float* h;             // [(topk+1)][I]  SwiGLU activations
    float* logits;        // [V]
    float* cand_val;      // [kMaxCtas]
    int* cand_idx;        // [kMaxCtas]
    unsigned* counters;   // [64]
    uint32_t* err;        // [1]
    float2* rope;         // [max_pages*16][rot_dim/2] (cos, sin) per position
    uint64_t* trace;      // [kTraceSlots] %globaltimer stamps of kernel phases, or null
    uint64_t* ktrace;     // [kMaxTraceKernels][4] per-launch timeline records, or null
};

// Scratch of the batched decode step: `n` sequences (n <= cap <= kMaxBatch), batch row b
// decodes one token of sequence slot slots[b].  Per-sequence state (GDN state, conv ring,
// KV pages, page table, position) stays in Buffers, indexed by the slot.
constexpr int kMaxBatch = 64;       // rows of one rank's batched step
constexpr int kMaxRanks = 8;        // expert-parallel group (one process per GPU)
constexpr int kSrcWords = kMaxBatch * kMaxRanks / 64;  // 64-bit words of a source-row mask
constexpr int kSegTok = 32;         // tokens of one expert segment (hi + lo rows: 64 accumulator columns)
constexpr int kSmTok = 8;           // segments of at most this many tokens use the small-segment kernels
constexpr int kSqTok = 4;           // ... split into pieces of at most this many tokens
constexpr int kHeadChunks = 32;     // vocabulary chunks of the batched argmax

// The expert-parallel group as seen by one rank: every rank runs the same batched step on
// its own n rows; expert e is computed by rank e / (E / world) for the rows of every rank
// (its activation row is read from the source rank's memory, its result written into the
// source rank's expert-output buffer), the shared expert by each rank for its own rows.
// Peer pointers are the peers' arenas mapped into this process (same layout on every
// rank); world == 1 is the single-GPU step with the local buffers.
struct EpView {
    int rank = 0, world = 1;
    const int* ids[kMaxRanks];       // [n][topk] routed experts of each rank's rows
    const float* xn[kMaxRanks];      // [n][H] normalised MoE inputs of each rank's rows
    float* eout[kMaxRanks];          // [n][topk + 1][H] expert outputs of each rank's rows
    unsigned* flags[kMaxRanks];      // [2][kMaxRanks] barrier flags of each rank
};

struct BatchBuffers {
    int cap = 0;
    int max_segs = 0;
    int max_pairs = 0;
    size_t c_cap = 0;     // floats of c (the GEMM partials share it: S x 2n x N <= c_cap)
    int* slots;           // [cap] sequence slot of batch row b
    int* tok;             // [cap] input token of row b, replaced by its argmax
    float* x;             // [cap][H] residual stream (block input / output)
    float* xm;            // [cap][H] after the token mixer
    uint16_t* xcat;       // [2 cap][Kmax] bf16 GEMM operand: rows 0..n-1 = hi, n..2n-1 = lo
    float* c;             // [2 cap][Nmax] fp32 GEMM result (same row split)
    float* z;             // [cap][z_dim]
    float* ab;            // [cap][2 nv]
    float* o;             // [cap][z_dim]
    float* qg;            // [cap][2 Hq D]
    float* kvnew;         // [cap][2 Hkv D]
    float* attn_part;     // [cap][Hq][kMaxSplits][D + 2]
    float* attn_out;      // [cap][Hq D]
    unsigned* attn_cnt;   // [cap][Hkv] last-CTA counters of the batched attention
    float* xn;            // [cap][H] normalised MoE input (canonical RMSNorm)
    float* logits;        // [cap][E + 1] router logits + shared gate logit
    int* ids;             // [cap][topk]
    float* probs;         // [cap][topk]
    float* sg;            // [cap] shared-expert gate
    unsigned* rcnt;       // [cap + 1] finished router CTAs per block of rows
    uint32_t* err;        // the context's device error word
    int4* segs;           // [max_segs] (expert, first pair, tokens, 0); expert E = shared
    int* work;            // [4] large segments, gate/up work counter, down work counter, all segments
    unsigned* stats;      // [4] routing statistics since the last reset: sum over layer-steps of
                          //     experts touched (by this rank), sum of segments, max rows of one
                          //     routed expert, layer-steps
    int* pair_src;        // [max_pairs] source of each pair: (src rank * cap + row) * 32 + k
    int max_cols = 0;     // staged operand rows: every segment's hi/lo rows padded to 16
    uint8_t* xgu;         // [max_cols][H] bf16: staged gate/up operand (64-column swizzled tiles per segment)
    uint8_t* xdn;         // [max_cols][I] bf16: staged down operand (SwiGLU activations, hi/lo)
    uint8_t* xrec;        // [max_pairs] small-segment gate/up inputs as digit records (q4_vrec_bytes(H))
    uint8_t* hrec;        // [max_pairs] small-segment down inputs (SwiGLU activations, q4_vrec_bytes(I))
    float* eout;          // [cap][topk + 1][H] expert outputs of this rank's rows (k = topk: shared)
    // prefill only (rows = prompt tokens of one sequence)
    float* pf_raw;        // [cap][qkv_dim] pre-conv GDN projections of the chunk's tokens
    float* pf_u;          // [cap][qkv_dim] their causal conv + SiLU (k heads normalised)
    uint16_t* pf_qhi;     // [cap][Hq][D] prepared q, bf16 hi
    uint16_t* pf_qlo;     // [cap][Hq][D] bf16 lo
    unsigned* ep_flags;   // [2][kMaxRanks] barrier flags written by the peers
    unsigned* ep_epoch;   // [2] barriers passed (per kind)
    float* cand_val;      // [cap][kHeadChunks]
    int* cand_idx;        // [cap][kHeadChunks]
    float* head_logits;   // [cap][V] logits (written when requested)
    int* gen_out;         // [gen_cap] tokens of a device loop, [step][n]
    int* gen_idx;         // [1] step counter of the device loop
    int gen_cap = 0;
    EpView ep;
};

constexpr int kTraceSlots = 2304;
constexpr int kTrCta = 64;        // per-CTA region: decode attention, 6 slots per CTA
constexpr int kTrCtaSlots = 6;    // start, ready, pages done, cluster merged, end, SM id
constexpr int kTrMoeCta = 1024;   // per-CTA region: fused MoE, 8 slots per CTA
constexpr int kTrMoeCtaSlots = 8; // start, ready, ids known, up data in, up done, barrier, end, SM id
// small-segment expert kernels (after the tcgen05 experts' 640 stamps): per kernel 2 stamps
// per CTA (entry, exit) for up to kTrQ4MaxCtas CTAs, then CTA 0's detail
constexpr int kTrQ4 = kTrCta + 640;
constexpr int kTrQ4MaxCtas = 160;
constexpr int kTrQ4Detail = 40;
constexpr int kTrQ4Slots = 2 * kTrQ4MaxCtas + kTrQ4Detail;
// trace slot bases per kernel kind
constexpr int kTrAttn = 0;   // 8 stamps
constexpr int kTrMoe = 16;   // 16 stamps
constexpr int kTrGdn = 2208; // fused GDN kernel: 8 stamps of CTA 0, 8 latest over the CTAs

constexpr int kMaxCtas = 1024;
// counter slots
constexpr int kCntRouter = 0;
constexpr int kCntHead = 1;
constexpr int kCntAttnBase = 8;   // + kv head (< 32)
constexpr int kCntGdnSync = 40;   // 2 words: u64 grid-barrier arrivals of the fused GDN core + out kernel
constexpr int kCntMoeSync = 48;   // 2 words: u64 up-phase arrivals of the fused MoE kernel (2 spare)
constexpr int kCntMoeFlag = 56;   // 8 words (4 x u64, 8-byte aligned) of released id words

struct Ctx;  // host-side context (dm_api.cu)

struct LaunchCfg {
    cudaStream_t stream;
    int num_sms;
    bool pdl;
    uint64_t* kt;   // timeline record of this launch (start, inputs ready, end) or null
};

// Timeline record kinds (dm_trace_timeline)
enum TraceKind { TK_EMBED = 0, TK_GDN_IN = 1, TK_GDN_REC = 2, TK_GDN_OUT = 3, TK_ATTN_IN = 4, TK_ATTN = 5,
                 TK_ATTN_OUT = 6, TK_MOE = 7, TK_HEAD = 8, TK_GDN_CORE_OUT = 9 };
constexpr int kMaxTraceKernels = 512;

// Kernel launchers (dm_kernels.cu).  `slot` selects the sequence.
cudaError_t launch_embed(const LaunchCfg& lc, const Dims& d, const uint16_t* embed,
                         const Buffers& b, int slot);
cudaError_t launch_gdn_in(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                          const Buffers& b, int slot);
cudaError_t launch_gdn_rec(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                           const Buffers& b, int slot);
cudaError_t launch_gdn_out(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                           const Buffers& b, int slot);
// GDN recurrence + output projection fused (grid = #SMs); supported() says whether the
// shapes fit it (else the two kernels above are used).
cudaError_t launch_gdn_core_out(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                                const Buffers& b, int slot);
bool gdn_fused_supported(const Dims& d, int num_sms);
cudaError_t gdn_set_attrs();
bool gdn_fused_fits(const Dims& d, int num_sms);
cudaError_t moe_fused_fits(const Dims& d, int num_sms, bool* ok);
cudaError_t launch_attn_in(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                           const Buffers& b, int slot);
cudaError_t launch_attn_decode(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                               const Buffers& b, int slot);
cudaError_t launch_attn_out(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                            const Buffers& b, int slot);
// router: normalise_input = 1 applies post_norm to b.xmid[slot]; 0 takes b.xn as given.
cudaError_t launch_router(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                          const Buffers& b, int slot, int normalise_input);
// Whole MoE mixer of one layer (router, experts, residual) in one kernel; x_mid -> xres.
// l2_next / l2_next_bytes: the weights of the kernel that follows (prefetched into L2 while
// the MoE's latency-bound phases leave HBM idle), or null.
cudaError_t launch_moe_fused(const LaunchCfg& lc, const Dims& d, const LayerW& w, const Buffers& b, int slot,
                             const void* l2_next = nullptr, uint64_t l2_next_bytes = 0);
cudaError_t launch_head(const LaunchCfg& lc, const Dims& d, const uint16_t* final_norm,
                        const uint16_t* lm_head, const Buffers& b, int slot, int advance,
                        int record_gen);

// ---- batched decode step (dm_batch.cu, dm_batch_moe.cu and the batched variants of the
// GDN recurrence and the attention).  n = batch rows of this step.
enum BPrepMode { BPREP_RMS = 0, BPREP_HEADNORM = 1, BPREP_COPY = 2 };
enum BEpiMode { BEPI_GDN_IN = 0, BEPI_ATTN_IN = 1, BEPI_RESID = 2, BEPI_GDN_PF = 3 };
cudaError_t launch_b_embed(const LaunchCfg& lc, const Dims& d, const uint16_t* embed, const BatchBuffers& bb,
                           const Buffers& b, int n);
// xcat rows from x [n][K]: RMSNorm with gamma, head norm (o = x, z, w), or a copy
cudaError_t launch_b_prep(const LaunchCfg& lc, int mode, const float* x, int K, const uint16_t* gamma, float eps,
                          const float* z, const uint16_t* hw, int dv, uint16_t* xcat, int n);
cudaError_t launch_b_epi_gdn_in(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& bb,
                                const Buffers& b, int n, int splits);
cudaError_t launch_b_epi_attn_in(const LaunchCfg& lc, const Dims& d, const BatchBuffers& bb, int n, int splits);
cudaError_t launch_b_epi_resid(const LaunchCfg& lc, const float* c, int N, const float* res, float* out, int n,
                              int splits);
// Dense projection of the batched step on the tensor cores: c[S][ncols][N] partials of
// X[ncols][K] . W[N][K]^T (tensor maps of W and of the operand rows, see dm_gemm_tc.cu).
cudaError_t tc_gemm_set_attrs();
int tc_gemm_splits(int tiles, int K, int num_sms, int max_splits);
cudaError_t launch_tc_gemm(const LaunchCfg& lc, const void* wmap, const void* xmap, float* c, int N, int K, int ncols,
                           int splits, uint32_t* err);
cudaError_t launch_gdn_rec_batch(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& bb,
                                 const Buffers& b, int n);
cudaError_t launch_attn_decode_batch(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& bb,
                                     const Buffers& b, int n);
int attn_nsplit_batch(int num_sms, int Hkv, int n);
// merges the batched attention's split partials, output gate, into the out-projection's
// hi / lo GEMM operand rows
cudaError_t launch_attn_merge_batch(const LaunchCfg& lc, const Dims& d, const BatchBuffers& bb, int n);
// MoE of one layer for n rows: router (canonical), top-k + grouping, experts, combine.
cudaError_t launch_b_router(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& bb,
                            const float* x, int normalise, int n);
// slot_of: [E] record slot of each routed expert of this layer when the pool spills, else null
cudaError_t launch_b_topk_group(const LaunchCfg& lc, const Dims& d, const BatchBuffers& bb, const Buffers& b,
                                int n, const int* slot_of = nullptr);
cudaError_t launch_b_experts(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& bb,
                             const Buffers& b, int n);
int b_expert_launches(const Dims& d, const BatchBuffers& bb, int n);  // kernels launch_b_experts launches
cudaError_t launch_b_combine(const LaunchCfg& lc, const Dims& d, const BatchBuffers& bb, const float* xm, float* out,
                             int n);
// Cross-rank barrier of the expert-parallel group (kind 0 or 1), one small kernel.
cudaError_t launch_ep_barrier(const LaunchCfg& lc, const BatchBuffers& bb, const Buffers& b, int kind);
// advance: the rows' sequence positions grow by one (decode); 0 leaves them (prefill)
cudaError_t launch_b_argmax(const LaunchCfg& lc, const Dims& d, const BatchBuffers& bb, const Buffers& b, int n,
                            int write_logits, int record_gen, int advance = 1);
cudaError_t batch_set_attrs();
// rows (sources x 1) the top-k grouping kernel can take for E experts on one rank
int b_group_max_rows(int E);
// ---- prefill of one sequence: n prompt tokens (rows) at positions pos0 .. pos0 + n - 1 ----
// GDN input-projection epilogue of a prefill chunk: pre-conv rows -> pf_raw, SiLU(z), the
// decay g and beta of every V head -> pb.ab
cudaError_t launch_b_epi_gdn_pf(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& pb, int n,
                                int splits);
// GDN recurrence over the chunk's tokens (state and conv window of (layer, slot)), then the
// conv window advanced to the chunk's last positions
cudaError_t launch_pf_gdn(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& pb,
                          const Buffers& b, int slot, int pos0, int n);
// causal attention of the chunk: preparation + append, split partials, merge + gate into pb.xcat
cudaError_t launch_pf_attn(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& pb,
                           const Buffers& b, int slot, int pos0, int n);
int pf_attn_nsplit(int num_sms, int Hkv, int n);
bool pf_gdn_supported(const Dims& d);
cudaError_t pf_attn_set_attrs();
bool expert_tc_supported(int K);
// Small-segment expert kernels (integer mma.sync on the 4-bit rows, dm_expert_q4.cu).
bool expert_q4_supported(int H, int I, int G);
size_t q4_vrec_bytes(int K);  // bytes of one K-element input vector as a digit record
cudaError_t launch_b_experts_q4(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& bb,
                                const Buffers& b, int n, bool gateup);
// SHA-256 (FIPS 180-4) of the concatenation of n buffers (dm_sha256.cu).
void sha256_parts(const uint8_t* const* parts, const size_t* sizes, int n, uint8_t out[32]);

// Residency of the expert cache when the pool spills to host memory (dm_spill.cu).
// stats: [0] accesses, [1] hits, [2] misses, [3] evictions, [4] records loaded,
// [5] pin requests kept unpinned (over the 25 % budget).
struct SpillPolicy {
    int L = 0, E = 0, C = 0;
    uint64_t clock = 0;
    std::vector<int> slot_of;        // [L][E] slot or -1
    std::vector<int> expert_in;      // [L][C] expert or -1
    std::vector<uint64_t> stamp;     // [L][C] last use
    std::vector<uint8_t> pinned;     // [L][C]
    std::vector<uint8_t> in_use;     // [C] needed by the step being resolved
    std::vector<int> pinned_count;   // [L]
    uint64_t stats[6] = {};
    void init(int L, int E, int C);
    // the distinct experts of ids[0..count) for layer l become resident; (expert, slot)
    // loads to perform are returned in order; false when the cache cannot hold them all
    bool resolve(int l, const int* ids, int count, std::vector<std::pair<int, int>>& loads);
    // 1 pinned, 0 kept unpinned (budget), -1 no slot
    int pin(int l, int e, std::vector<std::pair<int, int>>& loads);
    int victim(int l) const;
    int place(int l, int e, std::vector<std::pair<int, int>>& loads);
};
}  // namespace dm
