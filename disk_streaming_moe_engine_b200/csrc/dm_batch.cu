// dm_batch.cu — the batched decode step's small kernels (sm_100a): embedding, the
// operand preparation and epilogues around the dense projections, the canonical batched
// router, top-k + expert grouping, the MoE combine and the vocabulary argmax.
//
// Dense projections of a batch of n rows run as one tensor-core GEMM each (bf16 in, fp32
// accumulate).  To keep fp32 activations, every activation row x is split into two bf16
// rows, hi = bf16(x) and lo = bf16(x - hi) (|x - hi - lo| <= 2^-16 |x|), stacked as rows
// b and n + b of the GEMM operand; the epilogue adds the two result rows.  The weights
// are bf16 in the model, so the only rounding left is fp32 accumulation.
//
// Semantics per row are those of the single-token kernels (reference rmsnorm.mojo:10,
// gdn.mojo:897-1183 for the GDN projections and head norm, attention.mojo:219-435 for the
// attention projections, router.mojo:15-185 + topk.mojo:11-131 for routing, moe.mojo:105
// for the weighted combine, cmd_decode.mojo:115 for the first-maximum argmax).
#include <cuda_fp16.h>

#include "dm_common.cuh"
#include "dm_kernels.h"
#include "dm_router.cuh"

namespace dm {

// ---- embedding -----------------------------------------------------------------------
__global__ void __launch_bounds__(256) b_embed_kernel(const uint16_t* __restrict__ embed, int H, int V,
                                                      const int* tok, float* x, uint32_t* err) {
    const int b = blockIdx.y;
    pdl_wait();
    int t = tok[b];
    if (t < 0 || t >= V) {
        if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(err, DM_DEVERR_TOKEN);
        t = 0;
    }
    pdl_launch_dependents();
    const uint16_t* row = embed + static_cast<size_t>(t) * H;
    float* xo = x + static_cast<size_t>(b) * H;
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < H; k += gridDim.x * blockDim.x) xo[k] = bf16_to_f32(row[k]);
}

cudaError_t launch_b_embed(const LaunchCfg& lc, const Dims& d, const uint16_t* embed, const BatchBuffers& bb,
                           const Buffers& b, int n) {
    const int blocks = (d.H + 255) / 256;
    return launch_kernel(lc, b_embed_kernel, dim3(blocks, n), dim3(256), 0, embed, d.H, d.V, bb.tok, bb.x, b.err);
}

// ---- GEMM operand: hi / lo bf16 rows --------------------------------------------------
struct BPrepArgs {
    const float* x;        // [n][K] (head norm: o)
    const uint16_t* gamma; // RMSNorm weight [K] / head-norm weight [dv]
    const float* z;        // head norm: SiLU(z) [n][K]
    float eps;
    int K, dv, n;
    uint16_t* xcat;        // [2n][K]
};

DM_DEV void split_store(uint16_t* xcat, int n, int K, int b, int k, float y) {
    const uint16_t hi = f32_to_bf16(y);
    xcat[static_cast<size_t>(b) * K + k] = hi;
    xcat[static_cast<size_t>(n + b) * K + k] = f32_to_bf16(y - bf16_to_f32(hi));
}

constexpr int kPrepThreads = 256;

// One CTA per row.  RMS: y = x / sqrt(mean(x^2) + eps) * gamma; HEADNORM: per head of dv
// values y = o * rsqrt(mean_head(o^2) + eps) * w * z; COPY: y = x.
template <int MODE>
__global__ void __launch_bounds__(kPrepThreads) b_prep_kernel(const __grid_constant__ BPrepArgs a) {
    const int b = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    pdl_wait();
    const float* x = a.x + static_cast<size_t>(b) * a.K;
    if (MODE == BPREP_RMS) {
        __shared__ float red[kPrepThreads / 32];
        float acc = 0.0f;
        for (int k = tid; k < a.K; k += kPrepThreads) acc = fmaf(x[k], x[k], acc);
        acc = warp_sum(acc);
        if (lane == 0) red[warp] = acc;
        __syncthreads();
        float ss = 0.0f;
#pragma unroll
        for (int w = 0; w < kPrepThreads / 32; ++w) ss += red[w];
        const float rs = 1.0f / sqrtf(ss / static_cast<float>(a.K) + a.eps);
        pdl_launch_dependents();
        for (int k = tid; k < a.K; k += kPrepThreads) split_store(a.xcat, a.n, a.K, b, k, x[k] * rs * bf16_to_f32(a.gamma[k]));
    } else if (MODE == BPREP_HEADNORM) {
        const float* z = a.z + static_cast<size_t>(b) * a.K;
        const int nh = a.K / a.dv;
        pdl_launch_dependents();
        // grid.y slices the heads: CTA y takes heads 8 y .. 8 y + 7, one per warp
        for (int h = blockIdx.y * (kPrepThreads / 32) + warp; h < nh && h < (blockIdx.y + 1) * (kPrepThreads / 32);
             h += kPrepThreads / 32) {
            const float* oh = x + h * a.dv;
            float acc = 0.0f;
            for (int dd = lane; dd < a.dv; dd += 32) acc = fmaf(oh[dd], oh[dd], acc);
            acc = warp_sum(acc);
            const float rs = 1.0f / sqrtf(acc / static_cast<float>(a.dv) + a.eps);
            for (int dd = lane; dd < a.dv; dd += 32)
                split_store(a.xcat, a.n, a.K, b, h * a.dv + dd, oh[dd] * rs * bf16_to_f32(a.gamma[dd]) * z[h * a.dv + dd]);
        }
    } else {
        pdl_launch_dependents();
        for (int k = tid; k < a.K; k += kPrepThreads) split_store(a.xcat, a.n, a.K, b, k, x[k]);
    }
}

cudaError_t launch_b_prep(const LaunchCfg& lc, int mode, const float* x, int K, const uint16_t* gamma, float eps,
                          const float* z, const uint16_t* hw, int dv, uint16_t* xcat, int n) {
    BPrepArgs a{};
    a.x = x;
    a.gamma = mode == BPREP_HEADNORM ? hw : gamma;
    a.z = z;
    a.eps = eps;
    a.K = K;
    a.dv = dv;
    a.n = n;
    a.xcat = xcat;
    if (mode == BPREP_RMS) return launch_kernel(lc, b_prep_kernel<BPREP_RMS>, dim3(n), dim3(kPrepThreads), 0, a);
    if (mode == BPREP_HEADNORM) {
        const int nh = K / dv, per = kPrepThreads / 32;
        return launch_kernel(lc, b_prep_kernel<BPREP_HEADNORM>, dim3(n, (nh + per - 1) / per), dim3(kPrepThreads), 0, a);
    }
    return launch_kernel(lc, b_prep_kernel<BPREP_COPY>, dim3(n), dim3(kPrepThreads), 0, a);
}

// ---- GEMM epilogues: v = C[b][col] + C[n + b][col] -------------------------------------
struct BEpiArgs {
    const float* c;    // [S][2n][N]: S partial products over slices of K
    int N, n, splits;
    // GDN input projection: [qkv | z | a b] -> conv ring slot pos % 4, SiLU(z), a b
    float* ring;       // layer base [max_seqs][4][qkv_dim]
    float* raw;        // prefill: [n][qkv_dim] pre-conv rows of the chunk
    const float* a_log;    // prefill: [nv] of the layer (decay g written instead of a)
    const float* dt_bias;  // prefill: [nv]
    const int* slots;
    const int* pos;
    int qkv_dim, z_dim;
    float* z;          // [n][z_dim]
    float* ab;         // [n][2 nv]
    // attention input projection: [q gate | k v]
    float* qg;         // [n][2 Hq D]
    float* kvnew;      // [n][2 Hkv D]
    int qg_rows;
    // residual: out[b][col] = v + res[b][col]
    const float* res;
    float* out;
};

template <int MODE>
__global__ void __launch_bounds__(256) b_epi_kernel(const __grid_constant__ BEpiArgs a) {
    const int b = blockIdx.y;
    const int col = blockIdx.x * 256 + threadIdx.x;
    pdl_wait();
    pdl_launch_dependents();
    if (col >= a.N) return;
    // the S slices in order, hi + lo of each: the sum does not depend on timing
    float v = 0.0f;
    for (int s = 0; s < a.splits; ++s) {
        const float* cs = a.c + static_cast<size_t>(s) * 2 * a.n * a.N;
        v += cs[static_cast<size_t>(b) * a.N + col] + cs[static_cast<size_t>(a.n + b) * a.N + col];
    }
    if (MODE == BEPI_GDN_IN) {
        if (col < a.qkv_dim) {
            const int slot = a.slots[b];
            const int p = a.pos[slot];
            a.ring[(static_cast<size_t>(slot) * kConvRing + (p & 3)) * a.qkv_dim + col] = v;
        } else if (col < a.qkv_dim + a.z_dim) {
            a.z[static_cast<size_t>(b) * a.z_dim + (col - a.qkv_dim)] = silu_f(v);
        } else {
            const int nab = a.N - a.qkv_dim - a.z_dim;
            a.ab[static_cast<size_t>(b) * nab + (col - a.qkv_dim - a.z_dim)] = v;
        }
    } else if (MODE == BEPI_GDN_PF) {
        if (col < a.qkv_dim) {
            a.raw[static_cast<size_t>(b) * a.qkv_dim + col] = v;
        } else if (col < a.qkv_dim + a.z_dim) {
            a.z[static_cast<size_t>(b) * a.z_dim + (col - a.qkv_dim)] = silu_f(v);
        } else {  // the recurrence's decay g and beta of every V head
            const int nab = a.N - a.qkv_dim - a.z_dim, nv = nab / 2, j = col - a.qkv_dim - a.z_dim;
            a.ab[static_cast<size_t>(b) * nab + j] = j < nv ? gdn_decay(v, a.a_log[j], a.dt_bias[j]) : sigmoid_f(v);
        }
    } else if (MODE == BEPI_ATTN_IN) {
        if (col < a.qg_rows) a.qg[static_cast<size_t>(b) * a.qg_rows + col] = v;
        else a.kvnew[static_cast<size_t>(b) * (a.N - a.qg_rows) + (col - a.qg_rows)] = v;
    } else {
        a.out[static_cast<size_t>(b) * a.N + col] = v + a.res[static_cast<size_t>(b) * a.N + col];
    }
}

cudaError_t launch_b_epi_gdn_in(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& bb,
                                const Buffers& b, int n, int splits) {
    BEpiArgs a{};
    a.c = bb.c;
    a.N = d.gdn_in_rows;
    a.n = n;
    a.splits = splits;
    a.ring = b.ring + static_cast<size_t>(w.sub) * d.max_seqs * kConvRing * d.qkv_dim;
    a.slots = bb.slots;
    a.pos = b.pos;
    a.qkv_dim = d.qkv_dim;
    a.z_dim = d.z_dim;
    a.z = bb.z;
    a.ab = bb.ab;
    return launch_kernel(lc, b_epi_kernel<BEPI_GDN_IN>, dim3((a.N + 255) / 256, n), dim3(256), 0, a);
}

cudaError_t launch_b_epi_gdn_pf(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& pb, int n,
                                int splits) {
    BEpiArgs a{};
    a.a_log = w.a_log;
    a.dt_bias = w.dt_bias;
    a.c = pb.c;
    a.N = d.gdn_in_rows;
    a.n = n;
    a.splits = splits;
    a.raw = pb.pf_raw;
    a.qkv_dim = d.qkv_dim;
    a.z_dim = d.z_dim;
    a.z = pb.z;
    a.ab = pb.ab;
    return launch_kernel(lc, b_epi_kernel<BEPI_GDN_PF>, dim3((a.N + 255) / 256, n), dim3(256), 0, a);
}

cudaError_t launch_b_epi_attn_in(const LaunchCfg& lc, const Dims& d, const BatchBuffers& bb, int n, int splits) {
    BEpiArgs a{};
    a.c = bb.c;
    a.N = d.attn_in_rows;
    a.n = n;
    a.splits = splits;
    a.qg = bb.qg;
    a.kvnew = bb.kvnew;
    a.qg_rows = 2 * d.Hq * d.D;
    return launch_kernel(lc, b_epi_kernel<BEPI_ATTN_IN>, dim3((a.N + 255) / 256, n), dim3(256), 0, a);
}

cudaError_t launch_b_epi_resid(const LaunchCfg& lc, const float* c, int N, const float* res, float* out, int n,
                              int splits) {
    BEpiArgs a{};
    a.c = c;
    a.N = N;
    a.n = n;
    a.splits = splits;
    a.res = res;
    a.out = out;
    return launch_kernel(lc, b_epi_kernel<BEPI_RESID>, dim3((N + 255) / 256, n), dim3(256), 0, a);
}

// ---- batched router (canonical arithmetic, bit-identical logits to the one-token router)
// Grid (ceil((E+1)/16), ceil(n/tpc)), 512 threads: warp w owns router row 16 bx + w
// (weights in registers before griddepcontrol.wait); the CTA loads its tpc <= kBRTok input
// rows (fewer rows per CTA for small batches, so that more CTAs share the work)
// at once, normalises them into shared memory (split layout), then every warp dots its
// row with each of them.  CTAs of row block 0 also write the normalised rows (the
// experts' input).  The last CTA of a block of rows to finish (counter per row block)
// computes their softmax and top-k, one warp per row.
constexpr int kBRThreads = 512;
constexpr int kBRTok = 8;

struct BRouterArgs {
    const uint16_t* W;      // [E+1][K]
    int E, n, topk;
    const float* x;         // [n][K]
    const uint16_t* gamma;  // nullptr: x is already normalised
    float eps;
    float* xn;              // [n][K]
    float* logits;          // [n][E+1]
    const float* bias;      // [E] logit offsets, or null
    unsigned* cnt;          // [ceil(cap / tpc)] finished CTAs per row block (reset by the last)
    int tpc;                // batch rows per CTA (<= kBRTok)
    int* ids;               // [n][topk]
    float* probs;           // [n][topk]
    float* sg;              // [n]
    uint32_t* err;
};

template <int K>
__global__ void __launch_bounds__(kBRThreads, 1) b_router_kernel(const __grid_constant__ BRouterArgs a) {
    constexpr int VPL = K / 256;
    constexpr int XPT = (K + kBRThreads - 1) / kBRThreads;  // elements of a row per thread
    constexpr int RB = K <= 2048 ? kBRTok : kBRTok / 2;       // rows loaded together
    extern __shared__ __align__(16) float xs_all[];  // [kBRTok][K]; then the top-k scratch
    __shared__ float red[kBRTok * (kBRThreads / 32)];
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int row = blockIdx.x * (kBRThreads / 32) + warp;
    const int b0 = blockIdx.y * a.tpc;
    const int nt = min(a.tpc, a.n - b0);
    uint4 wreg[VPL];
    if (row <= a.E) {
        const uint4* wr = reinterpret_cast<const uint4*>(a.W + static_cast<size_t>(row) * K);
#pragma unroll
        for (int i = 0; i < VPL; ++i) wreg[i] = ldg_nc_v4(wr + lane + 32 * i);
    }
    pdl_wait();
    if (!a.gamma) {  // rows already normalised: stage them all in one pass
        for (int i = tid; i < nt * K; i += kBRThreads) {
            const int t = i / K, k = i % K;
            const float v = a.x[static_cast<size_t>(b0 + t) * K + k];
            xs_store_split(xs_all + static_cast<size_t>(t) * K, K, k, v);
            if (blockIdx.x == 0 && a.xn) a.xn[static_cast<size_t>(b0 + t) * K + k] = v;
        }
        __syncthreads();
    } else {
        for (int t0 = 0; t0 < nt; t0 += RB) {
            float xv[RB][XPT];
#pragma unroll
            for (int r = 0; r < RB; ++r)
#pragma unroll
                for (int i = 0; i < XPT; ++i) {
                    const int k = i * kBRThreads + tid;
                    xv[r][i] = (t0 + r < nt && k < K) ? a.x[static_cast<size_t>(b0 + t0 + r) * K + k] : 0.0f;
                }
            // the RB rows' reductions together (one barrier), each row in the canonical order
            float* xn = (blockIdx.x == 0 && a.xn) ? a.xn + static_cast<size_t>(b0 + t0) * K : nullptr;
            canon_rmsnorm_split_loaded_rows<K, kBRThreads, RB>(xv, min(RB, nt - t0), a.gamma, a.eps,
                                                               xs_all + static_cast<size_t>(t0) * K, xn, red);
            __syncthreads();  // xs complete; red free for the next rows
        }
    }
    pdl_launch_dependents();
    if (row <= a.E) {
        for (int t = 0; t < nt; ++t) {
            const float* xs = xs_all + static_cast<size_t>(t) * K;
            float acc = canon_router_dot<VPL>(wreg, reinterpret_cast<const float4*>(xs),
                                              reinterpret_cast<const float4*>(xs + K / 2), lane);
            if (a.bias && row < a.E) acc = __fadd_rn(acc, a.bias[row]);
            if (lane == 0) a.logits[static_cast<size_t>(b0 + t) * (a.E + 1) + row] = acc;
        }
    }
    // ---- the last CTA of this row block: softmax + top-k of its rows ----
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned prev = atomicAdd(a.cnt + blockIdx.y, 1u);
        s_last = prev == gridDim.x - 1;
        if (s_last) __threadfence();
    }
    __syncthreads();
    if (!s_last) return;
    if (warp < nt) {
        float* lg = xs_all + static_cast<size_t>(warp) * (a.E + 1);
        const float* src = a.logits + static_cast<size_t>(b0 + warp) * (a.E + 1);
        for (int e = lane; e <= a.E; e += 32) lg[e] = __ldcg(src + e);
        __syncwarp();
        const int b = b0 + warp;
        canon_softmax_topk_warp(lg, a.E, a.topk, a.ids + b * a.topk, a.probs + b * a.topk, a.sg + b, a.err);
    }
    if (tid == 0) a.cnt[blockIdx.y] = 0u;
}

static size_t b_router_smem(int K, int E) {
    const size_t xs = static_cast<size_t>(kBRTok) * K * 4, lg = static_cast<size_t>(kBRTok) * (E + 1) * 4;
    return xs > lg ? xs : lg;
}

cudaError_t launch_b_router(const LaunchCfg& lc, const Dims& d, const LayerW& w, const BatchBuffers& bb,
                            const float* x, int normalise, int n) {
    BRouterArgs a{};
    a.W = w.w_router;
    a.bias = w.router_bias;
    a.E = d.E;
    a.n = n;
    a.topk = d.topk;
    a.x = x;
    a.gamma = normalise ? w.post_norm : nullptr;
    a.eps = d.eps;
    a.xn = (!normalise && x == bb.xn) ? nullptr : bb.xn;  // rows normalised in place already
    a.logits = bb.logits;
    a.cnt = bb.rcnt;
    // rows per CTA: enough CTAs to spread the work over the GPU at small batches
    a.tpc = n <= 8 ? 1 : (n <= 16 ? 2 : (n <= 32 ? 4 : kBRTok));
    a.ids = bb.ids;
    a.probs = bb.probs;
    a.sg = bb.sg;
    a.err = bb.err;
    const dim3 grid((d.E + 1 + kBRThreads / 32 - 1) / (kBRThreads / 32), (n + a.tpc - 1) / a.tpc);
    const size_t smem = b_router_smem(d.H, d.E);
    switch (d.H) {
        case 256: return launch_kernel(lc, b_router_kernel<256>, grid, dim3(kBRThreads), smem, a);
        case 512: return launch_kernel(lc, b_router_kernel<512>, grid, dim3(kBRThreads), smem, a);
        case 1024: return launch_kernel(lc, b_router_kernel<1024>, grid, dim3(kBRThreads), smem, a);
        case 2048: return launch_kernel(lc, b_router_kernel<2048>, grid, dim3(kBRThreads), smem, a);
        case 4096: return launch_kernel(lc, b_router_kernel<4096>, grid, dim3(kBRThreads), smem, a);
        default: return cudaErrorInvalidValue;
    }
}

// ---- top-k per row + grouping of the (expert, row) pairs by expert ---------------------
// One CTA of 1024 threads.  Warp w selects for rows w, w + 32 (canonical softmax/top-k).
// In an expert-parallel group the ranks then meet at barrier 0 (every rank's ids and
// normalised rows are published).  Then this rank's experts gather their pairs from the
// rows of every rank in a fixed order: expert ascending (the shared expert, id E, last, for
// this rank's own rows), source row ascending (source = rank * n + row; a bit mask of the
// sources of each expert makes the rank of a pair a population count).  Each expert's
// pairs are cut into segments of kSegTok.  Each segment also gets the first row of its
// staged expert operand: a segment of T tokens takes 2T rows (hi, lo) rounded up to 16,
// segments in the same order.
struct BGroupArgs {
    const float* logits;  // [n][E+1]
    int E, topk, n, max_segs, max_pairs, max_cols;
    int* ids;
    float* probs;
    float* sg;
    int4* segs;
    int* work;            // [0] large segments, [1] [2] work counters (reset here), [3] all segments
    int* pair_src;
    unsigned* stats;
    EpView ep;
    unsigned* my_flags;   // [2][kMaxRanks]
    unsigned* epoch;      // [2]
    const int* slot_of;   // [E] HBM slot of each routed expert when the pool spills, else null
    int E_res;            // resident routed records (the shared expert's record index)
    int sm_tok;           // segments of at most this many tokens go to the small-segment kernels (0: none)
    uint32_t* err;
};

constexpr int kBGThreads = 1024;
constexpr int kBGMaskWords = 2048;    // (experts of a rank) x (mask words) <= 2 E <= 2046

// Exclusive prefix sum of v over the 1024 threads (fixed order); *total gets the sum.
DM_DEV int block_excl_scan(int v, int* wsum, int* total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        int s = wsum[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += t;
        }
        wsum[lane] = s;  // inclusive over warps
    }
    __syncthreads();
    const int base = warp > 0 ? wsum[warp - 1] : 0;
    if (total) *total = wsum[31];
    return base + incl - v;
}

DM_DEV void st_release_sys_u32(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
DM_DEV unsigned ld_acquire_sys_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Barrier `kind` of the expert-parallel group, by the first warp of the calling CTA
// (every thread of the CTA calls it): this rank's epoch advances by one, lane q signals
// rank q, then waits (bounded) until every rank has signalled this epoch.  False on timeout.
DM_DEV bool ep_barrier(const EpView& ep, unsigned* my_flags, unsigned* epoch, int kind, uint32_t* err) {
    __shared__ unsigned s_epoch;
    __shared__ int s_ok;
    __threadfence_system();  // this thread's writes before the signal
    __syncthreads();
    if (threadIdx.x == 0) {
        s_epoch = epoch[kind] + 1u;
        epoch[kind] = s_epoch;
        s_ok = 1;
    }
    __syncthreads();
    const unsigned e = s_epoch;
    if (threadIdx.x < 32) {
        const int q = threadIdx.x;
        if (q < ep.world) st_release_sys_u32(ep.flags[q] + kind * kMaxRanks + ep.rank, e);
        if (q < ep.world) {
            const unsigned* f = my_flags + kind * kMaxRanks + q;
            if (ld_acquire_sys_u32(f) < e) {
                const uint64_t t0 = globaltimer_ns();
                uint32_t it = 0;
                while (ld_acquire_sys_u32(f) < e) {
                    if ((++it & 255u) == 0 && globaltimer_ns() - t0 > DM_WAIT_NS) {
                        raise_error(err, DM_DEVERR_TIMEOUT);
                        s_ok = 0;
                        break;
                    }
                }
            }
        }
    }
    __syncthreads();
    __threadfence_system();  // the peers' writes before their signals are visible from here
    return s_ok != 0;
}

__global__ void __launch_bounds__(kBGThreads, 1) b_topk_group_kernel(const __grid_constant__ BGroupArgs a) {
    extern __shared__ __align__(16) float lgw[];   // the ids of every source row
    __shared__ unsigned long long mask[kBGMaskWords];
    __shared__ int start[1025];
    __shared__ int wsum[32];
    __shared__ unsigned s_maxcnt;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int E = a.E, topk = a.topk, n = a.n;
    const int world = a.ep.world, rank = a.ep.rank;
    int* sids = reinterpret_cast<int*>(lgw);  // [world][n][topk]
    pdl_wait();  // the router's last CTAs wrote this rank's ids
    // a barrier that ran out leaves the peers' ids unpublished: the step then computes no
    // expert work (the host reports DM_ERR_TIMEOUT from the error word)
    bool ep_ok = true;
    if (world > 1) ep_ok = ep_barrier(a.ep, a.my_flags, a.epoch, 0, a.err);
    else __syncthreads();
    pdl_launch_dependents();

    const int Eo = E / world, e0 = rank * Eo;     // this rank's experts
    const int nsrc = world * n;
    const int words = (nsrc + 63) / 64;
    for (int i = tid; i < nsrc * topk; i += kBGThreads) {
        const int q = i / (n * topk), r = i % (n * topk);
        sids[i] = a.ep.ids[q][r];                  // the rows of rank q (local when q == rank)
    }
    for (int i = tid; i < Eo * words; i += kBGThreads) mask[i] = 0ull;
    if (tid == 0) s_maxcnt = 0;
    __syncthreads();
    for (int i = tid; i < nsrc * topk; i += kBGThreads) {
        const int e = sids[i] - e0;
        if (e >= 0 && e < Eo) {
            const int src = i / topk;
            atomicOr(&mask[e * words + (src >> 6)], 1ull << (src & 63));
        }
    }
    __syncthreads();
    // thread el: routed expert e0 + el (el < Eo) or the shared expert (el == Eo)
    const int el = tid;
    int cnt = 0;
    if (el < Eo)
        for (int w = 0; w < words; ++w) cnt += __popcll(mask[el * words + w]);
    else if (el == Eo)
        cnt = n;
    const int nsg = (cnt + kSegTok - 1) / kSegTok;
    // segments of <= sm_tok tokens (only an expert's last one can be) go to the small-segment
    // kernels as pieces of <= kSqTok tokens: listed after every large segment, those of 4
    // tokens first, then 3, 2, 1 (the heaviest items start first), no staged operand rows
    const int tk_last = nsg > 0 ? cnt - (nsg - 1) * kSegTok : 0;
    const bool small = nsg > 0 && tk_last <= a.sm_tok;
    const int nlg = nsg - (small ? 1 : 0);
    const int pc0 = small ? min(tk_last, kSqTok) : 0;   // first piece
    const int pc1 = small ? tk_last - pc0 : 0;          // second piece (0: none)
    static_assert(kSmTok <= 2 * kSqTok, "two pieces at most");
    auto seg_rows = [](int tokens) { return (2 * tokens + 15) / 16 * 16; };
    int ncol = 0;  // staged operand rows of this expert's large segments
    for (int s2 = 0; s2 < nlg; ++s2) ncol += seg_rows(min(kSegTok, cnt - s2 * kSegTok));
    if (el < Eo && cnt > 0) atomicMax(&s_maxcnt, static_cast<unsigned>(cnt));
    const int touched = __syncthreads_count(el < Eo && cnt > 0);
    int total_pairs = 0, total_segs = 0, total_cols = 0;
    const int p0 = block_excl_scan(cnt, wsum, &total_pairs);
    __syncthreads();
    int total_lg = 0;
    const int s0 = block_excl_scan(nlg, wsum, &total_lg);
    __syncthreads();
    // pieces per size bucket (4, 3, 2, 1 tokens), this expert's place in each
    int bofs[kSqTok], btot[kSqTok];
#pragma unroll
    for (int bk = 0; bk < kSqTok; ++bk) {
        const int sz = kSqTok - bk;
        bofs[bk] = block_excl_scan((pc0 == sz) + (pc1 == sz), wsum, &btot[bk]);
        __syncthreads();
    }
    total_segs = total_lg;
    int bbase[kSqTok];
#pragma unroll
    for (int bk = 0; bk < kSqTok; ++bk) {
        bbase[bk] = total_segs;
        total_segs += btot[bk];
    }
    const int c0 = block_excl_scan(ncol, wsum, &total_cols);
    const bool pairs_ok = total_pairs <= a.max_pairs && total_segs <= a.max_segs && total_cols <= a.max_cols;
    if (el <= Eo) {
        start[el] = p0;
        // the record index the expert kernels address: the expert itself, its cache slot
        // when the pool spills, or the shared expert's record after the routed ones
        const int gexp = el < Eo ? (a.slot_of ? a.slot_of[e0 + el] : e0 + el) : a.E_res;
        if (pairs_ok) {
            int col = c0;
            for (int s2 = 0; s2 < nlg; ++s2) {
                const int tk = min(kSegTok, cnt - s2 * kSegTok);
                a.segs[s0 + s2] = make_int4(gexp, p0 + s2 * kSegTok, tk, col);
                col += seg_rows(tk);
            }
            if (small) {
                const int q0 = p0 + nlg * kSegTok;
                const int b0 = kSqTok - pc0;
                a.segs[bbase[b0] + bofs[b0]] = make_int4(gexp, q0, pc0, 0);
                if (pc1 > 0) {
                    const int b1 = kSqTok - pc1;
                    a.segs[bbase[b1] + bofs[b1] + (b1 == b0 ? 1 : 0)] = make_int4(gexp, q0 + pc0, pc1, 0);
                }
            }
        }
    }
    __syncthreads();
    if (pairs_ok) {
        for (int i = tid; i < nsrc * topk; i += kBGThreads) {
            const int e = sids[i] - e0;
            if (e >= 0 && e < Eo) {
                const int src = i / topk, k = i % topk;
                const unsigned long long* m = mask + e * words;
                int below = 0;
                for (int w = 0; w < (src >> 6); ++w) below += __popcll(m[w]);
                below += __popcll(m[src >> 6] & ((1ull << (src & 63)) - 1ull));
                a.pair_src[start[e] + below] = src * 32 + k;
            }
        }
        for (int b = tid; b < n; b += kBGThreads) a.pair_src[start[Eo] + b] = (rank * n + b) * 32 + topk;
    }
    if (tid == 0) {
        atomicAdd(a.stats + 0, static_cast<unsigned>(touched));
        atomicAdd(a.stats + 1, static_cast<unsigned>(total_segs));
        atomicMax(a.stats + 2, s_maxcnt);
        atomicAdd(a.stats + 3, 1u);
        if (!pairs_ok) raise_error(a.err, DM_DEVERR_CAPACITY);
        a.work[0] = (pairs_ok && ep_ok) ? total_lg : 0;    // large segments: [0, work[0])
        a.work[1] = 0;
        a.work[2] = 0;
        a.work[3] = (pairs_ok && ep_ok) ? total_segs : 0;  // small ones: [work[0], work[3])
    }
}

int b_group_max_rows(int E) {
    const int words = kBGMaskWords / (E > 0 ? E : 1);  // mask words per expert
    const int by_mask = 64 * words, by_ids = kMaxRanks * kMaxBatch;
    return by_mask < by_ids ? by_mask : by_ids;
}

size_t b_topk_group_smem(int E, int topk) {
    (void)E;
    return static_cast<size_t>(kMaxRanks) * kMaxBatch * topk * 4;
}

cudaError_t launch_b_topk_group(const LaunchCfg& lc, const Dims& d, const BatchBuffers& bb, const Buffers& b, int n,
                                const int* slot_of) {
    BGroupArgs a{};
    a.logits = bb.logits;
    a.E = d.E;
    a.topk = d.topk;
    a.n = n;
    a.max_segs = bb.max_segs;
    a.max_pairs = bb.max_pairs;
    a.max_cols = bb.max_cols;
    a.ids = bb.ids;
    a.probs = bb.probs;
    a.sg = bb.sg;
    a.segs = bb.segs;
    a.work = bb.work;
    a.pair_src = bb.pair_src;
    a.stats = bb.stats;
    a.ep = bb.ep;
    a.my_flags = bb.ep_flags;
    a.epoch = bb.ep_epoch;
    a.slot_of = slot_of;
    a.E_res = d.E_res;
    a.sm_tok = expert_q4_supported(d.H, d.I, d.G) ? kSmTok : 0;
    a.err = b.err;
    return launch_kernel(lc, b_topk_group_kernel, dim3(1), dim3(kBGThreads), b_topk_group_smem(d.E, d.topk), a);
}

// Barrier 1 of the expert-parallel group: every rank's experts have written their results
// into the source ranks' expert-output buffers.
__global__ void __launch_bounds__(32) ep_barrier_kernel(const __grid_constant__ EpView ep, unsigned* my_flags,
                                                        unsigned* epoch, int kind, uint32_t* err) {
    pdl_wait();
    ep_barrier(ep, my_flags, epoch, kind, err);
    pdl_launch_dependents();
}

cudaError_t launch_ep_barrier(const LaunchCfg& lc, const BatchBuffers& bb, const Buffers& b, int kind) {
    return launch_kernel(lc, ep_barrier_kernel, dim3(1), dim3(32), 0, bb.ep, bb.ep_flags, bb.ep_epoch, kind, b.err);
}

// ---- combine: out[b] = xm[b] + sum_k p_k eout[b][k] + g_sh eout[b][topk] -------------------
struct BCombineArgs {
    const float* xm;
    const float* eout;
    const float* probs;
    const float* sg;
    float* out;
    int H, topk;
};

__global__ void __launch_bounds__(256) b_combine_kernel(const __grid_constant__ BCombineArgs a) {
    const int b = blockIdx.y;
    const int i = blockIdx.x * 256 + threadIdx.x;
    pdl_wait();
    pdl_launch_dependents();
    if (i >= a.H) return;
    const float* eo = a.eout + static_cast<size_t>(b) * (a.topk + 1) * a.H + i;
    float acc = 0.0f;
    for (int k = 0; k < a.topk; ++k) acc = fmaf(a.probs[b * a.topk + k], eo[static_cast<size_t>(k) * a.H], acc);
    acc = fmaf(a.sg[b], eo[static_cast<size_t>(a.topk) * a.H], acc);
    a.out[static_cast<size_t>(b) * a.H + i] = a.xm[static_cast<size_t>(b) * a.H + i] + acc;
}

cudaError_t launch_b_combine(const LaunchCfg& lc, const Dims& d, const BatchBuffers& bb, const float* xm, float* out,
                             int n) {
    BCombineArgs a{};
    a.xm = xm;
    a.eout = bb.eout;
    a.probs = bb.probs;
    a.sg = bb.sg;
    a.out = out;
    a.H = d.H;
    a.topk = d.topk;
    return launch_kernel(lc, b_combine_kernel, dim3((d.H + 255) / 256, n), dim3(256), 0, a);
}

// ---- vocabulary argmax: first maximum wins ----------------------------------------------
struct BArgmaxArgs {
    const float* c;       // [2n][V]
    int V, n;
    float* cand_val;      // [n][kHeadChunks]
    int* cand_idx;
    float* logits_out;    // [n][V] or null
    int* tok;             // [n]
    const int* slots;
    int* pos;             // [max_seqs], advanced by one per row (null: not advanced)
    int* token;           // [max_seqs]
    int* gen_out;         // [gen_cap] or null
    int* gen_idx;
    int gen_cap;
    uint32_t* err;
};

DM_DEV void argmax_merge(float& bv, int& bi, float ov, int oi) {
    if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
    }
}

__global__ void __launch_bounds__(256) b_argmax_partial_kernel(const __grid_constant__ BArgmaxArgs a) {
    const int b = blockIdx.y, ch = blockIdx.x;
    const int per = (a.V + kHeadChunks - 1) / kHeadChunks;
    const int v0 = ch * per, v1 = min(a.V, v0 + per);
    pdl_wait();
    pdl_launch_dependents();
    const float* hi = a.c + static_cast<size_t>(b) * a.V;
    const float* lo = a.c + static_cast<size_t>(a.n + b) * a.V;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    bool bad = false;
    for (int v = v0 + threadIdx.x; v < v1; v += 256) {
        const float x = hi[v] + lo[v];
        if (x != x) bad = true;
        if (a.logits_out) a.logits_out[static_cast<size_t>(b) * a.V + v] = x;
        argmax_merge(bv, bi, x, v);
    }
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1)
        argmax_merge(bv, bi, __shfl_xor_sync(0xffffffffu, bv, m), __shfl_xor_sync(0xffffffffu, bi, m));
    __shared__ float sv[8];
    __shared__ int si[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    if (bad) raise_error(a.err, DM_DEVERR_NONFINITE);
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; ++w) argmax_merge(bv, bi, sv[w], si[w]);
        a.cand_val[b * kHeadChunks + ch] = bv;
        a.cand_idx[b * kHeadChunks + ch] = bi;
    }
}

__global__ void __launch_bounds__(1024) b_argmax_final_kernel(const __grid_constant__ BArgmaxArgs a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_wait();
    pdl_launch_dependents();
    const int step = a.gen_out ? *a.gen_idx : 0;
    for (int b = warp; b < a.n; b += 32) {
        float bv = lane < kHeadChunks ? a.cand_val[b * kHeadChunks + lane] : -INFINITY;
        int bi = lane < kHeadChunks ? a.cand_idx[b * kHeadChunks + lane] : 0x7fffffff;
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1)
            argmax_merge(bv, bi, __shfl_xor_sync(0xffffffffu, bv, m), __shfl_xor_sync(0xffffffffu, bi, m));
        if (lane == 0) {
            if (bi < 0 || bi >= a.V) {  // every logit NaN
                raise_error(a.err, DM_DEVERR_NONFINITE);
                bi = 0;
            }
            const int slot = a.slots[b];
            a.tok[b] = bi;
            a.token[slot] = bi;
            if (a.pos) a.pos[slot] += 1;
            if (a.gen_out && (step + 1) * a.n <= a.gen_cap) a.gen_out[step * a.n + b] = bi;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0 && a.gen_out) *a.gen_idx = step + 1;
}

cudaError_t launch_b_argmax(const LaunchCfg& lc, const Dims& d, const BatchBuffers& bb, const Buffers& b, int n,
                            int write_logits, int record_gen, int advance) {
    BArgmaxArgs a{};
    a.c = bb.c;
    a.V = d.V;
    a.n = n;
    a.cand_val = bb.cand_val;
    a.cand_idx = bb.cand_idx;
    a.logits_out = write_logits ? bb.head_logits : nullptr;
    a.tok = bb.tok;
    a.slots = bb.slots;
    a.pos = advance ? b.pos : nullptr;
    a.token = b.token;
    a.gen_out = record_gen ? bb.gen_out : nullptr;
    a.gen_idx = bb.gen_idx;
    a.gen_cap = bb.gen_cap;
    a.err = b.err;
    cudaError_t e = launch_kernel(lc, b_argmax_partial_kernel, dim3(kHeadChunks, n), dim3(256), 0, a);
    if (e != cudaSuccess) return e;
    return launch_kernel(lc, b_argmax_final_kernel, dim3(1), dim3(1024), 0, a);
}

cudaError_t b_experts_set_attrs();
cudaError_t b_experts_q4_set_attrs();

cudaError_t batch_set_attrs() {
    cudaError_t e = cudaSuccess;
#define DM_BR_ATTR(KK)                                                                                      \
    if (e == cudaSuccess)                                                                                   \
        e = cudaFuncSetAttribute(b_router_kernel<KK>, cudaFuncAttributeMaxDynamicSharedMemorySize,            \
                                 static_cast<int>(b_router_smem(KK, 1023)));
    DM_BR_ATTR(256)
    DM_BR_ATTR(512)
    DM_BR_ATTR(1024)
    DM_BR_ATTR(2048)
    DM_BR_ATTR(4096)
#undef DM_BR_ATTR
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(b_topk_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(b_topk_group_smem(1023, kMaxTopK)));
    if (e == cudaSuccess) e = b_experts_set_attrs();
    if (e == cudaSuccess) e = b_experts_q4_set_attrs();
    return e;
}

}  // namespace dm
