// dm_moe.cu — MoE channel mixer of the decode step on sm_100a.
//
//  router_kernel   post-attention RMSNorm + router GEMV (E rows + shared-gate row) in a
//                  fixed reduction order, then in the last CTA: fp32 softmax with the
//                  deterministic exponential, top-k on probabilities with ties to the lower
//                  expert id, no renormalisation, shared gate sigmoid
//                  (reference router.mojo:15-185, topk.mojo:11-131, moe.mojo:17).
//  moe_fused_kernel the whole MoE mixer of a layer in one kernel: RMSNorm, router and
//                  top-k, then for the k routed experts and the shared expert: nibble
//                  unpack + group scale/zero dequant fused into the gate/up GEMVs, h =
//                  SiLU(g) * u (reference swiglu.mojo:52, nibble order of
//                  quant_format.md:831-854), the down GEMVs weighted by the router
//                  probability (shared expert by its sigmoid gate) and the residual
//                  (reference moe_aggregate_forward, moe.mojo:105-177).
//
// 4-bit dot product: with F(n) = bits(0x4B000000 | n) = 2^23 + n, F(q) - F(z) = q - z is
// exact, so each weight costs one byte-permute, one subtract and one fma; the group scale
// multiplies the 32-weight partial sum once.
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include "dismoen_cuda.h"
#include "dismoen_detmath.h"
#include "dm_common.cuh"
#include "dm_kernels.h"
#include "dm_q4mma.cuh"
#include "dm_router.cuh"

namespace dm {

struct RouterArgs {
    const uint16_t* W;      // [E+1][K]
    int E, topk;
    const float* x;         // input activation
    const uint16_t* gamma;  // post-attention norm (nullptr: x already normalised)
    float eps;
    float* xn_out;          // normalised activation for the experts (written by CTA 0)
    int* ids;
    float* probs;
    float* shared_g;
    const float* bias;      // [E] logit offsets, or null
    uint32_t* err;
};

constexpr int kRouterCluster = 16;   // CTAs of the router cluster (non-portable size)
constexpr int kRouterThreads = 512;

// Router as one thread-block cluster.  CTA r of the cluster owns rows r*R .. r*R+R-1 of
// [W_router; w_shared_gate] (R = ceil((E+1)/16)), holds their weights in registers from
// before griddepcontrol.wait, normalises x itself, and stores its logits straight into
// CTA 0's shared memory (distributed shared memory); after one cluster barrier CTA 0
// computes the softmax and the top-k.  No global round trip between the two phases.
//
// Canonical reduction orders (restated by the CPU oracle for bit-exact ids):
//   RMSNorm: 512 threads, thread t: fma-accumulate x[k]^2 for k = t, t+512, ...; warp
//            butterfly (xor 16..1); the 16 warp sums added in warp order; denom =
//            sqrt(ss / K + eps); y = (x / denom) * gamma.
//   dot:     lane l: fma over elements 8(l + 32i) + j, i then j ascending; butterfly.
//   softmax: m = max; e = det_exp(z - m); lane l sums e[l], e[l+32], ... in order;
//            butterfly; p = e * (1 / sum).  Top-k: max p, ties to the lower id.
template <int K>
__global__ void __launch_bounds__(kRouterThreads, 2) router_kernel(const __grid_constant__ RouterArgs a) {
    constexpr int VPL = K / 256;
    __shared__ __align__(16) float xs[K];
    __shared__ float red[kRouterThreads / 32];
    __shared__ float lg[1024];                      // logits, used in CTA 0 only
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int nrows = a.E + 1;
    const int R = (nrows + kRouterCluster - 1) / kRouterCluster;
    const int r0 = rank * R, r1 = min(nrows, r0 + R);

    uint4 wreg[VPL];
    int row = r0 + warp;
    if (row < r1) {
        const uint4* wr = reinterpret_cast<const uint4*>(a.W + static_cast<size_t>(row) * K);
#pragma unroll
        for (int i = 0; i < VPL; ++i) wreg[i] = ldg_nc_v4(wr + lane + 32 * i);
    }
    pdl_wait();
    if (a.gamma) {
        canon_rmsnorm_split<K, kRouterThreads>(a.x, a.gamma, a.eps, xs, rank == 0 ? a.xn_out : nullptr, red);
    } else {
        for (int k = tid; k < K; k += kRouterThreads) {
            const float v = a.x[k];
            xs_store_split(xs, K, k, v);
            if (rank == 0) a.xn_out[k] = v;
        }
    }
    __syncthreads();
    pdl_launch_dependents();

    float* lg0 = cluster.map_shared_rank(lg, 0);
    const float4* xlo = reinterpret_cast<const float4*>(xs);
    const float4* xhi = reinterpret_cast<const float4*>(xs + K / 2);
    while (row < r1) {
        float acc = canon_router_dot<VPL>(wreg, xlo, xhi, lane);
        if (a.bias && row < a.E) acc = __fadd_rn(acc, a.bias[row]);
        if (lane == 0) lg0[row] = acc;
        row += kRouterThreads / 32;
        if (row < r1) {
            const uint4* wr = reinterpret_cast<const uint4*>(a.W + static_cast<size_t>(row) * K);
#pragma unroll
            for (int i = 0; i < VPL; ++i) wreg[i] = ldg_nc_v4(wr + lane + 32 * i);
        }
    }
    cluster.sync();
    if (rank != 0 || warp != 0) return;

    // ---- softmax + top-k in one warp of CTA 0 ----
    canon_softmax_topk_warp(lg, a.E, a.topk, a.ids, a.probs, a.shared_g, a.err);
}

cudaError_t launch_router(const LaunchCfg& lc, const Dims& d, const LayerW& w,
                          const Buffers& b, int slot, int normalise_input) {
    RouterArgs a{};
    a.W = w.w_router;
    a.bias = w.router_bias;
    a.E = d.E;
    a.topk = d.topk;
    a.x = normalise_input ? b.xmid + static_cast<size_t>(slot) * d.H : b.xn;
    a.gamma = normalise_input ? w.post_norm : nullptr;
    a.eps = d.eps;
    a.xn_out = normalise_input ? b.xn : b.attn_out;  // pre-normalised input: copy to scratch
    a.ids = b.topk_ids;
    a.probs = b.topk_p;
    a.shared_g = b.shared_g;
    a.err = b.err;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(kRouterCluster);
    cfg.blockDim = dim3(kRouterThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = lc.stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = lc.pdl ? 1 : 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kRouterCluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    switch (d.H) {
        case 256: return cudaLaunchKernelEx(&cfg, router_kernel<256>, a);
        case 512: return cudaLaunchKernelEx(&cfg, router_kernel<512>, a);
        case 1024: return cudaLaunchKernelEx(&cfg, router_kernel<1024>, a);
        case 2048: return cudaLaunchKernelEx(&cfg, router_kernel<2048>, a);
        case 4096: return cudaLaunchKernelEx(&cfg, router_kernel<4096>, a);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t router_set_attrs() {
    cudaError_t e = cudaSuccess;
#define DM_ROUTER_ATTR(KK)                                                                            \
    if (e == cudaSuccess)                                                                             \
        e = cudaFuncSetAttribute(router_kernel<KK>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    DM_ROUTER_ATTR(256) DM_ROUTER_ATTR(512) DM_ROUTER_ATTR(1024) DM_ROUTER_ATTR(2048) DM_ROUTER_ATTR(4096)
#undef DM_ROUTER_ATTR
    return e;
}

constexpr int kMoeMaxSlots = 16;   // gate/up chunk slots (mbarriers) per CTA

bool moe_supported(int H, int I, int G) {
    return G == 64 && ((H == 2048 && I == 512) || (H == 256 && I == 128) || (H == 1024 && I == 256) ||
                       (H == 2048 && I == 256) || (H == 4096 && I == 512));
}

// ---------------------------------------------------------------------------------------
// The whole MoE channel mixer of one layer in one kernel (router -> top-k -> gate/up ->
// down -> weighted sum + residual), one 512-thread CTA per SM, phases separated by
// grid-wide flags in global memory (every wait bounded by DM_WAIT_NS):
//   pre-wait  : router rows of this CTA into registers; shared-expert chunks of this
//               CTA into shared memory (bulk copies); next layer's input projection into
//               L2.  Then griddepcontrol.wait.
//   phase 1   : every CTA normalises x_mid (canonical order); CTAs 0..R-1 compute the
//               router logits (canonical order) and store each as a tagged word; then
//               every CTA lets the next kernel launch (its weight preloads overlap the
//               top-k and stay clear of the router phase and of the routed-expert copies:
//               measured against triggering right after the wait, after the norm, after
//               the ids and after phase 2, this point is the fastest by 1-8 %).
//   phase 1b  : every CTA polls the E + 1 logit words and runs the softmax and the top-k
//               itself with all its threads (no id broadcast: the same arithmetic on the
//               same words gives every CTA the same ids).
//   issue     : every CTA bulk-copies its routed gate/up chunks and its 16-row down
//               chunk of every selected expert (the down data lands during phase 2).
//   phase 2   : gate/up GEMVs, h = SiLU(g) * u to global; grid barrier (arrivals on a
//               64-bit counter that is never reset: the target is the launch generation
//               read at the start, plus one, times the grid).
//   phase 3   : CTAs 0..H/16-1 produce their 16 output rows, one warp per row over all
//               experts (even and odd experts in two accumulators, added in a fixed
//               order) + residual.
//   exit      : nothing to reset (the barrier counter and the logit words carry the
//               launch generation), so the grid ends as its last rows are stored.
struct MoeFusedArgs {
    const uint16_t* Wr;       // [E+1][H] router rows + shared-gate row
    const float* rbias;       // [E] logit offsets, or null
    const uint16_t* gamma;    // post-attention norm
    float eps;
    const float* x_mid;       // [H]
    float* x_out;             // [H]
    float* xn_out;            // [H] normalised input (written by CTA 0, for inspection)
    const uint8_t* experts;
    const uint8_t* shared;
    int64_t expert_bytes, gu_part_bytes;
    int E, topk, I, gu_chunks, d_chunks, up_slots;
    unsigned long long* lslots; // [E+1] router logit words (launch tag << 32 | fp32 bits)
    int* ids;
    float* probs;
    float* shared_g;
    float* h;                 // [(topk+1)][I]
    unsigned long long* arrivals; // up-phase arrivals of every launch so far (never reset)
    uint64_t* trace;          // phase stamps of CTA 0 and of the last CTA, or null
    uint64_t* cta_trace;      // per-CTA stamps (kTrMoeCtaSlots per CTA, thread 0) or null
    uint64_t* kt;             // launch timeline record or null
    uint32_t* err;
    const uint8_t* l2_next;   // the next kernel's weights, prefetched into L2 while this
    uint64_t l2_next_bytes;   // kernel's phases leave HBM idle (or null / 0)
};

DM_DEV void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
DM_DEV unsigned ld_relaxed_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
DM_DEV void st_relaxed_u32(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Router logit slots: one 64-bit word per row, the launch tag (generation + 1, never 0) in
// the high half and the fp32 logit bits in the low half, written with one store.  A reader
// polls a slot until its tag matches this launch's: the previous launch's words never match,
// so nothing is emptied between launches (slots start as zero words).
DM_DEV float poll_slot(const unsigned long long* p, unsigned tag, uint32_t* err) {
    unsigned long long v = ld_relaxed_u64(p);
    if (static_cast<unsigned>(v >> 32) == tag) return __uint_as_float(static_cast<unsigned>(v));
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t n = 1;; ++n) {
        v = ld_relaxed_u64(p);
        if (static_cast<unsigned>(v >> 32) == tag) return __uint_as_float(static_cast<unsigned>(v));
        if (n % 256 == 0 && globaltimer_ns() - t0 > DM_WAIT_NS) {
            raise_error(err, DM_DEVERR_TIMEOUT);
            return 0.0f;
        }
    }
}

constexpr int kMoeThreads = 512;
// Share (in quarters) of the next kernel's weights prefetched into L2 during the top-k; the
// rest follows once the routed gate/up bytes are in.
constexpr int kMoeL2First = 2;
constexpr int kMoeMaxE = kMoeThreads;  // phase 1b: one thread per expert

template <int K, int KI, int G>
struct MoeFusedSmem {
    using QU = Q4<K, G>;
    using QD = Q4<KI, G>;
    __host__ __device__ static size_t up_off() { return 0; }
    __host__ __device__ static size_t dn_off(int up_slots) { return static_cast<size_t>(up_slots) * QU::CHUNK; }
    __host__ __device__ static size_t xn_off(int up_slots, int nexp) { return dn_off(up_slots) + static_cast<size_t>(nexp) * QD::CHUNK; }
    __host__ __device__ static size_t xs_off(int up_slots, int nexp) { return xn_off(up_slots, nexp) + K * 4; }
    __host__ __device__ static size_t h_off(int up_slots, int nexp) { return xs_off(up_slots, nexp) + K * 4; }
    // the h region holds phase 1b's logits and candidates (16 bytes per expert), then each
    // expert's h as vector fragments and scale groups
    __host__ __device__ static size_t h_bytes(int nexp, int E) {
        const size_t hb = static_cast<size_t>(nexp) * (KI * 4 + vfrag_bytes(KI) + (KI / kQ4G) * sizeof(VGroup));
        const size_t tb = static_cast<size_t>(E + 2) * 16;
        return hb > tb ? hb : tb;
    }
    __host__ __device__ static size_t total(int up_slots, int nexp, int E) { return h_off(up_slots, nexp) + h_bytes(nexp, E); }
};

template <int K, int KI, int G>
__global__ void __launch_bounds__(kMoeThreads, 2) moe_fused_kernel(const __grid_constant__ MoeFusedArgs a) {
    using QU = Q4<K, G>;   // global chunk layouts
    using QD = Q4<KI, G>;
    constexpr int NGU = K / kQ4G, NGD = KI / kQ4G;  // scale groups per gate/up and down row
    using SM = MoeFusedSmem<K, KI, G>;
    static_assert(G == kQ4G, "group size");
    constexpr int VPL = K / 256;
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ __align__(8) uint64_t bar_up[kMoeMaxSlots];
    __shared__ __align__(8) uint64_t bar_dn[kMaxTopK + 1];
    __shared__ __align__(8) uint64_t bar_h;  // phase 3's copy of h
    __shared__ int sid[kMaxTopK];
    __shared__ float sp[kMaxTopK + 1];
    __shared__ float red[kMoeThreads / 32];
    __shared__ unsigned long long s_gen;
    __shared__ float s_wred[kMoeThreads / 32];
    __shared__ int s_wcnt[kMoeThreads / 32];
    __shared__ int s_wcnt_b[kMoeThreads / 32];
    __shared__ float s_part[256];  // partial rows: phase 2 [group][quarter][16], phase 3 [warp][16]
    __shared__ uint32_t s_g8[kMoeMaxE / 8];
    __shared__ uint32_t s_thr;
    __shared__ float s_inv;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int nblk = gridDim.x, c = blockIdx.x;
    const int nexp = a.topk + 1;
    const int nrows = a.E + 1;
    const int R = (nrows + 15) / 16;                 // router CTAs, 16 rows each
    const int n_items = nexp * a.gu_chunks;
    const int i0 = static_cast<int>(static_cast<int64_t>(c) * n_items / nblk);
    const int i1 = static_cast<int>(static_cast<int64_t>(c + 1) * n_items / nblk);
    const bool has_down = c < a.d_chunks;
    uint8_t* up_s = dsm + SM::up_off();
    uint8_t* dn_s = dsm + SM::dn_off(a.up_slots);
    // x_norm as vector fragments, then its scale groups
    int8_t* xvf = reinterpret_cast<int8_t*>(dsm + SM::xn_off(a.up_slots, nexp));
    VGroup* xvg = reinterpret_cast<VGroup*>(xvf + vfrag_bytes(K));
    float* xsr = reinterpret_cast<float*>(dsm + SM::xs_off(a.up_slots, nexp));
    float* h4 = reinterpret_cast<float*>(dsm + SM::h_off(a.up_slots, nexp));

    uint64_t* tr = tid == 0 ? (c == 0 ? a.trace : (c == nblk - 1 && a.trace ? a.trace + 10 : nullptr)) : nullptr;
    uint64_t* ct = (tid == 0 && a.cta_trace) ? a.cta_trace + c * kTrMoeCtaSlots : nullptr;
    trace_stamp(tr, 0);
    trace_stamp(ct, 0);
    kt_start(a.kt);
    // ---- pre-wait: nothing here depends on the previous kernel ----
    const int rrow = c * 16 + warp;
    const bool router_cta = c < R;
    uint4 wreg[VPL];
    if (router_cta && warp < 16 && rrow < nrows) {
        const uint4* wr = reinterpret_cast<const uint4*>(a.Wr + static_cast<size_t>(rrow) * K);
#pragma unroll
        for (int i = 0; i < VPL; ++i) wreg[i] = ldg_nc_v4(wr + lane + 32 * i);
    }
    if (tid == 0) {
        for (int k = 0; k < i1 - i0; ++k) mbar_init(&bar_up[k], 1);
        for (int j = 0; j < nexp; ++j) mbar_init(&bar_dn[j], 1);
        mbar_init(&bar_h, 1);
        mbar_fence_init();
        for (int k = 0; k < i1 - i0; ++k) {
            const int item = i0 + k;
            if (item / a.gu_chunks != a.topk) continue;
            mbar_arrive_expect_tx(&bar_up[k], QU::CHUNK);
            bulk_g2s(up_s + static_cast<size_t>(k) * QU::CHUNK,
                     a.shared + static_cast<int64_t>(item % a.gu_chunks) * QU::CHUNK, QU::CHUNK, &bar_up[k]);
        }
        if (has_down) {
            mbar_arrive_expect_tx(&bar_dn[a.topk], QD::CHUNK);
            bulk_g2s(dn_s + static_cast<size_t>(a.topk) * QD::CHUNK,
                     a.shared + a.gu_part_bytes + static_cast<int64_t>(c) * QD::CHUNK, QD::CHUNK, &bar_dn[a.topk]);
        }
    }
    constexpr int XPT = (K + kMoeThreads - 1) / kMoeThreads;
    float gv[XPT];  // post-attention norm gains (weights) before the wait
#pragma unroll
    for (int i = 0; i < XPT; ++i) {
        const int k = i * kMoeThreads + tid;
        gv[i] = k < K ? bf16_to_f32(a.gamma[k]) : 0.0f;
    }
    pdl_wait();
    kt_ready(a.kt);
    trace_stamp(tr, 1);
    trace_stamp(ct, 1);
    // Launch generation: the arrival counter grows by nblk per launch and is never reset,
    // and this CTA reads it before it arrives itself, when fewer than nblk arrivals of this
    // launch can have happened, so the quotient is the number of earlier launches.  The id
    // words carry its parity, flipped, as their tag, so the previous launch's words never
    // match: no flag needs resetting at exit.
    if (tid == 0) s_gen = ld_relaxed_u64(a.arrivals) / static_cast<unsigned long long>(nblk);
    // residual of output row 16c + lane (phase 3, warp 0), fetched now, off the critical path
    const float xm_row = (has_down && warp == 0 && lane < 16) ? a.x_mid[16 * c + lane] : 0.0f;

    // ---- phase 1: canonical RMSNorm (512 threads), router rows ----
    {
        float xv[XPT];
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < XPT; ++i) {
            const int k = i * kMoeThreads + tid;
            xv[i] = k < K ? a.x_mid[k] : 0.0f;
            if (k < K) acc = __fmaf_rn(xv[i], xv[i], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) red[warp] = acc;
        __syncthreads();
        float ss = 0.0f;
#pragma unroll
        for (int w = 0; w < kMoeThreads / 32; ++w) ss = __fadd_rn(ss, red[w]);
        const float denom = __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, static_cast<float>(K)), a.eps));
#pragma unroll
        for (int i = 0; i < XPT; ++i) {
            const int k = i * kMoeThreads + tid;
            if (k < K) {
                const float y = __fmul_rn(__fdiv_rn(xv[i], denom), gv[i]);
                xs_store_split(xsr, K, k, y);
                if (c == 0 && a.xn_out) a.xn_out[k] = y;
            }
        }
    }
    __syncthreads();
    trace_stamp(tr, 2);
    const unsigned tag = static_cast<unsigned>(s_gen & 0x7FFFFFFFull) + 1u;  // this launch's slot tag
    if (router_cta) {
        if (rrow < nrows) {
            const float4* xlo = reinterpret_cast<const float4*>(xsr);
            const float4* xhi = reinterpret_cast<const float4*>(xsr + K / 2);
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
            acc = warp_sum(acc);
            if (a.rbias && rrow < a.E) acc = __fadd_rn(acc, a.rbias[rrow]);
            if (lane == 0)
                st_relaxed_u64(a.lslots + rrow, (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(acc));
        }
    }
    trace_stamp(tr, 3);
    pdl_launch_dependents();  // the next kernel's preloads overlap the top-k
    // the first part of the next kernel's weights into L2 while the top-k runs (HBM idle)
    if (warp == 0) prefetch_l2_share(a.l2_next, a.l2_next_bytes * kMoeL2First / 4, c, nblk, lane);
    // ---- phase 1b, in every CTA: the E + 1 logits, softmax and top-k.  Every CTA runs the
    // same arithmetic on the same words, so all reach the same ids without a broadcast ----
    {
        const int E = a.E, topk = a.topk;
        float* s_lg = h4;                                              // [E + 1] logits, then e^(z - m)
        uint2* s_cand = reinterpret_cast<uint2*>(h4 + ((E + 2) & ~1));  // [E] (key, id) of the candidates
        for (int e = tid; e <= E; e += kMoeThreads) s_lg[e] = poll_slot(a.lslots + e, tag, a.err);
        __syncthreads();
        trace_stamp(tr ? tr + 20 : nullptr, 0);
        // softmax in the canonical order: m = max; e = det_exp(z - m); lane l of one warp sums
        // e[l], e[l + 32], ... in order; butterfly; p = e * (1 / sum)
        const float z = tid < E ? s_lg[tid] : -INFINITY;
        const float mw = warp_max(fmaxf(-INFINITY, z));
        if (lane == 0) s_wred[warp] = mw;
        __syncthreads();
        float m = s_wred[0];
#pragma unroll
        for (int w = 1; w < kMoeThreads / 32; ++w) m = fmaxf(m, s_wred[w]);
        float p = 0.0f;
        if (tid < E) {
            p = dm_det_exp(DM_DET_SUB(z, m));
            s_lg[tid] = p;
        }
        __syncthreads();
        if (warp == 0) {
            float sum = 0.0f;
            for (int e = lane; e < E; e += 32) sum = DM_DET_ADD(sum, s_lg[e]);
            sum = warp_sum(sum);
            if (lane == 0) {
                s_inv = DM_DET_DIV(1.0f, sum);
                if (c == 0 && (sum != sum || isinf(sum))) raise_error(a.err, DM_DEVERR_NONFINITE);
            }
        }
        __syncthreads();
        trace_stamp(tr ? tr + 20 : nullptr, 1);
        const long long tk0 = clock64();
        // keys: probability bits (probabilities >= 0 order like their bits); 0 for p <= 0
        // or NaN.  Order: larger key first, ties to the lower id.
        uint32_t key = 0u;
        if (tid < E) {
            p = DM_DET_MUL(p, s_inv);
            key = p > 0.0f ? __float_as_uint(p) : 0u;
        }
        // threshold: each group of 8 consecutive experts offers its largest key; with at
        // least topk groups, thr = the topk-th largest of these maxima is held by topk
        // distinct experts, so every expert below thr ranks >= topk.  The top-k are then
        // A = {key > thr} (at most topk - 1 groups lie above thr: <= 8 (topk - 1) experts),
        // ranked among themselves, followed by B = {key == thr} in id order.
        const int ng8 = (E + 7) / 8;
        {
            uint32_t gm = key;
#pragma unroll
            for (int m = 1; m < 8; m <<= 1) gm = max(gm, __shfl_xor_sync(0xffffffffu, gm, m));
            if ((lane & 7) == 0 && tid < E) s_g8[tid >> 3] = gm;
        }
        __syncthreads();
        if (tid < ng8) {
            uint32_t t = 0u;  // fewer groups than topk: every expert is in A or B
            if (ng8 >= topk) {
                const uint32_t me = s_g8[tid];
                int r = 0;
                for (int j = 0; j < ng8; ++j) {
                    const uint32_t o = s_g8[j];
                    r += (o > me || (o == me && j < tid)) ? 1 : 0;
                }
                if (r == topk - 1) s_thr = me;
            } else if (tid == 0) {
                s_thr = t;
            }
        }
        __syncthreads();
        const uint32_t thr = s_thr;
        const bool in_a = tid < E && key > thr, in_b = tid < E && key == thr;
        const unsigned bal_a = __ballot_sync(0xffffffffu, in_a), bal_b = __ballot_sync(0xffffffffu, in_b);
        if (lane == 0) {
            s_wcnt[warp] = __popc(bal_a);
            s_wcnt_b[warp] = __popc(bal_b);
        }
        __syncthreads();
        int base_a = 0, na = 0, base_b = 0;
#pragma unroll
        for (int w = 0; w < kMoeThreads / 32; ++w) {
            const int n = s_wcnt[w];
            base_a += w < warp ? n : 0;
            base_b += w < warp ? s_wcnt_b[w] : 0;
            na += n;
        }
        const unsigned below = (1u << lane) - 1u;
        if (in_a) s_cand[base_a + __popc(bal_a & below)] = make_uint2(key, static_cast<unsigned>(tid));
        // B in id order: the first topk - na of them complete the selection
        if (in_b) {
            const int r = na + base_b + __popc(bal_b & below);
            if (r < topk) {
                sid[r] = tid;
                sp[r] = __uint_as_float(key);
            }
        }
        __syncthreads();
        trace_stamp(tr ? tr + 20 : nullptr, 2);
        // A's ranks among A are its ranks among all experts
        for (int i = tid; i < na; i += kMoeThreads) {
            const uint2 me = s_cand[i];
            int r = 0;
#pragma unroll 4
            for (int j = 0; j < na; ++j) {
                const uint2 o = s_cand[j];
                r += (o.x > me.x || (o.x == me.x && o.y < me.y)) ? 1 : 0;
            }
            if (r < topk) {
                sid[r] = static_cast<int>(me.y);
                sp[r] = __uint_as_float(me.x);
            }
        }
        if (tid == 0) sp[topk] = sigmoid_f(s_lg[E]);
        __syncthreads();
        if (tr && c == 0 && tid == 0) tr[44] = static_cast<uint64_t>(clock64() - tk0);  // top-k, SM cycles (slot 60)
        trace_stamp(tr ? tr + 20 : nullptr, 3);
        if (c == 0) {  // the selection, for inspection
            if (tid < topk) {
                a.ids[tid] = sid[tid];
                a.probs[tid] = sp[tid];
            }
            if (tid == 0) *a.shared_g = sp[topk];
        }
    }
    trace_stamp(tr, 5);
    trace_stamp(ct, 2);

    // ---- issue the routed chunks: gate/up items and this CTA's down chunk (one
    // thread per copy) ----
    if (tid < i1 - i0) {
        const int k = tid;
        const int item = i0 + k;
        const int j = item / a.gu_chunks;
        if (j != a.topk) {
            mbar_arrive_expect_tx(&bar_up[k], QU::CHUNK);
            bulk_g2s(up_s + static_cast<size_t>(k) * QU::CHUNK,
                     a.experts + static_cast<int64_t>(sid[j]) * a.expert_bytes +
                         static_cast<int64_t>(item % a.gu_chunks) * QU::CHUNK,
                     QU::CHUNK, &bar_up[k]);
        }
    }
    // this CTA's routed down chunks are needed only after the grid barrier: they are
    // issued once its first gate/up item has landed (or now, if it has none), so the
    // gate/up bytes go first
    auto issue_down = [&](int j) {
        mbar_arrive_expect_tx(&bar_dn[j], QD::CHUNK);
        bulk_g2s(dn_s + static_cast<size_t>(j) * QD::CHUNK,
                 a.experts + static_cast<int64_t>(sid[j]) * a.expert_bytes + a.gu_part_bytes +
                     static_cast<int64_t>(c) * QD::CHUNK,
                 QD::CHUNK, &bar_dn[j]);
    };
    const bool late_down = i1 > i0;
    if (!late_down && has_down && tid >= 32 && tid < 32 + a.topk) issue_down(tid - 32);

    // x_norm's digits, from its split copy, while the routed chunks are on their way (off
    // the path to the ids); the barrier orders them before the MMAs
#pragma unroll
    for (int i = 0; i < XPT; ++i) {
        const int k = i * kMoeThreads + tid;
        if (k < K) {
            const int kp = k ^ 32;
            vgroup_build(xvf, xvg, k, xsr[((k & 7) < 4 ? 0 : K / 2) + (k >> 3) * 4 + (k & 3)],
                         xsr[((kp & 7) < 4 ? 0 : K / 2) + (kp >> 3) * 4 + (kp & 3)]);
        }
    }
    __syncthreads();

    // ---- phase 2: gate/up on the tensor cores.  Four warps per item (item k to warp
    // group k % 4), each a quarter of the scale groups; the group's partial rows meet in
    // shared memory and its first warp forms h = SiLU(gate) * up for the item's 8 rows ----
    {
        constexpr int NSU = (NGU + 3) / 4;  // sets of four groups per row
        const int grp = warp >> 2, qw = warp & 3;
        const uint4* vf = reinterpret_cast<const uint4*>(xvf);
        float* part = s_part + grp * 64;  // [quarter][16 rows]
        for (int k = grp; k < i1 - i0; k += 4) {
            const int item = i0 + k;
            const int j = item / a.gu_chunks, cc = item % a.gu_chunks;
            const bool ok = mbar_wait_bounded(&bar_up[k], 0, a.err, nullptr);
            if (k == 0) trace_stamp(ct, 3);  // the CTA's first item landed
            if (late_down && k == 0 && warp == 0 && has_down && lane < a.topk) issue_down(lane);
            const uint8_t* chunk = up_s + static_cast<size_t>(k) * QU::CHUNK;
            float ya = 0.0f, yb = 0.0f;  // rows lane/4 and lane/4 + 8, group lane % 4 of each set
            if (ok) {
#pragma unroll 1
                for (int S = qw; S < NSU; S += 4)
                    q4_set_mma<K>(chunk, vf, xvg, S, NGU - 4 * S < 4 ? NGU - 4 * S : 4, lane, ya, yb);
            }
            ya += __shfl_xor_sync(0xffffffffu, ya, 1);
            yb += __shfl_xor_sync(0xffffffffu, yb, 1);
            ya += __shfl_xor_sync(0xffffffffu, ya, 2);
            yb += __shfl_xor_sync(0xffffffffu, yb, 2);
            if ((lane & 3) == 0) {
                part[qw * 16 + (lane >> 2)] = ya;
                part[qw * 16 + (lane >> 2) + 8] = yb;
            }
            named_bar_sync(1 + grp, 128);
            if (qw == 0 && lane < 8) {  // rows 0..7 are gate rows, 8..15 the matching up rows
                const float gt = ((part[lane] + part[16 + lane]) + part[32 + lane]) + part[48 + lane];
                const float up = ((part[8 + lane] + part[24 + lane]) + part[40 + lane]) + part[56 + lane];
                __stcg(a.h + j * a.I + 8 * cc + lane, silu_f(gt) * up);
            }
            named_bar_sync(1 + grp, 128);  // the group's partial rows are reused by its next item
        }
    }
    // the rest of the next kernel's weights, once this CTA's routed gate/up bytes are in
    if (warp == 1 && a.l2_next) {
        const uint64_t first = (a.l2_next_bytes * kMoeL2First / 4) & ~static_cast<uint64_t>(15);
        prefetch_l2_share(a.l2_next + first, a.l2_next_bytes - first, c, nblk, lane);
    }
    __syncthreads();
    trace_stamp(tr, 6);
    trace_stamp(ct, 4);
    if (tid == 0) {
        const unsigned long long target = (s_gen + 1) * static_cast<unsigned long long>(nblk);
        red_release_add_u64(a.arrivals, 1ull);
        if (has_down) {
            spin_geq_u64(a.arrivals, target, a.err);
            // every CTA's h (written before its release) into shared memory: the acquire above
            // orders those writes before this thread's bulk (async-proxy) read
            const uint32_t hb = static_cast<uint32_t>(nexp * KI * 4);
            asm volatile("fence.proxy.async.global;" ::: "memory");
            fence_proxy_async_smem();  // phase 1b's generic accesses of the region (before the barrier above)
            mbar_arrive_expect_tx(&bar_h, hb);
            bulk_g2s(h4, a.h, hb, &bar_h);
        }
    }
    __syncthreads();
    trace_stamp(tr, 7);
    trace_stamp(ct, 5);
    if (ct) {
        unsigned smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        ct[7] = smid;
    }

    // ---- phase 3: this CTA's 16 output rows (16c .. 16c + 15) over every selected
    // expert, on the tensor cores.  h of each expert becomes vector fragments; the units
    // (expert, up to four scale groups) are spread over the 16 warps; each adds
    // p_j * (its 16 rows against h_j), p_j the router probability (the shared expert: its
    // sigmoid gate); warp 0 sums the warps' partial rows in warp order + residual ----
    if (has_down) {
        constexpr int SETS = (NGD + 3) / 4;  // units per expert
        constexpr int VFB = vfrag_bytes(KI);
        const int nh = nexp * KI;
        // h of every expert (landed by the bulk copy issued at the barrier), then expert j's
        // fragments at hvf + j * VFB and scale groups at hvg + j * NGD
        const float* hfl = h4;
        int8_t* hvf = reinterpret_cast<int8_t*>(h4 + nh);
        VGroup* hvg = reinterpret_cast<VGroup*>(hvf + nexp * VFB);
        const bool okh = mbar_wait_bounded(&bar_h, 0, a.err, nullptr);
        // a warp's 32 consecutive t lie in one scale group of one expert (KI % 64 == 0), and
        // t ^ 32 is the other half of that group
#pragma unroll 3
        for (int t = tid; t < nh; t += kMoeThreads)
            vgroup_build(hvf + (t / KI) * VFB, hvg + (t / KI) * NGD, t % KI, okh ? hfl[t] : 0.0f,
                         okh ? hfl[t ^ 32] : 0.0f);
        __syncthreads();
        uint64_t* td = (tr && c == 0) ? tr + 40 : nullptr;  // down-phase detail of CTA 0 (slots 56..59)
        trace_stamp(td, 0);
        const bool okl = lane < nexp ? mbar_wait_bounded(&bar_dn[lane], 0, a.err, nullptr) : true;
        const bool ok = __all_sync(0xffffffffu, okl);  // lane j waited for expert j's chunk
        trace_stamp(td, 1);
        const long long cyc0 = clock64();
        float acc0 = 0.0f, acc1 = 0.0f;  // rows lane/4 and lane/4 + 8
        if (ok) {
#pragma unroll 1
            for (int u = warp; u < nexp * SETS; u += kMoeThreads / 32) {
                const int j = u / SETS, S = u % SETS;
                float ya = 0.0f, yb = 0.0f;
                q4_set_mma<KI>(dn_s + static_cast<size_t>(j) * QD::CHUNK, reinterpret_cast<const uint4*>(hvf + j * VFB),
                               hvg + j * NGD, S, NGD - 4 * S < 4 ? NGD - 4 * S : 4, lane, ya, yb);
                const float pj = j < a.topk ? sp[j] : sp[a.topk];
                acc0 = fmaf(pj, ya, acc0);
                acc1 = fmaf(pj, yb, acc1);
            }
        }
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
        if ((lane & 3) == 0) {
            s_part[warp * 16 + (lane >> 2)] = acc0;
            s_part[warp * 16 + (lane >> 2) + 8] = acc1;
        }
        __syncthreads();
        if (warp == 0 && lane < 16) {
            float acc = 0.0f;
#pragma unroll
            for (int w = 0; w < kMoeThreads / 32; ++w) acc += s_part[w * 16 + lane];
            a.x_out[16 * c + lane] = acc + xm_row;
        }
        trace_stamp(td, 2);
        if (td) td[3] = static_cast<uint64_t>(clock64() - cyc0);  // down compute, SM cycles (slot 59)
    }

    __syncthreads();
    trace_stamp(tr, 8);
    trace_stamp(ct, 6);
    kt_end(a.kt);
}

template <int K, int KI, int G>
static cudaError_t launch_moe_fused_t(const LaunchCfg& lc, MoeFusedArgs a) {
    const int nexp = a.topk + 1;
    const int grid = lc.num_sms;
    const int n_items = nexp * a.gu_chunks;
    a.up_slots = (n_items + grid - 1) / grid;
    if (a.up_slots > kMoeMaxSlots || a.d_chunks > grid || (a.E + 16) / 16 > grid || a.E > kMoeMaxE || a.topk > a.E)
        return cudaErrorInvalidValue;
    if (a.cta_trace && grid * kTrMoeCtaSlots > kTraceSlots - kTrMoeCta) a.cta_trace = nullptr;
    const size_t smem = MoeFusedSmem<K, KI, G>::total(a.up_slots, nexp, a.E);
    return launch_kernel(lc, moe_fused_kernel<K, KI, G>, dim3(grid), dim3(kMoeThreads), smem, a);
}

cudaError_t launch_moe_fused(const LaunchCfg& lc, const Dims& d, const LayerW& w, const Buffers& b, int slot,
                             const void* l2_next, uint64_t l2_next_bytes) {
    MoeFusedArgs a{};
    a.l2_next = static_cast<const uint8_t*>(l2_next);
    a.l2_next_bytes = l2_next ? l2_next_bytes : 0;
    a.Wr = w.w_router;
    a.rbias = w.router_bias;
    a.gamma = w.post_norm;
    a.eps = d.eps;
    a.x_mid = b.xmid + static_cast<size_t>(slot) * d.H;
    a.x_out = b.xres + static_cast<size_t>(slot) * d.H;
    a.xn_out = b.xn;
    a.experts = w.experts;
    a.shared = w.shared;
    a.expert_bytes = d.expert_bytes;
    a.gu_part_bytes = static_cast<int64_t>(d.gu_chunks) * d.gu_chunk_bytes;
    a.E = d.E;
    a.topk = d.topk;
    a.I = d.I;
    a.gu_chunks = d.gu_chunks;
    a.d_chunks = d.d_chunks;
    a.lslots = b.rslots;
    a.ids = b.topk_ids;
    a.probs = b.topk_p;
    a.shared_g = b.shared_g;
    a.h = b.h;
    a.arrivals = reinterpret_cast<unsigned long long*>(b.counters + kCntMoeSync);
    a.trace = b.trace ? b.trace + kTrMoe : nullptr;
    a.cta_trace = b.trace ? b.trace + kTrMoeCta : nullptr;
    a.kt = lc.kt;
    a.err = b.err;
    if (d.G != 64) return cudaErrorInvalidValue;
    if (d.H == 2048 && d.I == 512) return launch_moe_fused_t<2048, 512, 64>(lc, a);
    if (d.H == 256 && d.I == 128) return launch_moe_fused_t<256, 128, 64>(lc, a);
    if (d.H == 1024 && d.I == 256) return launch_moe_fused_t<1024, 256, 64>(lc, a);
    if (d.H == 2048 && d.I == 256) return launch_moe_fused_t<2048, 256, 64>(lc, a);
    if (d.H == 4096 && d.I == 512) return launch_moe_fused_t<4096, 512, 64>(lc, a);
    return cudaErrorInvalidValue;
}

#define DM_MOE_INSTANCES(X) X(2048, 512) X(256, 128) X(1024, 256) X(2048, 256) X(4096, 512)

template <int K, int KI, int G>
static cudaError_t moe_fused_fits_t(const Dims& d, int num_sms, bool* ok) {
    const int nexp = d.topk + 1;
    const int up_slots = (nexp * d.gu_chunks + num_sms - 1) / num_sms;
    *ok = false;
    if (up_slots > kMoeMaxSlots || d.d_chunks > num_sms || (d.E + 16) / 16 > num_sms || d.E > kMoeMaxE ||
        d.topk > d.E)
        return cudaSuccess;
    int per_sm = 0;
    const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &per_sm, moe_fused_kernel<K, KI, G>, kMoeThreads, MoeFusedSmem<K, KI, G>::total(up_slots, nexp, d.E));
    *ok = e == cudaSuccess && per_sm >= 1;
    return e;
}

// The fused kernel runs one CTA per SM and its phases wait on each other across the
// grid, so every CTA must be able to be resident at once: true when one CTA (with this
// shape's shared memory) fits on an SM and the grid covers the work.  An unsupported
// shape gives false.
cudaError_t moe_fused_fits(const Dims& d, int num_sms, bool* ok) {
    *ok = false;
    if (d.G != 64) return cudaSuccess;
#define DM_MOE_FITS(KK, II) \
    if (d.H == KK && d.I == II) return moe_fused_fits_t<KK, II, 64>(d, num_sms, ok);
    DM_MOE_INSTANCES(DM_MOE_FITS)
#undef DM_MOE_FITS
    return cudaSuccess;
}

cudaError_t moe_set_attrs() {
    cudaError_t e = cudaSuccess;
#define DM_MOE_FUSED_ATTR(KK, II)                                                                        \
    if (e == cudaSuccess)                                                                                \
        e = cudaFuncSetAttribute(moe_fused_kernel<KK, II, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 200 * 1024);
    DM_MOE_INSTANCES(DM_MOE_FUSED_ATTR)
#undef DM_MOE_FUSED_ATTR
    return e;
}

// ---------------------------------------------------------------------------------------
// Stand-alone dequantisation of a canonical (row-major, unchunked) 4-bit tensor.
__global__ void dequant_q4_kernel(const uint8_t* q, const uint16_t* s, const uint8_t* z, int rows,
                                  int cols, int group, float* out) {
    const int64_t n = static_cast<int64_t>(rows) * cols;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / cols;
        const int c = static_cast<int>(i % cols);
        const uint8_t byte = q[r * (cols / 2) + c / 2];
        const int qv = (c & 1) ? (byte >> 4) : (byte & 15);
        const int g = c / group;
        const int ng = cols / group;
        const uint8_t zb = z[r * (ng / 2) + g / 2];
        const int zv = (g & 1) ? (zb >> 4) : (zb & 15);
        const float sc = __half2float(__ushort_as_half(s[r * ng + g]));
        out[i] = sc * static_cast<float>(qv - zv);
    }
}

// The reference's own custom 4-bit format (src/quant/dequant_kernel.mojo:22-121): signed
// two's-complement nibbles in [-7, 7], low nibble first, one fp16 scale per group of G
// elements; w = fp32(s_g) * q, written as bf16 by one round-to-nearest-even and/or as fp32.
// Thread t handles packed bytes [8t, 8t + 8) (elements [16t, 16t + 16), inside one group
// since G >= 32).  A reserved nibble 0b1000 sets *bad; the host then discards the output.
__global__ void dequant_sym4_kernel(const uint2* __restrict__ packed, const uint16_t* __restrict__ scales,
                                    int64_t n16, int group, uint4* __restrict__ out_bf16,
                                    float4* __restrict__ out_f32, unsigned* bad) {
    const int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (t >= n16) return;
    const uint2 raw = packed[t];
    const float s = __half2float(__ushort_as_half(scales[(t * 16) / group]));
    float y[16];
    bool reserved = false;
#pragma unroll
    for (int b = 0; b < 8; ++b) {
        const uint32_t byte = ((b < 4 ? raw.x : raw.y) >> (8 * (b & 3))) & 0xFFu;
        const int lo = static_cast<int>(byte << 28) >> 28;  // sign-extended low nibble
        const int hi = static_cast<int>(byte << 24) >> 28;  // sign-extended high nibble
        reserved |= (lo == -8) | (hi == -8);
        y[2 * b] = s * static_cast<float>(lo);
        y[2 * b + 1] = s * static_cast<float>(hi);
    }
    if (reserved) atomicOr(bad, 1u);
    if (out_bf16) {
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i)
            w[i] = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(y[2 * i]))) |
                   (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(y[2 * i + 1]))) << 16);
        out_bf16[2 * t] = make_uint4(w[0], w[1], w[2], w[3]);
        out_bf16[2 * t + 1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
    if (out_f32)
#pragma unroll
        for (int i = 0; i < 4; ++i) out_f32[4 * t + i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
}

cudaError_t launch_dequant_sym4(cudaStream_t st, const uint8_t* packed, const uint16_t* scales, int64_t n, int group,
                                uint16_t* out_bf16, float* out_f32, unsigned* bad) {
    const int64_t n16 = n / 16;
    const int64_t blocks = (n16 + 255) / 256;
    dequant_sym4_kernel<<<static_cast<unsigned>(blocks), 256, 0, st>>>(
        reinterpret_cast<const uint2*>(packed), scales, n16, group, reinterpret_cast<uint4*>(out_bf16),
        reinterpret_cast<float4*>(out_f32), bad);
    return cudaGetLastError();
}

cudaError_t launch_dequant_q4_canonical(cudaStream_t st, const uint8_t* q, const uint16_t* s,
                                        const uint8_t* z, int rows, int cols, int group, float* out) {
    const int64_t n = static_cast<int64_t>(rows) * cols;
    int blocks = static_cast<int>((n + 255) / 256);
    if (blocks > 4096) blocks = 4096;
    dequant_q4_kernel<<<blocks, 256, 0, st>>>(q, s, z, rows, cols, group, out);
    return cudaGetLastError();
}

// Canonical rows -> chunked expert record (see dm_internal.h).  One block per source row.
__global__ void repack_rows_kernel(const uint8_t* q, const uint16_t* s, const uint8_t* z, int rows,
                                   int cols, int group, int kind, uint8_t* dst) {
    const int r = blockIdx.x;
    if (r >= rows) return;
    const int ng = cols / group;
    const int qb = cols / 2, sb = ng * 2, zb = ng / 2;
    const int64_t chunk_bytes = 16LL * (qb + sb + zb);
    int chunk, rin;
    if (kind == DM_PROJ_DOWN) {
        chunk = r / 16;
        rin = r % 16;
    } else {
        chunk = r / 8;
        rin = (kind == DM_PROJ_UP ? 8 : 0) + r % 8;
    }
    uint8_t* cbase = dst + chunk * chunk_bytes;
    for (int i = threadIdx.x; i < qb; i += blockDim.x) cbase[rin * qb + i] = q[static_cast<int64_t>(r) * qb + i];
    uint16_t* sdst = reinterpret_cast<uint16_t*>(cbase + 16 * qb);
    for (int i = threadIdx.x; i < ng; i += blockDim.x) sdst[rin * ng + i] = s[static_cast<int64_t>(r) * ng + i];
    uint8_t* zdst = cbase + 16 * qb + 16 * sb;
    for (int i = threadIdx.x; i < zb; i += blockDim.x) zdst[rin * zb + i] = z[static_cast<int64_t>(r) * zb + i];
}

cudaError_t launch_repack_rows(cudaStream_t st, const uint8_t* q, const uint16_t* s, const uint8_t* z,
                               int rows, int cols, int group, int kind, uint8_t* dst) {
    repack_rows_kernel<<<rows, 128, 0, st>>>(q, s, z, rows, cols, group, kind, dst);
    return cudaGetLastError();
}

}  // namespace dm
