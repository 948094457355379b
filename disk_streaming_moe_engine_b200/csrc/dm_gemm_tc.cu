// dm_gemm_tc.cu — the dense projections of the batched decode step on the 5th-generation
// tensor cores (tcgen05, accumulators in tensor memory), both operands fed by TMA.
//
// Reference: the dense projections inside forward_gdn_block (src/layers/gdn.mojo:897:
// in_proj qkv/z/a/b, out_proj) and forward_attention_qwen36 (src/layers/attention.mojo:219:
// q/k/v and o projections), and the lm_head of gguf_logits_from_hidden
// (gguf_port_loader.mojo:291), for the n rows of a batched step.
//
// C[col][row] = sum_k X[col][k] W[row][k]: W is a bf16 weight matrix [N][K] (row-major as
// loaded), X the step's operand rows [2n][K] in bf16 (rows 0..n-1 = hi(x), n..2n-1 =
// lo(x), x = hi + lo to 2^-16; written by the prep kernels), C fp32.  The weight rows are
// the MMA's M (128 per tile), the operand rows its N (2n rounded up to 16, <= 128 per column
// tile), so the weights stream from HBM once per step whatever n is.
//
// Work: an item is one 128-row weight tile, one 128-row column tile of the operand (one for
// a decode step; a prefill chunk of up to 512 rows has up to 8, the items of one weight tile
// adjacent so that its re-reads hit L2) and one of S slices of K; CTAs (one per SM,
// persistent) take items c, c + grid, ...  S is chosen per GEMM so that the items fill the
// SMs' waves (a 2048-row output projection has only 16 tiles), and each slice writes its own
// fp32 partial C_s; the kernels that consume C add the S partials (and hi + lo) in a fixed
// order: the result does not depend on timing (no atomics).
//
// Roles (192 threads): warp 0 producer (one thread: per stage of 128 K columns, two TMA boxes
// of the weight tile and two of the operand rows, 128-byte swizzle), warp 1 MMA (one thread:
// 8 tcgen05.mma per stage, M = 128, N = 2n rounded to 16, K = 16, bf16 -> fp32, one commit
// per stage that frees it, one per item that hands the accumulator on; it also allocates the
// tensor memory), warps 2-5 epilogue (warp w reads lanes 32 (w % 4) .. of the item's
// accumulator, 16 columns at a time, and stores C_s rows coalesced).  Stages: 3 x 64 KB;
// accumulators: 2 x 128 columns.  Every wait is bounded (1 s): on a timeout the kernel sets
// the error bit, the roles stop, the producer waits for its copies in flight, the MMA thread
// for its MMAs, and the tensor memory is freed.  No operand is ever another GPU's memory.
#include <cuda.h>

#include "dm_kernels.h"
#include "dm_tc.cuh"

namespace dm {

constexpr int kGtThreads = 192;
constexpr int kGtStages = 3;
constexpr int kGtKB = 128;                 // K columns per stage (two 64-column boxes)
constexpr int kGtA = 128 * kGtKB * 2;      // weight bytes per stage
constexpr int kGtB = 128 * kGtKB * 2;      // operand bytes per stage (N <= 128 rows)
constexpr int kGtStage = kGtA + kGtB;
constexpr int kGtAcc = 2;
constexpr size_t kGtSmem = static_cast<size_t>(kGtStages) * kGtStage + 1024;

struct TcGemmArgs {
    CUtensorMap wmap;   // W [N][K] bf16: dims {K, N}, box {64, 128}, 128-byte swizzle
    CUtensorMap xmap;   // X [rows][K] bf16: dims {K, rows}, box {64, ntile}, 128-byte swizzle
    float* c;           // [S][ncols][N] fp32 partials
    int N, K, ncols, ntile, tiles, ctiles, splits;
    uint32_t* err;
};

DM_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__global__ void __launch_bounds__(kGtThreads, 1) tc_gemm_kernel(const __grid_constant__ TcGemmArgs a) {
    extern __shared__ __align__(1024) uint8_t gsm_raw[];
    uint8_t* sm = gsm_raw + ((1024u - (smem_u32(gsm_raw) & 1023u)) & 1023u);
    __shared__ __align__(8) uint64_t full[kGtStages], empty[kGtStages], acc_full[kGtAcc], acc_empty[kGtAcc], done_bar;
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    volatile int* abort_flag = &s_abort;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kGtStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < kGtAcc; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 128);
        }
        mbar_init(&done_bar, 1);
        mbar_fence_init();
        s_abort = 0;
    }
    if (warp == 1) tc_alloc(&s_tmem, kGtAcc * 128);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s_tmem;
    const int nitems = a.tiles * a.ctiles * a.splits;
    const int kb_total = a.K / kGtKB;

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            uint32_t si = 0, sph = 0, issued = 0;
            const uint32_t bbytes = static_cast<uint32_t>(a.ntile) * kGtKB * 2;
            bool ok = true;
            // The weights do not depend on the kernel before: the first item's first stages
            // (as many as the ring holds) get their weight boxes before griddepcontrol.wait,
            // so they stream while that kernel finishes; their operand boxes follow the wait.
            int pre = 0;
            if (blockIdx.x < nitems) {
                const int item = blockIdx.x;
                const int tile = item / (a.ctiles * a.splits), sp = item % a.splits;
                const int kb0 = sp * kb_total / a.splits, kb1 = (sp + 1) * kb_total / a.splits;
                pre = min(kb1 - kb0, kGtStages);
                for (int p = 0; p < pre; ++p) {  // fresh stages: no empty wait
                    uint8_t* st = sm + p * kGtStage;
                    mbar_arrive_expect_tx(&full[p], kGtA + bbytes);
                    tma_load_2d(st, &a.wmap, (kb0 + p) * kGtKB, tile * 128, &full[p]);
                    tma_load_2d(st + kGtA / 2, &a.wmap, (kb0 + p) * kGtKB + 64, tile * 128, &full[p]);
                }
            }
            pdl_wait();  // the operand rows come from the kernel before
            pdl_launch_dependents();
            for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
                const int tile = item / (a.ctiles * a.splits), ct = (item / a.splits) % a.ctiles, sp = item % a.splits;
                // slice sp of K: [sp kbt / S, (sp + 1) kbt / S), at least 2 stages (S <= kbt / 2)
                const int kb0 = sp * kb_total / a.splits, kb1 = (sp + 1) * kb_total / a.splits;
                for (int kb = kb0; kb < kb1; ++kb) {
                    uint8_t* st = sm + si * kGtStage;
                    if (pre > 0) {  // weights already in flight: the operand boxes only
                        --pre;
                    } else {
                        if (!(ok = mbar_wait_bounded(&empty[si], sph ^ 1u, a.err, abort_flag))) break;
                        mbar_arrive_expect_tx(&full[si], kGtA + bbytes);
                        tma_load_2d(st, &a.wmap, kb * kGtKB, tile * 128, &full[si]);
                        tma_load_2d(st + kGtA / 2, &a.wmap, kb * kGtKB + 64, tile * 128, &full[si]);
                    }
                    tma_load_2d(st + kGtA, &a.xmap, kb * kGtKB, ct * 128, &full[si]);
                    tma_load_2d(st + kGtA + bbytes / 2, &a.xmap, kb * kGtKB + 64, ct * 128, &full[si]);
                    ++issued;
                    if (++si == kGtStages) {
                        si = 0;
                        sph ^= 1u;
                    }
                }
            }
            for (uint32_t u = issued > kGtStages ? issued - kGtStages : 0; u < issued; ++u)
                mbar_wait_bounded(&full[u % kGtStages], (u / kGtStages) & 1u, a.err, nullptr);
        }
    } else if (warp == 1) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            uint32_t si = 0, sph = 0, di = 0, dph = 0;
            const uint32_t idesc = tc_idesc_bf16(128, a.ntile);
            const uint32_t bbytes = static_cast<uint32_t>(a.ntile) * kGtKB * 2;
            bool ok = true;
            for (int item = blockIdx.x; item < nitems && ok; item += gridDim.x) {
                const int sp = item % a.splits;
                const int kb0 = sp * kb_total / a.splits, kb1 = (sp + 1) * kb_total / a.splits;
                if (!mbar_try_wait(&acc_empty[di], dph ^ 1u) &&
                    !(ok = mbar_wait_bounded(&acc_empty[di], dph ^ 1u, a.err, abort_flag)))
                    break;
                const uint32_t d = tmem + di * 128;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_try_wait(&full[si], sph) && !(ok = mbar_wait_bounded(&full[si], sph, a.err, abort_flag)))
                        break;
                    tc_fence_after();
                    const uint32_t st = smem_u32(sm + si * kGtStage);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint64_t ad = tc_desc_sw128(st + h * (kGtA / 2));
                        const uint64_t bd = tc_desc_sw128(st + kGtA + h * (bbytes / 2));
#pragma unroll
                        for (int k = 0; k < 4; ++k) tc_mma_bf16(d, ad + 2 * k, bd + 2 * k, idesc, kb > kb0 || h > 0 || k > 0);
                    }
                    tc_commit(&empty[si]);
                    if (++si == kGtStages) {
                        si = 0;
                        sph ^= 1u;
                    }
                }
                if (!ok) break;
                tc_commit(&acc_full[di]);
                if (++di == kGtAcc) {
                    di = 0;
                    dph ^= 1u;
                }
            }
            tc_commit(&done_bar);
            mbar_wait_bounded(&done_bar, 0, a.err, nullptr);
        }
    } else {
        // ---------------- epilogue: accumulator -> C_s ----------------
        const int sp4 = warp & 3;
        const int r = 32 * sp4 + lane;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(32 * sp4) << 16);
        uint32_t di = 0, dph = 0;
        for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
            const int tile = item / (a.ctiles * a.splits), ct = (item / a.splits) % a.ctiles, sp = item % a.splits;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&acc_full[di], dph, a.err, abort_flag))) break;
            tc_fence_after();
            const int row = tile * 128 + r;
            float* cs = a.c + (static_cast<size_t>(sp) * a.ncols + ct * 128) * a.N;
            const int nc = min(a.ntile, a.ncols - ct * 128);  // columns of this tile
            for (int c0 = 0; c0 < nc; c0 += 16) {
                float v[16];
                tc_ld16(lane_base + di * 128 + c0, v);
                tc_wait_ld();
                if (row < a.N) {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (c0 + j < nc) cs[static_cast<size_t>(c0 + j) * a.N + row] = v[j];
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[di]);
            if (++di == kGtAcc) {
                di = 0;
                dph ^= 1u;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tc_dealloc(tmem, kGtAcc * 128);
    }
}

cudaError_t tc_gemm_set_attrs() {
    return cudaFuncSetAttribute(tc_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kGtSmem));
}

// Slices of K for `tiles` weight tiles: the count (<= max_splits, at least 2 stages each)
// whose items fill the SMs' waves best; ties to fewer slices.
int tc_gemm_splits(int tiles, int K, int num_sms, int max_splits) {
    const int kbt = K / kGtKB;
    int best = 1;
    double best_eff = 0.0;
    for (int s = 1; s <= max_splits && (s == 1 || s <= kbt / 2); ++s) {
        const int items = tiles * s;
        const int waves = (items + num_sms - 1) / num_sms;
        const double eff = static_cast<double>(items) / (static_cast<double>(waves) * num_sms);
        if (eff > best_eff + 1e-9) {
            best_eff = eff;
            best = s;
        }
    }
    return best;
}

cudaError_t launch_tc_gemm(const LaunchCfg& lc, const void* wmap, const void* xmap, float* c, int N, int K, int ncols,
                           int splits, uint32_t* err) {
    if (ncols < 1 || ncols > 2 * kPfMaxRows || K % kGtKB != 0 || splits < 1) return cudaErrorInvalidValue;
    TcGemmArgs a{};
    a.wmap = *static_cast<const CUtensorMap*>(wmap);
    a.xmap = *static_cast<const CUtensorMap*>(xmap);
    a.c = c;
    a.N = N;
    a.K = K;
    a.ncols = ncols;
    a.ntile = ncols > 128 ? 128 : (ncols + 15) / 16 * 16;
    a.tiles = (N + 127) / 128;
    a.ctiles = (ncols + 127) / 128;
    a.splits = splits;
    if (splits > 1 && splits > K / kGtKB / 2) return cudaErrorInvalidValue;
    a.err = err;
    const int items = a.tiles * a.ctiles * splits;
    const int grid = items < lc.num_sms ? items : lc.num_sms;
    return launch_kernel(lc, tc_gemm_kernel, dim3(grid), dim3(kGtThreads), kGtSmem, a);
}

}  // namespace dm
