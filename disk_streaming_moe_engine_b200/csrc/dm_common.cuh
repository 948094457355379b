// dm_common.cuh — device helpers shared by every kernel of libdismoen_cuda.so (sm_100a).
//
//  * 1-D bulk copies (cp.async.bulk, the TMA engine's untiled mode) completing on
//    shared-memory mbarriers, never with cluster multicast;
//  * bounded mbarrier waits: every wait gives up after DM_WAIT_NS of %globaltimer time,
//    raises DM_DEVERR_TIMEOUT in the context's error word and lets the kernel finish;
//  * programmatic dependent launch (griddepcontrol) so that a kernel can stream its
//    weights while the previous kernel of the decode step is still running.
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "dm_internal.h"
#include "dm_kernels.h"

#define DM_DEV __device__ __forceinline__

namespace dm {

constexpr uint64_t DM_WAIT_NS = 1000000000ull;  // 1 s bound on any device-side wait

DM_DEV uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Phase trace: stamp slot k with %globaltimer when tracing is on (tr != nullptr).
DM_DEV void trace_stamp(uint64_t* tr, int k) {
    if (tr) tr[k] = globaltimer_ns();
}

// Launch timeline: CTA (0,0) stamps its start and the end of griddepcontrol.wait; every
// CTA folds its finish time into the record's end with atomicMax.
DM_DEV bool kt_lead() { return blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0; }
DM_DEV void kt_start(uint64_t* kt) {
    if (kt && kt_lead()) kt[0] = globaltimer_ns();
}
DM_DEV void kt_ready(uint64_t* kt) {
    if (kt && kt_lead()) kt[1] = globaltimer_ns();
}
DM_DEV void kt_end(uint64_t* kt) {  // call from thread 0 of the CTA once its work is done
    if (kt && threadIdx.x == 0)
        atomicMax(reinterpret_cast<unsigned long long*>(&kt[2]), static_cast<unsigned long long>(globaltimer_ns()));
}

DM_DEV void raise_error(uint32_t* err, uint32_t code) {
    if (err) atomicOr(err, code);
}

// ---- programmatic dependent launch -------------------------------------------------
// wait: blocks until every grid this one depends on has completed and its writes are
// visible.  launch_dependents: lets the next kernel in the stream be scheduled.
DM_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
DM_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// Named barrier over `count` threads (multiple of 32) that excludes the other warps.
DM_DEV void named_bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ---- shared-memory address helpers ---------------------------------------------------
DM_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ----------------------------------------------------------------------
DM_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
DM_DEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

DM_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}
DM_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}
DM_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for phase `parity` of `bar`.  Returns false (and raises the timeout bit)
// if DM_WAIT_NS elapsed; `abort_flag` (shared) short-circuits waits after a failure.
DM_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t* err,
                              volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = globaltimer_ns();
    uint32_t polls = 0;
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (++polls % 64 == 0) {
            if (abort_flag && *abort_flag) return false;
            if (globaltimer_ns() - t0 > DM_WAIT_NS) {
                raise_error(err, DM_DEVERR_TIMEOUT);
                if (abort_flag) *abort_flag = 1;
                return false;
            }
        }
    }
}

// ---- grid-wide flags (kernels whose CTAs are all co-resident) ----------------------
DM_DEV unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
DM_DEV void red_release_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// 64-bit grid counters that are never reset: a launch reads the count before it
// arrives itself and waits for (count / grid + 1) * grid.
DM_DEV unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
DM_DEV unsigned long long ld_relaxed_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
DM_DEV void red_release_add_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Bounded wait until *p >= target (64-bit counter); false on timeout.
DM_DEV bool spin_geq_u64(const unsigned long long* p, unsigned long long target, uint32_t* err) {
    if (ld_acquire_u64(p) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t n = 1;; ++n) {
        if (ld_acquire_u64(p) >= target) return true;
        if (n % 256 == 0 && globaltimer_ns() - t0 > DM_WAIT_NS) {
            raise_error(err, DM_DEVERR_TIMEOUT);
            return false;
        }
    }
}

// Bounded wait until *p >= target (thread-level; callers use one thread per CTA).
DM_DEV bool spin_geq(const unsigned* p, unsigned target, uint32_t* err) {
    if (ld_acquire_u32(p) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    uint32_t n = 0;
    while (true) {
        if (ld_acquire_u32(p) >= target) return true;
        if (++n % 256 == 0 && globaltimer_ns() - t0 > DM_WAIT_NS) {
            raise_error(err, DM_DEVERR_TIMEOUT);
            return false;
        }
    }
}

// ---- bulk copy global -> shared (TMA, untiled) ----------------------------------------
// Both addresses 16-byte aligned and bytes a multiple of 16 (checked by the callers'
// layout: every chunk is a multiple of 16 bytes and every base is 256-byte aligned).
// DM_L2_HINT=1 builds the weight and KV streams (read once per step, far more bytes than
// the L2 holds) with an L2 evict-first policy.  Measured in the decode step: 0.3 % slower
// than plain loads on the same box, and again with the generation-tagged MoE flags and
// the later MoE trigger: 580.4 vs 579.9 tok/s (noise).  The kernel code that the hint was
// meant to keep hot is lost from the SM's own instruction caches, not from the L2, so it
// is off.
#ifndef DM_L2_HINT
#define DM_L2_HINT 0
#endif
DM_DEV uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
DM_DEV void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
#if DM_L2_HINT
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(l2_evict_first_policy())
        : "memory");
#else
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
#endif
}
// Orders this thread's generic-proxy accesses of shared memory before later async-proxy
// (bulk / tensor copy) writes into the same bytes.
DM_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// L2 prefetch of a global range (no shared memory involved).
DM_DEV void bulk_prefetch_l2(const void* gmem_src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gmem_src), "r"(bytes)
                 : "memory");
}

// Prefetches this CTA's share [part/nparts] of [base, base + bytes) into L2 in 64 KB bulk
// prefetches issued by threads tid < 32 (fire and forget; no shared memory involved).
DM_DEV void prefetch_l2_share(const void* base, size_t bytes, int part, int nparts, int tid) {
    if (base == nullptr || bytes == 0 || tid >= 32) return;
    const size_t per = ((bytes + nparts - 1) / nparts + 15) & ~static_cast<size_t>(15);
    const size_t b0 = per * part;
    if (b0 >= bytes) return;
    const size_t b1 = b0 + per < bytes ? b0 + per : bytes;
    constexpr size_t kPiece = 64 * 1024;
    const char* p = static_cast<const char*>(base);
    for (size_t o = b0 + tid * kPiece; o < b1; o += 32 * kPiece) {
        const size_t n = (b1 - o) < kPiece ? (b1 - o) : kPiece;
        bulk_prefetch_l2(p + o, static_cast<uint32_t>(n & ~static_cast<size_t>(15)));
    }
}

// ---- loads ---------------------------------------------------------------------------
DM_DEV uint4 ldg_nc_v4(const void* p) {
    uint4 r;
#if DM_L2_HINT
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p), "l"(l2_evict_first_policy()));
#else
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
#endif
    return r;
}

// bf16 pair (packed in a u32, element 0 in the low half) -> two floats (exact).
DM_DEV float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
DM_DEV float bf16hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

DM_DEV float bf16_to_f32(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }

// D = A B + D on the tensor cores, bf16 inputs, fp32 accumulation (m16n8k16, A row-major,
// B column-major; fragment layouts of the PTX ISA for mma.sync .m16n8k16).
DM_DEV void mma_bf16_m16n8k16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                              uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// (q_j, q_{j+4}) of a word of 8 nibbles as the bf16 pair (128 + q_j, 128 + q_{j+4}): the
// nibble becomes the low mantissa bits of 128.0, an exact integer
DM_DEV uint32_t nib_pair128(uint32_t w) { return (w & 0x000F000Fu) | 0x43004300u; }
// fp32 -> bf16 round-to-nearest-even (NaN stays NaN).
DM_DEV uint16_t f32_to_bf16(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// ---- warp reductions -----------------------------------------------------------------
// Butterfly: every lane ends with the same value; addition order is fixed
// (xor 16, 8, 4, 2, 1), so the result is deterministic.
DM_DEV float warp_sum(float v) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}
DM_DEV float warp_max(float v) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
    return v;
}

// Numerically stable logistic and SiLU (reference src/layers/swiglu.mojo:11-40).
DM_DEV float sigmoid_f(float z) {
    if (z < -88.0f) return 0.0f;
    if (z > 88.0f) return 1.0f;
    if (z < 0.0f) {
        float e = expf(z);
        return e / (1.0f + e);
    }
    return 1.0f / (1.0f + expf(-z));
}
DM_DEV float silu_f(float z) { return z * sigmoid_f(z); }
// softplus with the reference's +-20 thresholds (_gdn_softplus, gdn.mojo:889-894)
DM_DEV float softplus_ref(float v) {
    if (v > 20.0f) return v;
    if (v < -20.0f) return expf(v);
    return logf(1.0f + expf(v));
}
// GDN decay of head h: exp(-exp(A_log) * softplus(a + dt_bias))
DM_DEV float gdn_decay(float a, float a_log, float dt_bias) { return expf(-expf(a_log) * softplus_ref(a + dt_bias)); }

// ---- cp.async (per-thread asynchronous global -> shared copies) -----------------------
DM_DEV void cp_async16(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
DM_DEV void cp_async4(void* smem_dst, const void* gmem_src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
DM_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
DM_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

}  // namespace dm
