// dm_noalloc.cu — dm_moe_layer_noalloc: the fused MoE mixer of one layer over buffers the
// caller owns, with the kernel's scratch in a fixed device array compiled into the
// library.  Nothing is allocated on the device or through an allocating library routine.
//
// Why: a host runtime that streams expert records from disk into an expert cache of its
// own (the setting this engine's reference targets) commits the device memory left after
// the weights to that cache.  Such a caller cannot let a library allocate in the middle of
// a step: a cudaMalloc there may synchronise the device, fail once the cache has taken the
// memory, and hands memory to a second owner that the cache's budget does not see.  It has
// no dm_ctx either (a context allocates its own weight arena and scratch when created).
//
// Scratch (g_moe_scratch, kNoAllocScratchBytes = 64 KiB), byte offsets:
//     0  control block (512 B, cleared on the stream before every launch): the 64-word
//        counter array in the layout a context uses (phase counters and released id
//        words of the fused kernel), then the device error word at 256
//   512  router logit words [E + 1] u64 (launch tag << 32 | fp32 bits; 8 KiB for E <= 512)
//   512 + 8 KiB  top-k ids, probabilities, shared gate   (256 B)
//   then normalised input [H] fp32 and SwiGLU activations [(k + 1) * I] fp32.
// The array keeps what the last call left in it; the control block and the router logit
// words have to start at zero (the kernel's launch generation restarts at 0 with the
// control block): the entry point clears both before each launch.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "dismoen_cuda.h"
#include "dm_internal.h"
#include "dm_kernels.h"

namespace dm {

constexpr size_t kNoAllocScratchBytes = DM_NOALLOC_SCRATCH_BYTES;
constexpr size_t kCtlBytes = 512;
constexpr size_t kErrOffset = 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_moe_scratch[kNoAllocScratchBytes];

static_assert(kNoAllocScratchBytes == 65536, "the header states a 64 KiB scratch");

struct NoAllocDevice {
    bool ready;
    unsigned char* scratch;  // device address of g_moe_scratch on this device
    int num_sms;
};
static NoAllocDevice g_dev[kMaxDevices];
static std::mutex g_dev_mu;
// Held for a whole call (enqueue through the final stream synchronisation): two threads of
// one process never have this entry point's kernels in flight at once, since they would
// share the scratch array.  Calls from other processes on the same device are not covered.
static std::mutex g_call_mu;

static int na_err(char* buf, uint64_t size, int code, const char* type, const char* fmt, ...) {
    if (buf && size > 0) {
        char detail[384];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(detail, sizeof detail, fmt, ap);
        va_end(ap);
        for (char* p = detail; *p; ++p)
            if (*p == '"' || *p == '\\') *p = '\'';
        snprintf(buf, size, "{\"error_type\":\"%s\",\"detail\":\"%s\",\"stage\":\"moe_noalloc\",\"layer\":-1}", type,
                 detail);
    }
    return code;
}

static int64_t q4_chunk_bytes(int cols) {  // 16 rows: nibbles, fp16 scales, uint4 zeros (g = 64)
    const int ng = cols / 64;
    return 16LL * (cols / 2 + ng * 2 + ng / 2);
}

// Scratch bytes a layer of these dimensions needs (control block, logits, top-k, x_norm, h).
static size_t scratch_need(int H, int I, int E, int topk) {
    return kCtlBytes + 8192 + 256 + static_cast<size_t>(H) * 4 + static_cast<size_t>(topk + 1) * I * 4;
}

// Once per device, with that device current: the scratch address and the kernel attributes.
static int setup_device(int dev, NoAllocDevice* out, char* eb, uint64_t es) {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    NoAllocDevice& s = g_dev[dev];
    if (!s.ready) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_moe_scratch);
        if (e != cudaSuccess)
            return na_err(eb, es, DM_ERR_CUDA, "CUDA_ERROR", "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e == cudaSuccess) e = moe_set_attrs();
        if (e != cudaSuccess)
            return na_err(eb, es, DM_ERR_CUDA, "CUDA_ERROR", "device set-up: %s", cudaGetErrorString(e));
        s.scratch = static_cast<unsigned char*>(p);
        s.num_sms = sms;
        s.ready = true;
    }
    *out = s;
    return DM_OK;
}

}  // namespace dm

using namespace dm;

extern "C" int32_t dm_moe_layer_noalloc(int32_t H, int32_t I, int32_t E, int32_t topk, float eps,
                                        const uint16_t* router_dev, const uint16_t* post_norm_dev,
                                        const uint8_t* experts_dev, const uint8_t* shared_dev,
                                        const float* x_mid_dev, float* x_out_dev, int32_t* ids_dev,
                                        float* probs_dev, void* stream, char* err_buf, uint64_t err_buf_size) {
    if (err_buf && err_buf_size > 0) err_buf[0] = '\0';
    if (!router_dev || !post_norm_dev || !experts_dev || !shared_dev || !x_mid_dev || !x_out_dev)
        return na_err(err_buf, err_buf_size, DM_ERR_INVALID_ARG, "INVALID_ARG", "null device pointer");
    if (x_out_dev < x_mid_dev + H && x_mid_dev < x_out_dev + H)
        return na_err(err_buf, err_buf_size, DM_ERR_INVALID_ARG, "INVALID_ARG", "x_out overlaps x_mid");
    if (!(eps > 0.0f) || H <= 0 || I <= 0 || E <= 0 || topk <= 0 || topk > E || topk > kMaxTopK || E > 512 ||
        H % 64 != 0 || I % 64 != 0)
        return na_err(err_buf, err_buf_size, DM_ERR_INVALID_ARG, "CONFIG_ERROR",
                      "need eps > 0, 0 < num_experts_per_tok <= min(num_experts, 16), num_experts <= 512, "
                      "hidden and intermediate sizes multiples of 64");
    const size_t need = scratch_need(H, I, E, topk);
    if (need > kNoAllocScratchBytes)
        return na_err(err_buf, err_buf_size, DM_ERR_INVALID_ARG, "SCRATCH_LIMIT",
                      "this layer needs %zu bytes of scratch; the fixed device scratch holds %zu "
                      "(H=%d, I=%d, E=%d, k=%d)",
                      need, kNoAllocScratchBytes, H, I, E, topk);
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return na_err(err_buf, err_buf_size, DM_ERR_CUDA, "CUDA_ERROR", "no current device (%s)",
                      cudaGetErrorString(e));
    NoAllocDevice sd{};
    int rc = setup_device(dev, &sd, err_buf, err_buf_size);
    if (rc != DM_OK) return rc;
    // the call waits for its stream at the end, which a capturing stream does not allow
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &cap);
    if (e != cudaSuccess || cap != cudaStreamCaptureStatusNone)
        return na_err(err_buf, err_buf_size, DM_ERR_INVALID_ARG, "INVALID_ARG",
                      "the stream is being captured (or cannot be queried: %s); this call synchronises its stream",
                      cudaGetErrorString(e));

    Dims d{};
    d.max_seqs = 1;
    d.H = H;
    d.I = I;
    d.E = E;
    d.topk = topk;
    d.G = 64;
    d.eps = eps;
    d.gu_chunk_bytes = q4_chunk_bytes(H);
    d.d_chunk_bytes = q4_chunk_bytes(I);
    d.gu_chunks = I / 8;
    d.d_chunks = H / 16;
    d.expert_bytes = d.gu_chunks * d.gu_chunk_bytes + d.d_chunks * d.d_chunk_bytes;

    // one CTA per SM, its phases waiting on each other: the shape must have a kernel
    // instance, at most one 16-row down chunk per SM and one resident CTA on every SM
    bool fits = false;
    e = moe_fused_fits(d, sd.num_sms, &fits);
    if (e != cudaSuccess)
        return na_err(err_buf, err_buf_size, DM_ERR_CUDA, "CUDA_ERROR", "occupancy query: %s", cudaGetErrorString(e));
    if (!fits)
        return na_err(err_buf, err_buf_size, DM_ERR_INVALID_ARG, "CONFIG_ERROR",
                      "no fused MoE kernel for hidden %d / intermediate %d on %d SMs (instances (hidden, "
                      "intermediate): (256,128) (1024,256) (2048,256) (2048,512), and (4096,512) on GPUs with at "
                      "least 256 SMs; the kernel needs hidden/16 <= SMs and one resident CTA per SM)",
                      H, I, sd.num_sms);

    LayerW w{};
    w.post_norm = post_norm_dev;
    w.w_router = router_dev;
    w.experts = experts_dev;
    w.shared = shared_dev;

    unsigned char* base = sd.scratch;
    unsigned long long* lg = reinterpret_cast<unsigned long long*>(base + kCtlBytes);
    unsigned char* small = base + kCtlBytes + 8192;
    float* xn = reinterpret_cast<float*>(small + 256);
    Buffers b{};
    // x_mid / x_out are addressed as slot 0 of the mixer / residual buffers
    b.xmid = const_cast<float*>(x_mid_dev);
    b.xres = x_out_dev;
    b.xn = xn;
    b.h = xn + H;
    b.rslots = lg;
    b.topk_ids = ids_dev ? ids_dev : reinterpret_cast<int*>(small);
    b.topk_p = probs_dev ? probs_dev : reinterpret_cast<float*>(small + 64);
    b.shared_g = reinterpret_cast<float*>(small + 128);
    b.counters = reinterpret_cast<unsigned*>(base);
    static_assert(kCntMoeFlag * 4 + 4 * 8 <= kErrOffset, "counter array must end before the error word");
    b.err = reinterpret_cast<uint32_t*>(base + kErrOffset);
    b.trace = nullptr;
    b.ktrace = nullptr;

    LaunchCfg lc{};
    lc.stream = static_cast<cudaStream_t>(stream);
    lc.num_sms = sd.num_sms;
    lc.pdl = false;
    lc.kt = nullptr;

    std::lock_guard<std::mutex> call_lock(g_call_mu);
    e = cudaMemsetAsync(base, 0, kCtlBytes, lc.stream);
    // router logit words start empty (tag 0 matches no launch)
    if (e == cudaSuccess) e = cudaMemsetAsync(lg, 0, static_cast<size_t>(E + 1) * 8, lc.stream);
    if (e == cudaSuccess) e = launch_moe_fused(lc, d, w, b, 0);
    if (e != cudaSuccess)
        return na_err(err_buf, err_buf_size, e == cudaErrorInvalidValue ? DM_ERR_INVALID_ARG : DM_ERR_CUDA,
                      "CUDA_ERROR", "launch: %s", cudaGetErrorString(e));
    uint32_t word = 0;
    e = cudaMemcpyAsync(&word, base + kErrOffset, 4, cudaMemcpyDeviceToHost, lc.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(lc.stream);
    if (e != cudaSuccess)
        return na_err(err_buf, err_buf_size, DM_ERR_CUDA, "CUDA_ERROR", "%s", cudaGetErrorString(e));
    if (word & DM_DEVERR_TIMEOUT)
        return na_err(err_buf, err_buf_size, DM_ERR_TIMEOUT, "DEVICE_TIMEOUT",
                      "a bounded device wait ran out (word 0x%x)", word);
    if (word)
        return na_err(err_buf, err_buf_size, DM_ERR_NONFINITE, "NONFINITE_ERROR",
                      "non-finite value detected (word 0x%x)", word);
    return DM_OK;
}
