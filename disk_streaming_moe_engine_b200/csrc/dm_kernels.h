// dm_kernels.h — argument structs and the launch helper shared by the .cu files.
#pragma once
#include <cuda_runtime.h>

#include "dm_internal.h"

namespace dm {

enum GemvPrologue { PRO_COPY = 0, PRO_RMSNORM = 1, PRO_HEADNORM = 2 };
enum GemvAct { ACT_STORE = 0, ACT_SILU = 1, ACT_RESID = 2, ACT_ARGMAX = 3 };

// Rows [previous row_end, row_end) of the GEMV output go to `out` (local row index),
// optionally shifted to conv-ring slot (pos % 4) * ring_stride.
struct GemvSeg {
    float* out;
    const float* res;
    int row_end;
    int act;
    int ring_stride;
};

struct GemvArgs {
    const uint16_t* W;
    int N;
    // prologue inputs
    const float* x;
    const uint16_t* gamma;
    float eps;
    float* xnorm_out;
    const float* hn_o;
    const float* hn_z;
    const uint16_t* hn_w;
    int hn_dim;
    // epilogue
    GemvSeg seg[4];
    int nseg;
    const int* pos;
    // argmax (lm_head)
    float* cand_val;
    int* cand_idx;
    unsigned* counter;
    int* token_out;
    int* pos_inc;
    int* gen_out;
    int* gen_idx;
    int gen_cap;
    uint32_t* err;
    uint64_t* kt;   // timeline record (set from LaunchCfg)
    int pf;         // rows of L2 look-ahead per warp
};

cudaError_t launch_gemv(const LaunchCfg& lc, int K, int pro, const GemvArgs& a);
bool gemv_supported_k(int K);
cudaError_t gemv_set_attrs();
cudaError_t moe_set_attrs();
cudaError_t router_set_attrs();
cudaError_t attn_set_attrs(int max_scores_smem);

// Launch with the programmatic-stream-serialization attribute when lc.pdl is set, so the
// kernel may start (and stream its weights) before the previous kernel completes.
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_kernel(const LaunchCfg& lc, void (*kern)(KArgs...), dim3 grid,
                                        dim3 block, size_t smem, Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = lc.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = lc.pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

}  // namespace dm
