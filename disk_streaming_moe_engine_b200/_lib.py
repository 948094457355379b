"""ctypes binding of libdismoen_cuda.so (declarations of include/dismoen_cuda.h).

The library is loaded from the package directory only; there is no fallback: if it is
missing or cannot be loaded, `load()` raises.
"""
from __future__ import annotations

import ctypes as C
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libdismoen_cuda.so")

DM_OK = 0
DM_ERR_INVALID_ARG = 1
DM_ERR_CUDA = 2
DM_ERR_OOM = 3
DM_ERR_POSITION = 4
DM_ERR_CAPACITY = 5
DM_ERR_NONFINITE = 6
DM_ERR_TIMEOUT = 7
DM_ERR_NOT_READY = 8
DM_ERR_ROUTER = 9
DM_ERR_IO = 10
DM_ERR_FORMAT = 11

DM_KERNEL_MIXER_IN, DM_KERNEL_MIXER_OUT, DM_KERNEL_MIXER_CORE = 0, 1, 2
DM_KERNEL_ROUTER, DM_KERNEL_MOE, DM_KERNEL_HEAD = 3, 4, 6
DM_BKERNEL_ATTN, DM_BKERNEL_GDN_REC, DM_BKERNEL_EXPERTS, DM_BKERNEL_ROUTER, DM_BKERNEL_GEMM_IN = 0, 1, 2, 3, 4
DM_EP_HANDLE_BYTES = 64

DM_GGML_F32, DM_GGML_F16, DM_GGML_Q8_0, DM_GGML_Q3_K, DM_GGML_Q4_K, DM_GGML_BF16 = 0, 1, 8, 11, 12, 30
DM_GGUF_Q4K_MOJO = 1
DM_LOAD_REQUANT = 2

DM_DTYPE_BF16 = 0
DM_DTYPE_F32 = 1
DM_PROJ_GATE, DM_PROJ_UP, DM_PROJ_DOWN = 0, 1, 2

(DM_T_INPUT_NORM, DM_T_POST_NORM, DM_T_GDN_QKV, DM_T_GDN_CONV, DM_T_GDN_Z, DM_T_GDN_A, DM_T_GDN_B,
 DM_T_GDN_DT_BIAS, DM_T_GDN_A_LOG, DM_T_GDN_NORM, DM_T_GDN_OUT, DM_T_ATTN_Q, DM_T_ATTN_K, DM_T_ATTN_V,
 DM_T_ATTN_Q_NORM, DM_T_ATTN_K_NORM, DM_T_ATTN_O, DM_T_ROUTER, DM_T_SHARED_GATE, DM_T_EMBED,
 DM_T_FINAL_NORM, DM_T_LM_HEAD) = range(22)


class DmModelConfig(C.Structure):
    _fields_ = [
        ("hidden_size", C.c_int32), ("num_hidden_layers", C.c_int32),
        ("full_attention_interval", C.c_int32), ("vocab_size", C.c_int32),
        ("rms_norm_eps", C.c_float), ("num_attention_heads", C.c_int32),
        ("num_key_value_heads", C.c_int32), ("head_dim", C.c_int32), ("rope_theta", C.c_float),
        ("partial_rotary_factor", C.c_float), ("linear_num_key_heads", C.c_int32),
        ("linear_num_value_heads", C.c_int32), ("linear_key_head_dim", C.c_int32),
        ("linear_value_head_dim", C.c_int32), ("linear_conv_kernel_dim", C.c_int32),
        ("num_experts", C.c_int32), ("num_experts_per_tok", C.c_int32),
        ("moe_intermediate_size", C.c_int32), ("shared_expert_intermediate_size", C.c_int32),
        ("norm_topk_prob", C.c_int32), ("quant_group_size", C.c_int32),
    ]


class DmRuntimeConfig(C.Structure):
    _fields_ = [("max_seqs", C.c_int32), ("kv_page_tokens", C.c_int32),
                ("kv_num_pages", C.c_int32), ("max_pages_per_seq", C.c_int32),
                ("expert_cache_slots", C.c_int32)]


class DmGgufTensorInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("ndim", C.c_int32), ("ggml_type", C.c_int32),
                ("dims", C.c_uint64 * 8), ("offset", C.c_uint64), ("file_offset", C.c_uint64),
                ("num_elements", C.c_uint64), ("raw_bytes", C.c_uint64)]


class DmQuantTensorInfo(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_char_p), ("ndim", C.c_int32), ("group_size", C.c_int32),
                ("shape", C.c_uint64 * 8), ("num_groups", C.c_uint64), ("num_elements", C.c_uint64),
                ("record_offset", C.c_uint64), ("scales_offset", C.c_uint64), ("data_offset", C.c_uint64),
                ("scales_bytes", C.c_uint64), ("weights_bytes", C.c_uint64)]


P = C.c_void_p
I32 = C.c_int32
U64 = C.c_uint64
F32 = C.c_float

# symbol -> (restype, argtypes); every symbol of include/dismoen_cuda.h
SIGNATURES = {
    "dm_ctx_create": (I32, [C.POINTER(DmModelConfig), C.POINTER(DmRuntimeConfig), I32, C.POINTER(P)]),
    "dm_ctx_destroy": (I32, [P]),
    "dm_last_error": (I32, [P, C.c_char_p, U64]),
    "dm_config_validate": (I32, [C.POINTER(DmModelConfig), C.c_char_p, U64]),
    "dm_abi_version": (I32, []),
    "dm_ctx_device_bytes": (I32, [P, C.POINTER(U64)]),
    "dm_upload_tensor": (I32, [P, I32, I32, I32, P, U64]),
    "dm_expert_upload": (I32, [P, I32, I32, I32, P, P, P]),
    "dm_weights_check": (I32, [P]),
    "dm_tensor_download": (I32, [P, I32, I32, I32, P, U64]),
    "dm_expert_download": (I32, [P, I32, I32, I32, P, P, P]),
    "dm_dequant_q4": (I32, [P, P, P, P, I32, I32, I32, P]),
    "dm_dequant_sym4": (I32, [P, P, P, C.c_int64, I32, P, P]),
    "dm_seq_reset": (I32, [P, I32]),
    "dm_seq_set_page_table": (I32, [P, I32, P, I32]),
    "dm_seq_get_len": (I32, [P, I32, C.POINTER(I32)]),
    "dm_seq_set_len": (I32, [P, I32, I32]),
    "dm_kv_import": (I32, [P, I32, I32, P, P, I32]),
    "dm_kv_export": (I32, [P, I32, I32, P, P, I32]),
    "dm_gdn_state_import": (I32, [P, I32, I32, P, P]),
    "dm_gdn_state_export": (I32, [P, I32, I32, P, P]),
    "dm_router": (I32, [P, I32, P, I32, P, P, P]),
    "dm_moe_block": (I32, [P, I32, P, I32, P]),
    "dm_mixer_block": (I32, [P, I32, I32, I32, P, I32, P]),
    "dm_block_forward": (I32, [P, I32, I32, I32, P, I32, P]),
    "dm_forward": (I32, [P, I32, P, I32, P, C.POINTER(I32)]),
    "dm_prefill": (I32, [P, I32, P, I32, P, C.POINTER(I32)]),
    "dm_prefill_rows": (I32, [P, C.POINTER(I32), C.POINTER(I32)]),
    "dm_kmss_save_conv": (I32, [P, I32, C.c_char_p, C.c_char_p]),
    "dm_kmss_load_conv": (I32, [P, I32, C.c_char_p, C.c_char_p]),
    "dm_seq_copy": (I32, [P, I32, I32]),
    "dm_decode_step": (I32, [P, I32, I32, C.POINTER(I32), P]),
    "dm_generate": (I32, [P, I32, I32, I32, P]),
    "dm_enqueue_decode": (I32, [P, I32, I32]),
    "dm_set_token": (I32, [P, I32, I32]),
    "dm_sync": (I32, [P]),
    "dm_get_stream": (I32, [P, C.POINTER(P)]),
    "dm_kernels_per_step": (I32, [P, C.POINTER(I32)]),
    "dm_trace_enable": (I32, [P, I32]),
    "dm_trace_read": (I32, [P, P, I32]),
    "dm_trace_timeline": (I32, [P, P, P, I32, C.POINTER(I32)]),
    "dm_time_kernel": (I32, [P, I32, I32, I32, C.POINTER(F32), C.POINTER(U64)]),
    "dm_synth_bf16": (I32, [U64, U64, U64, F32, F32, P]),
    "dm_synth_f32": (I32, [U64, U64, U64, F32, F32, P]),
    "dm_synth_u8": (I32, [U64, U64, U64, P]),
    "dm_synth_f16_absnormal": (I32, [U64, U64, U64, F32, P]),
    "dm_synth_model_device": (I32, [P, U64]),
    "dm_moe_layer_noalloc": (I32, [I32, I32, I32, I32, F32, P, P, P, P, P, P, P, P, P, C.c_char_p, U64]),
    "dm_batch_capacity": (I32, [P, C.POINTER(I32)]),
    "dm_decode_batch": (I32, [P, P, P, I32, P, P]),
    "dm_generate_batch": (I32, [P, P, P, I32, I32, P]),
    "dm_enqueue_decode_batch": (I32, [P, P, P, I32, I32]),
    "dm_batch_read_generated": (I32, [P, I32, I32, P]),
    "dm_batch_kernels_per_step": (I32, [P, I32, C.POINTER(I32), C.POINTER(I32)]),
    "dm_synth_state_device": (I32, [P, U64, F32, F32, I32]),
    "dm_tensor_add_rank1": (I32, [P, I32, I32, P, C.c_int64, P, I32]),
    "dm_batch_stats": (I32, [P, I32, P]),
    "dm_set_router_bias": (I32, [P, I32, P, I32]),
    "dm_ep_ipc_handle": (I32, [P, P]),
    "dm_ep_attach": (I32, [P, I32, I32, P]),
    "dm_ep_detach": (I32, [P]),
    "dm_kmss_save": (I32, [P, I32, C.c_char_p, P, I32, I32, P]),
    "dm_kmss_load": (I32, [P, I32, C.c_char_p, P, I32, C.POINTER(I32)]),
    "dm_sha256": (I32, [P, U64, P]),
    "dm_spill_stats": (I32, [P, C.POINTER(C.c_uint64)]),
    "dm_spill_pin": (I32, [P, I32, I32, C.POINTER(I32)]),
    "dm_spill_simulate": (I32, [I32, I32, I32, I32, I32, I32, P, P, I32, C.POINTER(C.c_uint64), P]),
    "dm_gguf_open": (I32, [C.c_char_p, C.POINTER(P), C.c_char_p, U64]),
    "dm_gguf_close": (None, [P]),
    "dm_gguf_summary": (I32, [P, C.POINTER(C.c_uint32), C.POINTER(U64), C.POINTER(U64), C.POINTER(U64),
                              C.POINTER(U64), C.POINTER(U64)]),
    "dm_gguf_tensor": (I32, [P, C.c_int64, C.POINTER(DmGgufTensorInfo)]),
    "dm_gguf_find": (C.c_int64, [P, C.c_char_p]),
    "dm_gguf_meta_key": (I32, [P, C.c_int64, C.c_char_p, U64]),
    "dm_gguf_meta": (I32, [P, C.c_char_p, C.c_char_p, U64]),
    "dm_gguf_read": (I32, [P, C.c_int64, U64, P, U64]),
    "dm_ggml_block_spec": (I32, [I32, C.POINTER(I32), C.POINTER(I32)]),
    "dm_gguf_dequant": (I32, [P, I32, P, U64, U64, C.c_uint32, P, P]),
    "dm_gguf_load_tensor": (I32, [P, P, C.c_char_p, I32, I32, C.c_uint32]),
    "dm_gguf_load_expert": (I32, [P, P, C.c_char_p, C.c_int64, C.c_int64, I32, I32, I32, C.c_uint32,
                                  C.POINTER(F32)]),
    "dm_quant_file_open": (I32, [C.c_char_p, C.POINTER(P), C.c_char_p, U64]),
    "dm_quant_file_close": (None, [P]),
    "dm_quant_file_summary": (I32, [P, C.POINTER(I32), C.POINTER(I32), C.POINTER(C.c_int64), C.POINTER(U64),
                                    C.c_char_p, U64]),
    "dm_quant_file_tensor": (I32, [P, C.c_int64, C.POINTER(DmQuantTensorInfo)]),
    "dm_quant_file_find": (C.c_int64, [P, C.c_char_p]),
    "dm_quant_file_read": (I32, [P, C.c_int64, I32, U64, P, U64]),
    "dm_quant_file_load_tensor": (I32, [P, P, C.c_char_p, I32, I32]),
    "dm_quant_file_load_expert": (I32, [P, P, C.c_char_p, C.c_int64, C.c_int64, I32, I32, I32, C.c_uint32,
                                        C.POINTER(F32)]),
    "dm_quant_file_load": (I32, [P, P, C.c_uint32]),
    "dm_time_batch_kernel": (I32, [P, I32, I32, I32, I32, C.POINTER(F32), C.POINTER(U64)]),
}

_LIB = None


def load(path: str | None = None) -> C.CDLL:
    """Loads the in-tree library (building it first is the caller's job: build.py)."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = path or os.environ.get("DISMOEN_LIB") or LIB_PATH  # DISMOEN_LIB: an alternative build
    if not os.path.exists(p):
        raise RuntimeError(
            f"libdismoen_cuda.so not found at {p}; build it with "
            "`python -m disk_streaming_moe_engine_b200.build` (there is no CPU fallback)")
    lib = C.CDLL(p)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _LIB = lib
    return lib


class DmError(RuntimeError):
    """A non-zero status of the C ABI, carrying the library's JSON error message."""

    def __init__(self, code: int, message: str):
        super().__init__(f"status {code}: {message}")
        self.code = code
        self.message = message
