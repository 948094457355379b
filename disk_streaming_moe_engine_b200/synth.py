"""Seeded synthetic checkpoints in canonical host layouts.

Every tensor is produced by the library's counter-based generator (dm_synth_*), keyed by
(seed, stream id) as documented in csrc/dm_synth.h, so a tensor can be regenerated
anywhere without storing it.  Layouts:
  dense  bf16 bit patterns (uint16) row-major [out, in]; dt_bias / A_log fp32
  experts (per layer, index E = shared expert):
    gq/uq uint8 [E+1, I, H/2]   gs/us uint16(fp16) [E+1, I, H/G]   gz/uz uint8 [E+1, I, H/G/2]
    dq    uint8 [E+1, H, I/2]   ds    uint16(fp16) [E+1, H, I/G]   dz    uint8 [E+1, H, I/G/2]
"""
from __future__ import annotations

import math

import numpy as np

from . import _lib
from .config import ModelConfig

NORM = (1.0, 0.02)
W = (0.0, 0.02)


def dense_stream(layer: int, tensor_id: int) -> int:
    return ((layer + 1) << 8) | tensor_id


def expert_stream(layer: int, expert: int, proj: int, part: int) -> int:
    return (1 << 40) | (layer << 20) | ((expert + 1) << 4) | (3 * proj + part)


def _bf16(lib, seed, sid, shape, mean, std):
    out = np.empty(shape, dtype=np.uint16)
    rc = lib.dm_synth_bf16(seed, sid, out.size, mean, std, out.ctypes.data)
    assert rc == 0
    return out


def _f32(lib, seed, sid, shape, mean, std):
    out = np.empty(shape, dtype=np.float32)
    assert lib.dm_synth_f32(seed, sid, out.size, mean, std, out.ctypes.data) == 0
    return out


def _u8(lib, seed, sid, shape):
    out = np.empty(shape, dtype=np.uint8)
    assert lib.dm_synth_u8(seed, sid, out.size, out.ctypes.data) == 0
    return out


def _f16abs(lib, seed, sid, shape, std):
    out = np.empty(shape, dtype=np.uint16)
    assert lib.dm_synth_f16_absnormal(seed, sid, out.size, std, out.ctypes.data) == 0
    return out


def synth_experts(cfg: ModelConfig, layer: int, seed: int, lib=None) -> dict:
    lib = lib or _lib.load()
    E, I, H, G = cfg.num_experts, cfg.moe_intermediate_size, cfg.hidden_size, cfg.quant_group_size
    out = {}
    for name, proj, rows, cols in (("g", _lib.DM_PROJ_GATE, I, H), ("u", _lib.DM_PROJ_UP, I, H),
                                   ("d", _lib.DM_PROJ_DOWN, H, I)):
        q = np.empty((E + 1, rows, cols // 2), np.uint8)
        s = np.empty((E + 1, rows, cols // G), np.uint16)
        z = np.empty((E + 1, rows, cols // G // 2), np.uint8)
        for idx in range(E + 1):
            e = idx if idx < E else -1
            q[idx] = _u8(lib, seed, expert_stream(layer, e, proj, 0), q[idx].shape)
            s[idx] = _f16abs(lib, seed, expert_stream(layer, e, proj, 1), s[idx].shape, 0.02)
            z[idx] = _u8(lib, seed, expert_stream(layer, e, proj, 2), z[idx].shape)
        out[name + "q"], out[name + "s"], out[name + "z"] = q, s, z
    return out


def synth_layer(cfg: ModelConfig, layer: int, seed: int, lib=None, experts: bool = True) -> dict:
    lib = lib or _lib.load()
    H = cfg.hidden_size
    d = {}

    def bf(name, tid, shape, dist):
        d[name] = _bf16(lib, seed, dense_stream(layer, tid), shape, *dist)

    bf("in_norm", _lib.DM_T_INPUT_NORM, (H,), NORM)
    bf("post_norm", _lib.DM_T_POST_NORM, (H,), NORM)
    bf("router", _lib.DM_T_ROUTER, (cfg.num_experts, H), (0.0, 1.0 / math.sqrt(H)))
    bf("shared_gate", _lib.DM_T_SHARED_GATE, (H,), W)
    if cfg.is_attention_layer(layer):
        D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
        bf("q", _lib.DM_T_ATTN_Q, (2 * Hq * D, H), W)
        bf("k", _lib.DM_T_ATTN_K, (Hkv * D, H), W)
        bf("v", _lib.DM_T_ATTN_V, (Hkv * D, H), W)
        bf("qn", _lib.DM_T_ATTN_Q_NORM, (D,), NORM)
        bf("kn", _lib.DM_T_ATTN_K_NORM, (D,), NORM)
        bf("o", _lib.DM_T_ATTN_O, (H, Hq * D), W)
    else:
        nv = cfg.linear_num_value_heads
        bf("qkv", _lib.DM_T_GDN_QKV, (cfg.qkv_dim, H), W)
        bf("z", _lib.DM_T_GDN_Z, (cfg.z_dim, H), W)
        bf("a", _lib.DM_T_GDN_A, (nv, H), W)
        bf("b", _lib.DM_T_GDN_B, (nv, H), W)
        bf("conv", _lib.DM_T_GDN_CONV, (cfg.qkv_dim, 4), W)
        d["dt_bias"] = _f32(lib, seed, dense_stream(layer, _lib.DM_T_GDN_DT_BIAS), (nv,), *W)
        d["a_log"] = _f32(lib, seed, dense_stream(layer, _lib.DM_T_GDN_A_LOG), (nv,), *W)
        bf("gnorm", _lib.DM_T_GDN_NORM, (cfg.linear_value_head_dim,), NORM)
        bf("out", _lib.DM_T_GDN_OUT, (H, cfg.z_dim), W)
    if experts:
        d.update(synth_experts(cfg, layer, seed, lib))
    return d


def synth_model(cfg: ModelConfig, seed: int, layers: list[int] | None = None, head: bool = True,
                lib=None) -> dict:
    """Synthetic model dict: {'cfg', 'layers': {idx: tensors}, 'embed', 'final_norm', 'lm_head'}."""
    lib = lib or _lib.load()
    H, V = cfg.hidden_size, cfg.vocab_size
    idx = list(range(cfg.num_hidden_layers)) if layers is None else layers
    m = {"cfg": cfg, "seed": seed, "layers": {l: synth_layer(cfg, l, seed, lib) for l in idx}}
    if head:
        m["embed"] = _bf16(lib, seed, dense_stream(-1, _lib.DM_T_EMBED), (V, H), *W)
        m["final_norm"] = _bf16(lib, seed, dense_stream(-1, _lib.DM_T_FINAL_NORM), (H,), *NORM)
        m["lm_head"] = _bf16(lib, seed, dense_stream(-1, _lib.DM_T_LM_HEAD), (V, H), *W)
    return m


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r[nan] = 0x7FC0
    return r
