"""ctypes wrapper of the CPU oracle liboracle.so — TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this package;
the product path (disk_streaming_moe_engine_b200) never does.  See dm_oracle.h for the
semantics and the reference lines each function restates.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

ORACLE_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(ORACLE_DIR, "liboracle.so")


class OrDims(C.Structure):
    _fields_ = [("H", C.c_int), ("L", C.c_int), ("interval", C.c_int), ("V", C.c_int), ("eps", C.c_float),
                ("Hq", C.c_int), ("Hkv", C.c_int), ("D", C.c_int), ("rot_dim", C.c_int), ("theta", C.c_float),
                ("nk", C.c_int), ("nv", C.c_int), ("dk", C.c_int), ("dv", C.c_int),
                ("E", C.c_int), ("topk", C.c_int), ("I", C.c_int), ("G", C.c_int), ("kv_bf16", C.c_int)]


_LAYER_FIELDS = ["in_norm", "post_norm", "qkv", "z", "a", "b", "conv", "gnorm", "out", "dt_bias", "a_log",
                 "q", "k", "v", "qn", "kn", "o", "router", "shared_gate", "gq", "gz", "uq", "uz", "dq", "dz",
                 "gs", "us", "ds"]


class OrLayer(C.Structure):
    _fields_ = [(f, C.c_void_p) for f in _LAYER_FIELDS]


class OrModel(C.Structure):
    _fields_ = [("d", OrDims), ("layers", C.POINTER(OrLayer)), ("embed", C.c_void_p),
                ("final_norm", C.c_void_p), ("lm_head", C.c_void_p)]


class OrState(C.Structure):
    _fields_ = [("S", C.c_void_p), ("conv", C.c_void_p), ("kcache", C.c_void_p), ("vcache", C.c_void_p),
                ("cap", C.c_int), ("len", C.c_int)]


_LIB = None


def load() -> C.CDLL:
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            subprocess.run(["make", "-C", ORACLE_DIR], check=True, capture_output=True)
        lib = C.CDLL(LIB_PATH)
        P = C.c_void_p
        lib.or_decode_step.restype = C.c_int
        lib.or_decode_step.argtypes = [C.POINTER(OrModel), C.POINTER(OrState), C.c_int, P, P]
        lib.or_block_forward.argtypes = [C.POINTER(OrModel), C.POINTER(OrState), C.c_int, P, P, P]
        lib.or_moe_block.argtypes = [C.POINTER(OrDims), C.POINTER(OrLayer), P, P, P, P]
        lib.or_gdn_block.argtypes = [C.POINTER(OrDims), C.POINTER(OrLayer), P, P, C.c_int, P, P]
        lib.or_attn_block.argtypes = [C.POINTER(OrDims), C.POINTER(OrLayer), P, P, C.c_int, P, P]
        lib.or_router.argtypes = [C.POINTER(OrDims), C.POINTER(OrLayer), P, P, P, P, P]
        lib.or_rmsnorm_canonical.argtypes = [P, P, C.c_int, C.c_float, P]
        lib.or_dequant_q4.argtypes = [P, P, P, C.c_int, C.c_int, C.c_int, P]
        lib.or_dequant_sym4.restype = C.c_int
        lib.or_dequant_sym4.argtypes = [P, P, C.c_longlong, C.c_int, P, P]
        lib.or_gguf_dequant.restype = C.c_int
        lib.or_gguf_dequant.argtypes = [C.c_int, P, C.c_longlong, C.c_uint, P]
        lib.or_sym4_to_pool.restype = C.c_uint
        lib.or_sym4_to_pool.argtypes = [P, P, C.c_longlong, C.c_int, C.c_int, C.c_int, C.c_int, P, P, P]
        lib.or_requant_pool.restype = C.c_uint
        lib.or_requant_pool.argtypes = [P, C.c_int, C.c_int, C.c_int, P, P, P, C.POINTER(C.c_float)]
        lib.or_f32_to_f16.restype = C.c_uint16
        lib.or_f32_to_f16.argtypes = [C.c_float]
        lib.or_f16_to_f32.restype = C.c_float
        lib.or_f16_to_f32.argtypes = [C.c_uint16]
        lib.or_head.restype = C.c_int
        lib.or_head.argtypes = [C.POINTER(OrModel), P, P]
        lib.or_det_exp.restype = C.c_float
        lib.or_det_exp.argtypes = [C.c_float]
        U64 = C.c_uint64
        for name, extra in (("or_synth_bf16", [C.c_float, C.c_float]), ("or_synth_f32", [C.c_float, C.c_float]),
                            ("or_synth_u8", []), ("or_synth_f16_absnormal", [C.c_float])):
            fn = getattr(lib, name)
            fn.restype = C.c_int
            fn.argtypes = [U64, U64, U64, *extra, P]
        lib.or_set_threads.argtypes = [C.c_int]
        lib.or_get_threads.restype = C.c_int
        _LIB = lib
    return _LIB


def _p(a):
    return None if a is None else a.ctypes.data


class SynthLib:
    """The oracle's restatement of the seeded generator under the names the product's
    `synth` module calls (dm_synth_*), so a synthetic model can be built without loading
    the CUDA library: synth.synth_model(cfg, seed, lib=oracle.SynthLib())."""

    def __init__(self):
        lib = load()
        self.dm_synth_bf16 = lib.or_synth_bf16
        self.dm_synth_f32 = lib.or_synth_f32
        self.dm_synth_u8 = lib.or_synth_u8
        self.dm_synth_f16_absnormal = lib.or_synth_f16_absnormal


def dims_from_cfg(cfg, kv_bf16: bool = True) -> OrDims:
    return OrDims(cfg.hidden_size, cfg.num_hidden_layers, cfg.full_attention_interval, cfg.vocab_size,
                  cfg.rms_norm_eps, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim,
                  int(cfg.head_dim * cfg.partial_rotary_factor), cfg.rope_theta, cfg.linear_num_key_heads,
                  cfg.linear_num_value_heads, cfg.linear_key_head_dim, cfg.linear_value_head_dim,
                  cfg.num_experts, cfg.num_experts_per_tok, cfg.moe_intermediate_size, cfg.quant_group_size,
                  1 if kv_bf16 else 0)


def layer_struct(t: dict) -> OrLayer:
    L = OrLayer()
    for f in _LAYER_FIELDS:
        if f in t:
            setattr(L, f, t[f].ctypes.data)
    return L


class OracleModel:
    """Binds a synthetic model dict (disk_streaming_moe_engine_b200.synth layout)."""

    def __init__(self, m: dict, kv_bf16: bool = True):
        self.lib = load()
        self.m = m
        cfg = m["cfg"]
        self.cfg = cfg
        self.d = dims_from_cfg(cfg, kv_bf16)
        n = cfg.num_hidden_layers
        self._layers = (OrLayer * n)()
        for l in range(n):
            if l in m["layers"]:
                self._layers[l] = layer_struct(m["layers"][l])
        self.model = OrModel(self.d, self._layers, _p(m.get("embed")), _p(m.get("final_norm")),
                             _p(m.get("lm_head")))

    def layer(self, l: int) -> OrLayer:
        return self._layers[l]


class OracleState:
    def __init__(self, cfg, cap: int, kv_bf16: bool = True):
        ng, na = cfg.num_gdn_layers(), cfg.num_attention_layers()
        self.S = np.zeros((max(ng, 1), cfg.linear_num_value_heads, cfg.linear_value_head_dim,
                           cfg.linear_key_head_dim), np.float32)
        self.conv = np.zeros((max(ng, 1), 3, cfg.qkv_dim), np.float32)
        dt = np.uint16 if kv_bf16 else np.float32
        self.k = np.zeros((max(na, 1), cap, cfg.num_key_value_heads, cfg.head_dim), dt)
        self.v = np.zeros_like(self.k)
        self.st = OrState(_p(self.S), _p(self.conv), _p(self.k), _p(self.v), cap, 0)

    @property
    def len(self) -> int:
        return self.st.len


def decode_step(om: OracleModel, st: OracleState, token: int, hidden: bool = False):
    lib = load()
    cfg = om.cfg
    logits = np.empty(cfg.vocab_size, np.float32)
    hid = np.empty((cfg.num_hidden_layers, cfg.hidden_size), np.float32) if hidden else None
    nxt = lib.or_decode_step(C.byref(om.model), C.byref(st.st), int(token), _p(logits), _p(hid))
    return nxt, logits, hid


def gdn_block(om: OracleModel, layer: int, S: np.ndarray, conv: np.ndarray, pos: int, x: np.ndarray):
    y = np.empty_like(x)
    load().or_gdn_block(C.byref(om.d), C.byref(om._layers[layer]), _p(S), _p(conv), pos, _p(x), _p(y))
    return y


def attn_block(om: OracleModel, layer: int, k: np.ndarray, v: np.ndarray, pos: int, x: np.ndarray):
    y = np.empty_like(x)
    load().or_attn_block(C.byref(om.d), C.byref(om._layers[layer]), _p(k), _p(v), pos, _p(x), _p(y))
    return y


def moe_block(om: OracleModel, layer: int, x_mid: np.ndarray):
    y = np.empty_like(x_mid)
    ids = np.empty(om.cfg.num_experts_per_tok, np.int32)
    probs = np.empty(om.cfg.num_experts_per_tok, np.float32)
    load().or_moe_block(C.byref(om.d), C.byref(om._layers[layer]), _p(x_mid), _p(y), _p(ids), _p(probs))
    return y, ids, probs


def router(om: OracleModel, layer: int, xn: np.ndarray):
    k, E = om.cfg.num_experts_per_tok, om.cfg.num_experts
    ids, probs = np.empty(k, np.int32), np.empty(k, np.float32)
    sg = np.empty(1, np.float32)
    logits = np.empty(E + 1, np.float32)
    load().or_router(C.byref(om.d), C.byref(om._layers[layer]), _p(xn), _p(ids), _p(probs), _p(sg), _p(logits))
    return ids, probs, float(sg[0]), logits


def rmsnorm(x: np.ndarray, gamma_bf16: np.ndarray, eps: float):
    y = np.empty_like(x)
    load().or_rmsnorm_canonical(_p(x), _p(gamma_bf16), x.size, eps, _p(y))
    return y


def dequant_q4(q, s, z, rows, cols, group=64):
    out = np.empty((rows, cols), np.float32)
    load().or_dequant_q4(_p(np.ascontiguousarray(q)), _p(np.ascontiguousarray(s)), _p(np.ascontiguousarray(z)),
                         rows, cols, group, _p(out))
    return out


def dequant_sym4(packed, scales_f16_bits, n, group=128):
    """(bf16 bits uint16 [n], fp32 [n], status) for the reference's custom 4-bit format;
    status 0 ok, -1 reserved nibble 0b1000, -2 NaN / Inf / non-positive scale."""
    ob = np.empty(n, np.uint16)
    of = np.empty(n, np.float32)
    rc = load().or_dequant_sym4(_p(np.ascontiguousarray(packed, np.uint8)),
                                _p(np.ascontiguousarray(scales_f16_bits, np.uint16)), n, group, _p(ob), _p(of))
    return ob, of, rc


def gguf_dequant(raw: bytes, ggml_type: int, n: int, q4k_mojo: bool = False) -> np.ndarray:
    """fp32 [n] of GGML blocks (or_formats.c); raises on an unsupported type or a ragged n."""
    buf = np.frombuffer(bytes(raw), np.uint8)
    out = np.empty(n, np.float32)
    rc = load().or_gguf_dequant(ggml_type, _p(buf), n, 1 if q4k_mojo else 0, _p(out))
    if rc != 0:
        raise ValueError(f"or_gguf_dequant: status {rc}")
    return out


def sym4_to_pool(packed, scales, e0: int, rows: int, cols: int, gf: int, gp: int = 64):
    """(q [rows, cols/2], s [rows, cols/gp], z [rows, cols/gp/2], flags) of the exact
    custom-4-bit -> pool conversion."""
    q = np.empty((rows, cols // 2), np.uint8)
    s = np.empty((rows, cols // gp), np.uint16)
    z = np.empty((rows, cols // gp // 2), np.uint8)
    f = load().or_sym4_to_pool(_p(np.ascontiguousarray(packed, np.uint8)), _p(np.ascontiguousarray(scales, np.uint16)),
                               e0, rows, cols, gf, gp, _p(q), _p(s), _p(z))
    return q, s, z, f


def requant_pool(w, gp: int = 64):
    """(q, s, z, flags, max_err) of the round-to-nearest re-quantisation of w [rows, cols]."""
    w = np.ascontiguousarray(w, np.float32)
    rows, cols = w.shape
    q = np.zeros((rows, cols // 2), np.uint8)
    s = np.empty((rows, cols // gp), np.uint16)
    z = np.zeros((rows, cols // gp // 2), np.uint8)
    err = C.c_float()
    f = load().or_requant_pool(_p(w), rows, cols, gp, _p(q), _p(s), _p(z), C.byref(err))
    return q, s, z, f, err.value


def f32_to_f16_bits(x: float) -> int:
    return load().or_f32_to_f16(x)


def det_exp(x: float) -> float:
    return load().or_det_exp(x)


def set_threads(n: int):
    load().or_set_threads(n)


def get_threads() -> int:
    return load().or_get_threads()
