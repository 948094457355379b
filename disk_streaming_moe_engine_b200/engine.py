"""Host-side mirror of the reference engine's layer API over libdismoen_cuda.so.

The reference Mojo engine exposes, per layer (src/layers/port_scheduler.mojo,
gguf_port_loader.mojo, router.mojo, gated_attention.mojo, gdn.mojo):

  forward_port_block(x, block, gdn_states, kv_cache, layer_idx, pos_offset, seq_len, ...)
  forward_port_macro_scheduler_gguf(x, index, gdn_states, kv_cache, pos_offset, seq_len, ...)
  router_forward(x, w_router, seq_len, hidden, RouterConfig, layer_idx) -> RoutingInfo
  GatedAttnKVCache(capacity, l_att, h_kv, head_dim): store_tokens / get_k / get_v / zero
  GDNState(layers, dv, dk): zero / clone / check_finite

Here the weights live in the device context (uploaded once instead of streamed per
step), so the per-call weight arguments disappear; argument meaning, shapes and error
behaviour follow the reference: errors raise `DmError` carrying the library's JSON
message in the reference shape {"error_type", "detail", "stage", "layer"}.
"""
from __future__ import annotations

import ctypes as C
import dataclasses
import os

import numpy as np

from . import _lib
from .config import ModelConfig, RuntimeConfig


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


@dataclasses.dataclass
class RoutingInfo:
    """reference src/layers/router_types.mojo:48 (selected experts, probabilities)."""
    selected_experts: np.ndarray   # [seq_len, top_k] int32
    routing_weights: np.ndarray    # [seq_len, top_k] fp32, not renormalised
    shared_gate: np.ndarray        # [seq_len] sigmoid(w_sh . x)
    seq_len: int
    top_k: int


class Engine:
    """One device context: model weights in HBM plus `max_seqs` sequence slots."""

    def __init__(self, cfg: ModelConfig, rt: RuntimeConfig | None = None, device: int = 0):
        self.cfg = cfg
        self.rt = rt or RuntimeConfig.for_context(1024)
        self.lib = _lib.load()
        self._mc = cfg.to_c()
        self._rc = self.rt.to_c()
        buf = C.create_string_buffer(512)
        if self.lib.dm_config_validate(C.byref(self._mc), buf, 512) != 0:
            raise _lib.DmError(_lib.DM_ERR_INVALID_ARG, buf.value.decode())
        h = C.c_void_p()
        rc = self.lib.dm_ctx_create(C.byref(self._mc), C.byref(self._rc), device, C.byref(h))
        if rc != 0:
            raise _lib.DmError(rc, "dm_ctx_create failed (see stderr)")
        self.ctx = h

    # ---- plumbing ----
    def close(self):
        if getattr(self, "ctx", None):
            self.lib.dm_ctx_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def last_error(self) -> str:
        buf = C.create_string_buffer(1024)
        self.lib.dm_last_error(self.ctx, buf, 1024)
        return buf.value.decode()

    def _ok(self, rc: int):
        if rc != 0:
            raise _lib.DmError(rc, self.last_error())

    def device_bytes(self) -> int:
        v = C.c_uint64()
        self._ok(self.lib.dm_ctx_device_bytes(self.ctx, C.byref(v)))
        return v.value

    def stream(self) -> int:
        s = C.c_void_p()
        self._ok(self.lib.dm_get_stream(self.ctx, C.byref(s)))
        return s.value or 0

    def time_kernel(self, which: int, layer: int, iters: int = 20):
        """(mean ms per launch, algorithmic bytes per launch) of one kernel kind."""
        ms, nb = C.c_float(), C.c_uint64()
        self._ok(self.lib.dm_time_kernel(self.ctx, which, layer, iters, C.byref(ms), C.byref(nb)))
        return ms.value, nb.value

    def trace_enable(self, on: bool = True):
        self._ok(self.lib.dm_trace_enable(self.ctx, 1 if on else 0))

    def trace_read(self, n: int = 64) -> np.ndarray:
        out = np.zeros(n, np.uint64)
        self._ok(self.lib.dm_trace_read(self.ctx, _ptr(out), n))
        return out

    TRACE_KINDS = ["embed", "gdn_in", "gdn_rec", "gdn_out", "attn_in", "attn", "attn_out", "moe", "head",
                   "gdn_core_out"]

    def trace_timeline(self, n: int = 512):
        """[(kind, layer, start_ns, ready_ns, end_ns)] of the last traced decode step."""
        rec = np.zeros((n, 4), np.uint64)
        kinds = np.zeros(n, np.int32)
        cnt = C.c_int32()
        self._ok(self.lib.dm_trace_timeline(self.ctx, _ptr(rec), _ptr(kinds), n, C.byref(cnt)))
        out = []
        for i in range(cnt.value):
            k = int(kinds[i])
            out.append((self.TRACE_KINDS[k >> 16], k & 0xFFFF, int(rec[i, 0]), int(rec[i, 1]), int(rec[i, 2])))
        return out

    def kernels_per_step(self) -> int:
        v = C.c_int32()
        self._ok(self.lib.dm_kernels_per_step(self.ctx, C.byref(v)))
        return v.value

    # ---- weights (quant loader / tensor-name contract) ----
    def upload_tensor(self, layer: int, tensor_id: int, arr: np.ndarray):
        arr = np.ascontiguousarray(arr)
        dt = _lib.DM_DTYPE_F32 if arr.dtype == np.float32 else _lib.DM_DTYPE_BF16
        if arr.dtype not in (np.float32, np.uint16):
            raise TypeError("dense tensors are bf16 bit patterns (uint16) or float32")
        self._ok(self.lib.dm_upload_tensor(self.ctx, layer, tensor_id, dt, _ptr(arr), arr.size))

    def upload_expert(self, layer: int, expert: int, proj: int, q: np.ndarray, s: np.ndarray, z: np.ndarray):
        q, s, z = (np.ascontiguousarray(a) for a in (q, s, z))
        self._ok(self.lib.dm_expert_upload(self.ctx, layer, expert, proj, _ptr(q), _ptr(s), _ptr(z)))

    _GDN = {"qkv": _lib.DM_T_GDN_QKV, "z": _lib.DM_T_GDN_Z, "a": _lib.DM_T_GDN_A, "b": _lib.DM_T_GDN_B,
            "conv": _lib.DM_T_GDN_CONV, "dt_bias": _lib.DM_T_GDN_DT_BIAS, "a_log": _lib.DM_T_GDN_A_LOG,
            "gnorm": _lib.DM_T_GDN_NORM, "out": _lib.DM_T_GDN_OUT}
    _ATT = {"q": _lib.DM_T_ATTN_Q, "k": _lib.DM_T_ATTN_K, "v": _lib.DM_T_ATTN_V, "qn": _lib.DM_T_ATTN_Q_NORM,
            "kn": _lib.DM_T_ATTN_K_NORM, "o": _lib.DM_T_ATTN_O}
    _COMMON = {"in_norm": _lib.DM_T_INPUT_NORM, "post_norm": _lib.DM_T_POST_NORM, "router": _lib.DM_T_ROUTER,
               "shared_gate": _lib.DM_T_SHARED_GATE}

    def load_layer(self, layer: int, t: dict):
        """Binds one layer's tensors (the role of load_port_block_from_gguf,
        reference gguf_port_loader.mojo:115)."""
        table = dict(self._COMMON)
        table.update(self._ATT if self.cfg.is_attention_layer(layer) else self._GDN)
        for name, tid in table.items():
            self.upload_tensor(layer, tid, t[name])
        if "gq" in t:
            E = self.cfg.num_experts
            for idx in range(E + 1):
                e = idx if idx < E else -1
                self.upload_expert(layer, e, _lib.DM_PROJ_GATE, t["gq"][idx], t["gs"][idx], t["gz"][idx])
                self.upload_expert(layer, e, _lib.DM_PROJ_UP, t["uq"][idx], t["us"][idx], t["uz"][idx])
                self.upload_expert(layer, e, _lib.DM_PROJ_DOWN, t["dq"][idx], t["ds"][idx], t["dz"][idx])

    def load_model(self, m: dict):
        for l, t in m["layers"].items():
            self.load_layer(l, t)
        if "embed" in m:
            self.upload_tensor(-1, _lib.DM_T_EMBED, m["embed"])
            self.upload_tensor(-1, _lib.DM_T_FINAL_NORM, m["final_norm"])
            self.upload_tensor(-1, _lib.DM_T_LM_HEAD, m["lm_head"])

    def synth_on_device(self, seed: int):
        self._ok(self.lib.dm_synth_model_device(self.ctx, seed))

    def weights_check(self):
        self._ok(self.lib.dm_weights_check(self.ctx))

    def dequant_q4(self, q: np.ndarray, s: np.ndarray, z: np.ndarray, rows: int, cols: int, group: int = 64):
        out = np.empty((rows, cols), np.float32)
        q, s, z = (np.ascontiguousarray(a) for a in (q, s, z))
        self._ok(self.lib.dm_dequant_q4(self.ctx, _ptr(q), _ptr(s), _ptr(z), rows, cols, group, _ptr(out)))
        return out

    def dequant_sym4(self, packed: np.ndarray, scales_f16_bits: np.ndarray, n: int, group: int = 128,
                     want_bf16: bool = True, want_f32: bool = True):
        """The reference's custom 4-bit format -> (bf16 bits uint16 [n] or None, fp32 [n] or None)
        (dequant_kernel_simd / dequant_kernel_simd_f32)."""
        p = np.ascontiguousarray(packed, np.uint8)
        sc = np.ascontiguousarray(scales_f16_bits, np.uint16)
        ob = np.empty(n, np.uint16) if want_bf16 else None
        of = np.empty(n, np.float32) if want_f32 else None
        self._ok(self.lib.dm_dequant_sym4(self.ctx, _ptr(p), _ptr(sc), n, group,
                                          None if ob is None else _ptr(ob), None if of is None else _ptr(of)))
        return ob, of

    def tensor_download(self, layer: int, tensor_id: int, n: int) -> np.ndarray:
        """A dense weight as uploaded: bf16 bits (uint16) or fp32 for dt_bias / A_log."""
        f32 = tensor_id in (_lib.DM_T_GDN_DT_BIAS, _lib.DM_T_GDN_A_LOG)
        out = np.empty(n, np.float32 if f32 else np.uint16)
        self._ok(self.lib.dm_tensor_download(self.ctx, layer, tensor_id,
                                             _lib.DM_DTYPE_F32 if f32 else _lib.DM_DTYPE_BF16, _ptr(out), n))
        return out

    def expert_download(self, layer: int, expert: int, proj: int):
        """(q [rows, cols/2], scales [rows, cols/g], zeros [rows, cols/g/2]) of one projection."""
        cfg = self.cfg
        H, I, G = cfg.hidden_size, cfg.moe_intermediate_size, cfg.quant_group_size
        rows, cols = (H, I) if proj == _lib.DM_PROJ_DOWN else (I, H)
        q = np.empty((rows, cols // 2), np.uint8)
        s = np.empty((rows, cols // G), np.uint16)
        z = np.empty((rows, cols // G // 2), np.uint8)
        self._ok(self.lib.dm_expert_download(self.ctx, layer, expert, proj, _ptr(q), _ptr(s), _ptr(z)))
        return q, s, z

    # ---- spilling expert pool (RuntimeConfig.expert_cache_slots > 0) ----
    SPILL_KEYS = ("accesses", "hits", "misses", "evictions", "loads", "pins_kept_unpinned", "bytes_h2d", "slots")

    def spill_stats(self) -> dict:
        out = (C.c_uint64 * 8)()
        self._ok(self.lib.dm_spill_stats(self.ctx, out))
        return dict(zip(self.SPILL_KEYS, (int(v) for v in out)))

    def spill_pin(self, layer: int, expert: int) -> bool:
        """Makes the expert resident and pins it (False: kept unpinned, over the 25 % budget)."""
        r = C.c_int32()
        self._ok(self.lib.dm_spill_pin(self.ctx, layer, expert, C.byref(r)))
        return bool(r.value)

    # ---- quant-file loaders (formats.py parses; these dequantise / load on the device) ----
    def gguf_dequant(self, raw: bytes, ggml_type: int, n: int, q4k_mojo: bool = False,
                     want_f32: bool = True, want_bf16: bool = False):
        """GGML blocks -> (fp32 [n] or None, bf16 bits [n] or None) on the GPU
        (dequantize_q8_0 / _q4_k / _q3_k, gguf.mojo:414-561)."""
        buf = np.frombuffer(bytes(raw), np.uint8)
        of = np.empty(n, np.float32) if want_f32 else None
        ob = np.empty(n, np.uint16) if want_bf16 else None
        flags = _lib.DM_GGUF_Q4K_MOJO if q4k_mojo else 0
        self._ok(self.lib.dm_gguf_dequant(self.ctx, ggml_type, _ptr(buf), buf.size, n, flags,
                                          None if of is None else _ptr(of), None if ob is None else _ptr(ob)))
        return of, ob

    def load_gguf_tensor(self, index, name: str, layer: int, tensor_id: int, q4k_mojo: bool = False):
        """One GGUF tensor -> dense weight (layer, tensor_id) (stream_gguf_tensor_f32, gguf.mojo:563)."""
        flags = _lib.DM_GGUF_Q4K_MOJO if q4k_mojo else 0
        self._ok(self.lib.dm_gguf_load_tensor(self.ctx, index.handle, name.encode(), layer, tensor_id, flags))

    def load_gguf_expert(self, index, name: str, layer: int, expert: int, proj: int, slab: int = 0,
                         row0: int = 0, requant: bool = False, q4k_mojo: bool = False) -> float:
        """One expert projection from a GGUF tensor, re-quantised into the pool; returns the
        largest |w - w'|."""
        flags = (_lib.DM_LOAD_REQUANT if requant else 0) | (_lib.DM_GGUF_Q4K_MOJO if q4k_mojo else 0)
        err = C.c_float()
        self._ok(self.lib.dm_gguf_load_expert(self.ctx, index.handle, name.encode(), slab, row0, layer, expert, proj,
                                              flags, C.byref(err)))
        return err.value

    def load_quant_tensor(self, index, name: str, layer: int, tensor_id: int):
        """load_one_quant_tensor_bf16 / _f32 (quant_loader.mojo:27-58) into a dense weight."""
        self._ok(self.lib.dm_quant_file_load_tensor(self.ctx, index.handle, name.encode(), layer, tensor_id))

    def load_quant_expert(self, index, name: str, layer: int, expert: int, proj: int, slab: int = 0,
                          row0: int = 0, requant: bool = False) -> float:
        """One expert projection from a quant-file tensor (exact when the groups allow)."""
        err = C.c_float()
        self._ok(self.lib.dm_quant_file_load_expert(self.ctx, index.handle, name.encode(), slab, row0, layer, expert,
                                                    proj, _lib.DM_LOAD_REQUANT if requant else 0, C.byref(err)))
        return err.value

    def load_quant_file(self, path_or_index, requant: bool = False):
        """Every weight of the configured model from the reference's custom 4-bit quant file
        (checkpoint names; per-expert or stacked experts)."""
        from .formats import scan_quant_file
        idx = scan_quant_file(path_or_index) if isinstance(path_or_index, str) else path_or_index
        try:
            self._ok(self.lib.dm_quant_file_load(self.ctx, idx.handle, _lib.DM_LOAD_REQUANT if requant else 0))
        finally:
            if isinstance(path_or_index, str):
                idx.close()

    # ---- sequence state (KV-cache object, GDN state) ----
    def seq_reset(self, slot: int = 0):
        self._ok(self.lib.dm_seq_reset(self.ctx, slot))

    def seq_len(self, slot: int = 0) -> int:
        v = C.c_int32()
        self._ok(self.lib.dm_seq_get_len(self.ctx, slot, C.byref(v)))
        return v.value

    def seq_set_len(self, slot: int, n: int):
        self._ok(self.lib.dm_seq_set_len(self.ctx, slot, n))

    def set_page_table(self, slot: int, pages):
        p = np.ascontiguousarray(pages, dtype=np.int32)
        self._ok(self.lib.dm_seq_set_page_table(self.ctx, slot, _ptr(p), p.size))

    def kv_import(self, att_layer: int, slot: int, k_bf16: np.ndarray, v_bf16: np.ndarray):
        k, v = np.ascontiguousarray(k_bf16, np.uint16), np.ascontiguousarray(v_bf16, np.uint16)
        n = k.shape[0]
        self._ok(self.lib.dm_kv_import(self.ctx, att_layer, slot, _ptr(k), _ptr(v), n))

    def kv_export(self, att_layer: int, slot: int, n: int):
        shape = (n, self.cfg.num_key_value_heads, self.cfg.head_dim)
        k, v = np.empty(shape, np.uint16), np.empty(shape, np.uint16)
        self._ok(self.lib.dm_kv_export(self.ctx, att_layer, slot, _ptr(k), _ptr(v), n))
        return k, v

    def gdn_state_import(self, gdn_layer: int, slot: int, S: np.ndarray | None, conv: np.ndarray | None = None):
        s = None if S is None else np.ascontiguousarray(S, np.float32)
        c = None if conv is None else np.ascontiguousarray(conv, np.float32)
        self._ok(self.lib.dm_gdn_state_import(self.ctx, gdn_layer, slot, None if s is None else _ptr(s),
                                              None if c is None else _ptr(c)))

    def gdn_state_export(self, gdn_layer: int, slot: int):
        cfg = self.cfg
        S = np.empty((cfg.linear_num_value_heads, cfg.linear_value_head_dim, cfg.linear_key_head_dim), np.float32)
        conv = np.empty((3, cfg.qkv_dim), np.float32)
        self._ok(self.lib.dm_gdn_state_export(self.ctx, gdn_layer, slot, _ptr(S), _ptr(conv)))
        return S, conv

    # ---- compute: reference-facing ----
    def router_forward(self, x: np.ndarray, layer_idx: int) -> RoutingInfo:
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        n, k = x.shape[0], self.cfg.num_experts_per_tok
        ids, probs, sg = np.empty((n, k), np.int32), np.empty((n, k), np.float32), np.empty(n, np.float32)
        self._ok(self.lib.dm_router(self.ctx, layer_idx, _ptr(x), n, _ptr(ids), _ptr(probs), _ptr(sg)))
        return RoutingInfo(ids, probs, sg, n, k)

    def moe_block(self, x_mid: np.ndarray, layer_idx: int) -> np.ndarray:
        x = np.ascontiguousarray(np.atleast_2d(x_mid), np.float32)
        y = np.empty_like(x)
        self._ok(self.lib.dm_moe_block(self.ctx, layer_idx, _ptr(x), x.shape[0], _ptr(y)))
        return y

    def mixer_block(self, x: np.ndarray, layer_idx: int, pos_offset: int, slot: int = 0) -> np.ndarray:
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        y = np.empty_like(x)
        self._ok(self.lib.dm_mixer_block(self.ctx, layer_idx, slot, pos_offset, _ptr(x), x.shape[0], _ptr(y)))
        return y

    def forward_port_block(self, x: np.ndarray, layer_idx: int, pos_offset: int, slot: int = 0) -> np.ndarray:
        """reference forward_port_block (port_scheduler.mojo:286) for seq_len = len(x)."""
        x = np.ascontiguousarray(np.atleast_2d(x), np.float32)
        y = np.empty_like(x)
        self._ok(self.lib.dm_block_forward(self.ctx, layer_idx, slot, pos_offset, _ptr(x), x.shape[0], _ptr(y)))
        return y

    def forward(self, tokens, slot: int = 0, want_logits: bool = True):
        """Macro scheduler over all blocks for `tokens` appended to `slot` (reference
        forward_port_macro_scheduler_gguf, gguf_port_loader.mojo:329) -> (logits, argmax)."""
        t = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(self.cfg.vocab_size, np.float32) if want_logits else None
        nxt = C.c_int32()
        self._ok(self.lib.dm_forward(self.ctx, slot, _ptr(t), t.size, None if logits is None else _ptr(logits),
                                     C.byref(nxt)))
        return logits, nxt.value

    def prefill(self, tokens, slot: int = 0, want_logits: bool = True):
        """The prompt `tokens` appended to `slot` as chunked prefill (dm_prefill: chunks of
        prefill_rows() tokens through every layer together) -> (logits, argmax)."""
        t = np.ascontiguousarray(tokens, np.int32)
        logits = np.empty(self.cfg.vocab_size, np.float32) if want_logits else None
        nxt = C.c_int32()
        self._ok(self.lib.dm_prefill(self.ctx, slot, _ptr(t), t.size, None if logits is None else _ptr(logits),
                                     C.byref(nxt)))
        return logits, nxt.value

    def prefill_rows(self):
        """(rows of one prefill chunk, kernel launches of a chunk without the head)."""
        r, k = C.c_int32(), C.c_int32()
        self._ok(self.lib.dm_prefill_rows(self.ctx, C.byref(r), C.byref(k)))
        return r.value, k.value

    def decode_step(self, token: int, slot: int = 0, want_logits: bool = False):
        logits = np.empty(self.cfg.vocab_size, np.float32) if want_logits else None
        out = C.c_int32()
        self._ok(self.lib.dm_decode_step(self.ctx, slot, int(token), C.byref(out),
                                         None if logits is None else _ptr(logits)))
        return out.value, logits

    def generate(self, token: int, n_steps: int, slot: int = 0) -> np.ndarray:
        out = np.empty(n_steps, np.int32)
        self._ok(self.lib.dm_generate(self.ctx, slot, int(token), n_steps, _ptr(out)))
        return out

    def enqueue_decode(self, n_steps: int, slot: int = 0):
        self._ok(self.lib.dm_enqueue_decode(self.ctx, slot, n_steps))

    def set_token(self, token: int, slot: int = 0):
        self._ok(self.lib.dm_set_token(self.ctx, slot, int(token)))

    def sync(self):
        self._ok(self.lib.dm_sync(self.ctx))

    # ---- batched decode: row i decodes one token of sequence slots[i] ----
    def batch_capacity(self) -> int:
        v = C.c_int32()
        self._ok(self.lib.dm_batch_capacity(self.ctx, C.byref(v)))
        return v.value

    def decode_batch(self, slots, tokens, want_logits: bool = False):
        s = np.ascontiguousarray(slots, np.int32)
        t = np.ascontiguousarray(tokens, np.int32)
        if s.shape != t.shape or s.ndim != 1:
            raise ValueError("slots and tokens must be 1-D of equal length")
        out = np.empty(s.size, np.int32)
        logits = np.empty((s.size, self.cfg.vocab_size), np.float32) if want_logits else None
        self._ok(self.lib.dm_decode_batch(self.ctx, _ptr(s), _ptr(t), s.size, _ptr(out),
                                          None if logits is None else _ptr(logits)))
        return out, logits

    def generate_batch(self, slots, tokens, n_steps: int) -> np.ndarray:
        s = np.ascontiguousarray(slots, np.int32)
        t = np.ascontiguousarray(tokens, np.int32)
        if s.shape != t.shape or s.ndim != 1:
            raise ValueError("slots and tokens must be 1-D of equal length")
        out = np.empty((n_steps, s.size), np.int32)
        self._ok(self.lib.dm_generate_batch(self.ctx, _ptr(s), _ptr(t), s.size, n_steps, _ptr(out)))
        return out

    def enqueue_decode_batch(self, slots, tokens, n_steps: int):
        s = np.ascontiguousarray(slots, np.int32)
        t = np.ascontiguousarray(tokens, np.int32)
        self._ok(self.lib.dm_enqueue_decode_batch(self.ctx, _ptr(s), _ptr(t), s.size, n_steps))

    def batch_read_generated(self, n: int, n_steps: int) -> np.ndarray:
        out = np.empty((n_steps, n), np.int32)
        self._ok(self.lib.dm_batch_read_generated(self.ctx, n, n_steps, _ptr(out)))
        return out

    def batch_stats(self, reset: bool = False) -> dict:
        """Routing statistics of batched steps since the last reset."""
        v = np.zeros(4, np.uint32)
        self._ok(self.lib.dm_batch_stats(self.ctx, int(reset), _ptr(v)))
        ls = max(int(v[3]), 1)
        return {"experts_touched_per_layer": float(v[0]) / ls, "segments_per_layer": float(v[1]) / ls,
                "max_rows_one_expert": int(v[2]), "layer_steps": int(v[3])}

    def time_batch_kernel(self, n: int, which: int, layer: int, iters: int):
        ms, by = C.c_float(), C.c_uint64()
        self._ok(self.lib.dm_time_batch_kernel(self.ctx, n, which, layer, iters, C.byref(ms), C.byref(by)))
        return ms.value, by.value

    def set_router_bias(self, layer: int, bias):
        """Per-expert router logit offsets (None removes them): a synthetic-workload device."""
        if bias is None:
            self._ok(self.lib.dm_set_router_bias(self.ctx, layer, None, 0))
            return
        b = np.ascontiguousarray(bias, np.float32)
        self._ok(self.lib.dm_set_router_bias(self.ctx, layer, _ptr(b), b.size))

    def synth_state(self, seed: int, kv_std: float, state_std: float, length: int):
        """Seeded synthetic state for every slot (KV pool, GDN states, conv windows), length."""
        self._ok(self.lib.dm_synth_state_device(self.ctx, seed, kv_std, state_std, length))

    def add_rank1(self, layer: int, tensor_id: int, beta: np.ndarray, u: np.ndarray):
        beta = np.ascontiguousarray(beta, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        self._ok(self.lib.dm_tensor_add_rank1(self.ctx, layer, tensor_id, _ptr(beta), beta.size, _ptr(u), u.size))

    # ---- session files (reference KMSS v1, src/format/kmss.mojo) ----
    def save_session(self, path: str, tokens, slot: int = 0, kv_dtype: int = 1, manifest_hash: bytes | None = None,
                     conv_window: bool = True):
        """write_kmss_v1 (kmss.mojo:90): the slot's KV cache and GDN states + the token prefix;
        with conv_window also the GDN conv window in the sidecar `path + ".conv"`
        (dm_kmss_save_conv), so that a resumed sequence decodes exactly as an uninterrupted one."""
        t = np.ascontiguousarray(tokens, np.int32)
        mh = None
        if manifest_hash is not None:
            if len(manifest_hash) != 32:
                raise ValueError("manifest hash: 32 bytes")
            mh = C.create_string_buffer(bytes(manifest_hash), 32)
        self._ok(self.lib.dm_kmss_save(self.ctx, slot, path.encode(), _ptr(t) if t.size else None, t.size, kv_dtype, mh))
        if conv_window:
            self._ok(self.lib.dm_kmss_save_conv(self.ctx, slot, path.encode(), (path + ".conv").encode()))

    def load_session(self, path: str, slot: int = 0, max_tokens: int = 1 << 20) -> np.ndarray:
        """read_kmss_v1 (kmss.mojo:280) into `slot`; returns the token prefix.  A sidecar
        `path + ".conv"` written with the file restores the GDN conv window as well."""
        out = np.empty(max_tokens, np.int32)
        n = C.c_int32()
        self._ok(self.lib.dm_kmss_load(self.ctx, slot, path.encode(), _ptr(out), out.size, C.byref(n)))
        if os.path.exists(path + ".conv"):
            self._ok(self.lib.dm_kmss_load_conv(self.ctx, slot, path.encode(), (path + ".conv").encode()))
        return out[:min(n.value, out.size)].copy()

    def seq_copy(self, src_slot: int, dst_slot: int):
        """The whole sequence state of src_slot into dst_slot, on the device (dm_seq_copy)."""
        self._ok(self.lib.dm_seq_copy(self.ctx, src_slot, dst_slot))

    # ---- expert-parallel group (one process per GPU) ----
    def ep_ipc_handle(self) -> bytes:
        buf = C.create_string_buffer(_lib.DM_EP_HANDLE_BYTES)
        self._ok(self.lib.dm_ep_ipc_handle(self.ctx, buf))
        return buf.raw

    def ep_attach(self, rank: int, world: int, handles: list[bytes]):
        if len(handles) != world or any(len(h) != _lib.DM_EP_HANDLE_BYTES for h in handles):
            raise ValueError("one handle of DM_EP_HANDLE_BYTES bytes per rank")
        blob = C.create_string_buffer(b"".join(handles), world * _lib.DM_EP_HANDLE_BYTES)
        self._ok(self.lib.dm_ep_attach(self.ctx, rank, world, blob))

    def ep_detach(self):
        self._ok(self.lib.dm_ep_detach(self.ctx))

    def batch_kernels_per_step(self, n: int) -> tuple[int, int]:
        own, gemms = C.c_int32(), C.c_int32()
        self._ok(self.lib.dm_batch_kernels_per_step(self.ctx, n, C.byref(own), C.byref(gemms)))
        return own.value, gemms.value


class GatedAttnKVCache:
    """View of one slot's paged KV cache with the reference object's surface
    (gated_attention.mojo:38-153 / kv_cache.mojo:213-420)."""

    def __init__(self, engine: Engine, slot: int = 0):
        self.engine, self.slot = engine, slot

    def zero(self):
        self.engine.seq_reset(self.slot)

    def store_prefill(self, att_layer: int, k_bf16: np.ndarray, v_bf16: np.ndarray):
        self.engine.kv_import(att_layer, self.slot, k_bf16, v_bf16)

    def get_k(self, att_layer: int, length: int) -> np.ndarray:
        return self.engine.kv_export(att_layer, self.slot, length)[0]

    def get_v(self, att_layer: int, length: int) -> np.ndarray:
        return self.engine.kv_export(att_layer, self.slot, length)[1]

    @property
    def current_len(self) -> int:
        return self.engine.seq_len(self.slot)


class GDNState:
    """View of one slot's GDN recurrent state (reference GDNState, gdn.mojo:64-124)."""

    def __init__(self, engine: Engine, slot: int = 0):
        self.engine, self.slot = engine, slot

    def zero(self):
        self.engine.seq_reset(self.slot)

    def get(self, gdn_layer: int):
        return self.engine.gdn_state_export(gdn_layer, self.slot)

    def set(self, gdn_layer: int, S: np.ndarray, conv: np.ndarray | None = None):
        self.engine.gdn_state_import(gdn_layer, self.slot, S, conv)

    def check_finite(self) -> bool:
        return all(np.isfinite(self.get(g)[0]).all() for g in range(self.engine.cfg.num_gdn_layers()))
