"""Model and runtime configuration (mirror of reference src/core/config.mojo:11-175).

`ModelConfig` keeps the reference field names; the GDN shape fields are the ones the
reference hard-codes inside forward_gdn_block (src/layers/gdn.mojo:897-1183).  The presets
are the benchmark configurations of this port:

  mini      config 0: 4 blocks (3 GDN + 1 attention), hidden 256, vocab 1024, 16 experts
            top-4 + shared (I = 128), attention 4Q/1KV x 64, GDN 2 QK / 4 V heads x 64
  layer     config 1: one GDN block and one attention block at full shape (hidden 2048,
            256 experts top-8 + shared, I = 512), full-attention interval 2
  full      config 2: 40 blocks [GDN, GDN, GDN, Attn] x 10, vocab 151936
"""
from __future__ import annotations

import dataclasses
import json

from . import _lib


@dataclasses.dataclass
class ModelConfig:
    hidden_size: int
    num_hidden_layers: int
    vocab_size: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    num_experts: int
    num_experts_per_tok: int
    moe_intermediate_size: int
    shared_expert_intermediate_size: int
    linear_num_key_heads: int
    linear_num_value_heads: int
    linear_key_head_dim: int
    linear_value_head_dim: int
    linear_conv_kernel_dim: int = 4
    full_attention_interval: int = 4
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e7
    partial_rotary_factor: float = 0.25
    norm_topk_prob: bool = False
    quant_group_size: int = 64
    architecture: str = "qwen3.6"

    # ---- reference ModelConfig helpers ----
    def head_dim_(self) -> int:
        return self.head_dim

    def is_gdn_layer(self, layer_idx: int) -> bool:
        return (layer_idx % self.full_attention_interval) != (self.full_attention_interval - 1)

    def is_attention_layer(self, layer_idx: int) -> bool:
        return not self.is_gdn_layer(layer_idx)

    def num_attention_layers(self) -> int:
        return sum(1 for l in range(self.num_hidden_layers) if self.is_attention_layer(l))

    def num_gdn_layers(self) -> int:
        return self.num_hidden_layers - self.num_attention_layers()

    def gqa_group_size(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    def sub_index(self, layer_idx: int) -> int:
        """Index among GDN layers or among attention layers (reference port_scheduler
        mapping gdn_idx = 3*(l//4) + l%4, att_idx = l//4 for interval 4)."""
        same = self.is_attention_layer(layer_idx)
        return sum(1 for l in range(layer_idx) if self.is_attention_layer(l) == same)

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def qkv_dim(self) -> int:
        return (2 * self.linear_num_key_heads * self.linear_key_head_dim
                + self.linear_num_value_heads * self.linear_value_head_dim)

    @property
    def z_dim(self) -> int:
        return self.linear_num_value_heads * self.linear_value_head_dim

    def expert_bytes(self) -> int:
        """Bytes of one expert (gate + up + down) in the 4-bit group format."""
        H, I, G = self.hidden_size, self.moe_intermediate_size, self.quant_group_size
        per = lambda rows, cols: rows * cols // 2 + rows * (cols // G) * 2 + rows * (cols // G) // 2
        return 2 * per(I, H) + per(H, I)

    def to_c(self) -> _lib.DmModelConfig:
        c = _lib.DmModelConfig()
        for f, _ in _lib.DmModelConfig._fields_:
            v = getattr(self, f)
            setattr(c, f, int(v) if not isinstance(v, float) else v)
        return c

    @classmethod
    def from_hf_config(cls, path: str, **overrides) -> "ModelConfig":
        """Reads a HF config.json (text_config when present), as the reference
        config_parser does (src/cli/config_parser.mojo; Qwen3.6: theta 1e7, partial 0.25)."""
        with open(path, encoding="utf-8") as f:
            raw = json.load(f)
        t = raw.get("text_config", raw)
        rope = t.get("rope_parameters", {})
        kw = dict(
            hidden_size=t["hidden_size"], num_hidden_layers=t["num_hidden_layers"],
            vocab_size=t["vocab_size"], num_attention_heads=t["num_attention_heads"],
            num_key_value_heads=t.get("num_key_value_heads", t["num_attention_heads"]),
            head_dim=t.get("head_dim", t["hidden_size"] // t["num_attention_heads"]),
            num_experts=t["num_experts"], num_experts_per_tok=t["num_experts_per_tok"],
            moe_intermediate_size=t["moe_intermediate_size"],
            shared_expert_intermediate_size=t.get("shared_expert_intermediate_size", t["moe_intermediate_size"]),
            linear_num_key_heads=t.get("linear_num_key_heads", 16),
            linear_num_value_heads=t.get("linear_num_value_heads", 32),
            linear_key_head_dim=t.get("linear_key_head_dim", 128),
            linear_value_head_dim=t.get("linear_value_head_dim", 128),
            linear_conv_kernel_dim=t.get("linear_conv_kernel_dim", 4),
            full_attention_interval=t.get("full_attention_interval", 4),
            rms_norm_eps=t.get("rms_norm_eps", 1e-6),
            rope_theta=rope.get("rope_theta", t.get("rope_theta", 1e7)),
            partial_rotary_factor=rope.get("partial_rotary_factor", t.get("partial_rotary_factor", 0.25)),
            norm_topk_prob=bool(t.get("norm_topk_prob", False)),
        )
        kw.update(overrides)
        return cls(**kw)


@dataclasses.dataclass
class RuntimeConfig:
    max_seqs: int = 1
    kv_page_tokens: int = 16
    kv_num_pages: int = 0          # 0: max_seqs * max_pages_per_seq
    max_pages_per_seq: int = 64
    expert_cache_slots: int = 0    # 0: all experts in HBM; C: C per layer in HBM, the rest in host memory

    @classmethod
    def for_context(cls, max_ctx: int, max_seqs: int = 1, extra_pages: int = 0) -> "RuntimeConfig":
        pages = (max_ctx + 15) // 16
        return cls(max_seqs=max_seqs, max_pages_per_seq=pages, kv_num_pages=max_seqs * pages + extra_pages)

    def to_c(self) -> _lib.DmRuntimeConfig:
        n = self.kv_num_pages or self.max_seqs * self.max_pages_per_seq
        return _lib.DmRuntimeConfig(self.max_seqs, self.kv_page_tokens, n, self.max_pages_per_seq,
                                    self.expert_cache_slots)


def preset(name: str) -> ModelConfig:
    if name in ("mini", "config0"):
        return ModelConfig(hidden_size=256, num_hidden_layers=4, vocab_size=1024, num_attention_heads=4,
                           num_key_value_heads=1, head_dim=64, num_experts=16, num_experts_per_tok=4,
                           moe_intermediate_size=128, shared_expert_intermediate_size=128,
                           linear_num_key_heads=2, linear_num_value_heads=4, linear_key_head_dim=64,
                           linear_value_head_dim=64)
    full = dict(hidden_size=2048, num_attention_heads=16, num_key_value_heads=2, head_dim=256,
                num_experts=256, num_experts_per_tok=8, moe_intermediate_size=512,
                shared_expert_intermediate_size=512, linear_num_key_heads=16, linear_num_value_heads=32,
                linear_key_head_dim=128, linear_value_head_dim=128)
    if name in ("layer", "config1"):
        return ModelConfig(num_hidden_layers=2, full_attention_interval=2, vocab_size=1024, **full)
    if name in ("full", "config2"):
        return ModelConfig(num_hidden_layers=40, vocab_size=151936, **full)
    raise KeyError(name)
