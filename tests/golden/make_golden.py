"""Generates the golden vectors that pin the CPU oracle to the reference implementation.

Run where a checkout of the reference repository is available, giving its path as an
argument or in the environment variable DISMOEN_REFERENCE:

    python tests/golden/make_golden.py --reference <reference checkout>

The reference's own PyTorch fp32 oracle (tools/oracle/oracle_full.py: forward_gdn_step,
forward_attn_step, forward_moe_step) is imported from the reference checkout and run on
seeded synthetic inputs produced by this repository's counter-based generator
(disk_streaming_moe_engine_b200.synth); only the small outputs are stored, the inputs are
regenerated from the seeds by the tests.  The reference is never needed at test time.

Cases (all fp32 outputs, no residual):
  gdn_full   forward_gdn_step at the full Qwen3.6 shape (the reference hard-codes 8192 qkv
             channels, 16 QK / 32 V heads x 128), T=6 tokens from a random initial state;
             y [T, 2048] and a strided sample of the final state.
  attn_c0    forward_attn_step at config-0 shape (4Q/1KV x 64, theta 1e7, partial 0.25),
             T=20 causal tokens (fp32 K/V as in the reference prefill path).
  attn_c1    forward_attn_step at config-1 shape (16Q/2KV x 256), T=6.
  moe_c0     forward_moe_step at config-0 shape (16 experts top-4 + shared, I=128) with the
             4-bit experts dequantised as fp32 (w = scale * (q - zero), low nibble first),
             T=8 tokens; also the selected expert ids.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from disk_streaming_moe_engine_b200 import _lib, preset, synth  # noqa: E402

SEED = 11
X_STREAM = 0xF100      # input activations N(0, 1)
S_STREAM = 0xF000      # initial GDN state N(0, 0.1)


def inputs(lib, T, H, stream):
    x = np.empty((T, H), np.float32)
    lib.dm_synth_f32(SEED, stream, x.size, 0.0, 1.0, x.ctypes.data)
    return x


def rms_ref(torch, x, w_bf16, eps):
    """reference forward_single_hybrid_layer RMSNorm (oracle_full.py:449-451)."""
    w = torch.from_numpy(synth.bf16_to_f32(w_bf16))
    xt = torch.from_numpy(x)
    var = torch.mean(xt ** 2, dim=-1, keepdim=True)
    return xt * torch.rsqrt(var + eps) * w


def deq_np(q, s, z, group=64):
    """Independent numpy dequantisation of the asymmetric 4-bit format."""
    rows = q.shape[0]
    cols = q.shape[1] * 2
    qv = np.empty((rows, cols), np.int32)
    qv[:, 0::2] = q & 15
    qv[:, 1::2] = q >> 4
    ng = cols // group
    zv = np.empty((rows, ng), np.int32)
    zv[:, 0::2] = z & 15
    zv[:, 1::2] = z >> 4
    sc = s.view(np.float16).astype(np.float32)
    return (np.repeat(sc, group, axis=1) * (qv - np.repeat(zv, group, axis=1)).astype(np.float32)).astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DISMOEN_REFERENCE", ""),
                    help="reference checkout (default: $DISMOEN_REFERENCE)")
    args = ap.parse_args()
    if not args.reference or not os.path.isdir(args.reference):
        raise SystemExit("make_golden.py: give the reference checkout with --reference or DISMOEN_REFERENCE")
    sys.path.insert(0, os.path.join(args.reference, "tools", "oracle"))
    import torch
    import oracle_full as ref  # the reference's fp32 oracle
    from safetensors.torch import save_file

    lib = _lib.load()
    out = {}
    meta = {"seed": SEED, "x_stream": X_STREAM, "s_stream": S_STREAM, "reference": "tools/oracle/oracle_full.py"}

    # ---- GDN at full shape ----
    c1 = preset("layer")
    t = synth.synth_layer(c1, 0, SEED, lib, experts=False)
    T = 6
    x = inputs(lib, T, c1.hidden_size, X_STREAM)
    S0 = np.empty((32, 128, 128), np.float32)
    lib.dm_synth_f32(SEED, S_STREAM, S0.size, 0.0, 0.1, S0.ctypes.data)
    f = lambda a: torch.from_numpy(synth.bf16_to_f32(a) if a.dtype == np.uint16 else a)
    w = {
        "linear_attn.in_proj_qkv.weight": f(t["qkv"]),
        "linear_attn.conv1d.weight": f(t["conv"]).view(8192, 1, 4),
        "linear_attn.in_proj_z.weight": f(t["z"]),
        "linear_attn.in_proj_a.weight": f(t["a"]),
        "linear_attn.in_proj_b.weight": f(t["b"]),
        "linear_attn.dt_bias": f(t["dt_bias"]),
        "linear_attn.A_log": f(t["a_log"]),
        "linear_attn.norm.weight": f(t["gnorm"]),
        "linear_attn.out_proj.weight": f(t["out"]),
    }
    xn = rms_ref(torch, x, t["in_norm"], c1.rms_norm_eps)
    with torch.no_grad():
        y, s_new = ref.forward_gdn_step(xn, w, torch.from_numpy(S0.copy()), T, c1.rms_norm_eps)
    out["gdn_full_y"] = y.numpy().astype(np.float32)
    out["gdn_full_S_sample"] = s_new.numpy().reshape(-1)[::97].astype(np.float32)
    meta["gdn_full"] = {"T": T, "layer": 0, "preset": "layer", "S_sample_stride": 97}

    # ---- attention ----
    for name, pre, layer, T in (("attn_c0", "mini", 3, 20), ("attn_c1", "layer", 1, 6)):
        cfg = preset(pre)
        t = synth.synth_layer(cfg, layer, SEED, lib, experts=False)
        x = inputs(lib, T, cfg.hidden_size, X_STREAM + 1)
        w = {"self_attn.q_proj.weight": f(t["q"]), "self_attn.k_proj.weight": f(t["k"]),
             "self_attn.v_proj.weight": f(t["v"]), "self_attn.q_norm.weight": f(t["qn"]),
             "self_attn.k_norm.weight": f(t["kn"]), "self_attn.o_proj.weight": f(t["o"])}
        rcfg = {"num_attention_heads": cfg.num_attention_heads, "num_key_value_heads": cfg.num_key_value_heads,
                "head_dim": cfg.head_dim, "rms_norm_eps": cfg.rms_norm_eps, "rope_theta": cfg.rope_theta,
                "partial_rotary_factor": cfg.partial_rotary_factor}
        xn = rms_ref(torch, x, t["in_norm"], cfg.rms_norm_eps)
        with torch.no_grad():
            y = ref.forward_attn_step(xn, w, T, rcfg)
        out[name + "_y"] = y.numpy().astype(np.float32)
        meta[name] = {"T": T, "layer": layer, "preset": pre}

    # ---- MoE at config-0 shape ----
    cfg = preset("mini")
    layer, T = 1, 8
    t = synth.synth_layer(cfg, layer, SEED, lib, experts=True)
    E, I, H = cfg.num_experts, cfg.moe_intermediate_size, cfg.hidden_size
    gate = np.stack([deq_np(t["gq"][e], t["gs"][e], t["gz"][e]) for e in range(E + 1)])
    up = np.stack([deq_np(t["uq"][e], t["us"][e], t["uz"][e]) for e in range(E + 1)])
    down = np.stack([deq_np(t["dq"][e], t["ds"][e], t["dz"][e]) for e in range(E + 1)])
    pfx = f"model.language_model.layers.{layer}."
    tensors = {
        pfx + "mlp.gate.weight": f(t["router"]).contiguous(),
        pfx + "mlp.experts.gate_up_proj": torch.from_numpy(np.concatenate([gate[:E], up[:E]], axis=1)),
        pfx + "mlp.experts.down_proj": torch.from_numpy(down[:E].copy()),
        pfx + "mlp.shared_expert.gate_proj.weight": torch.from_numpy(gate[E].copy()),
        pfx + "mlp.shared_expert.up_proj.weight": torch.from_numpy(up[E].copy()),
        pfx + "mlp.shared_expert.down_proj.weight": torch.from_numpy(down[E].copy()),
        pfx + "mlp.shared_expert_gate.weight": f(t["shared_gate"]).view(1, H).contiguous(),
    }
    x_mid = inputs(lib, T, H, X_STREAM + 2)
    with tempfile.TemporaryDirectory() as tmp:
        save_file(tensors, os.path.join(tmp, "model.safetensors"))
        wmap = {k: "model.safetensors" for k in tensors}
        rcfg = {"num_experts_per_tok": cfg.num_experts_per_tok, "moe_intermediate_size": I}
        xn = rms_ref(torch, x_mid, t["post_norm"], cfg.rms_norm_eps)
        routing = os.path.join(tmp, "routing")
        os.makedirs(routing)
        with torch.no_grad():
            y = ref.forward_moe_step(xn, tmp, wmap, pfx, layer, rcfg, routing)
        with open(os.path.join(routing, f"routing_L{layer}.json")) as fh:
            sel = json.load(fh)["selected_experts"]
    out["moe_c0_y"] = y.numpy().astype(np.float32)
    out["moe_c0_ids"] = np.asarray(sel, np.int32)
    meta["moe_c0"] = {"T": T, "layer": layer, "preset": "mini"}

    np.savez_compressed(os.path.join(HERE, "reference_oracle_full.npz"), **out)
    with open(os.path.join(HERE, "reference_oracle_full.json"), "w") as fh:
        json.dump(meta, fh, indent=2)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
