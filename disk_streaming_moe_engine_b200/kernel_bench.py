"""Times one decode-step kernel in isolation (CUDA events on the library stream).

    python -m disk_streaming_moe_engine_b200.kernel_bench --preset layer --kernel in_proj \
        --layer 0 --iters 20
    python -m disk_streaming_moe_engine_b200.kernel_bench --preset layer --kernel battn \
        --batch 16 --ctx 8192 --iters 5

The model is synthesised on the device; with --warm the layer first runs one real token
(so router ids, activations and the KV position are those of a real step).  Prints one
JSON line: mean microseconds per launch, algorithmic bytes per launch and GB/s.  This is
the small-case driver for ncu captures of a single kernel.
"""
from __future__ import annotations

import argparse
import dataclasses
import json

import numpy as np

from . import _lib
from .config import RuntimeConfig, preset
from .engine import Engine

KERNELS = {"in_proj": _lib.DM_KERNEL_MIXER_IN, "out_proj": _lib.DM_KERNEL_MIXER_OUT,
           "core": _lib.DM_KERNEL_MIXER_CORE, "router": _lib.DM_KERNEL_ROUTER, "moe": _lib.DM_KERNEL_MOE,
           "head": _lib.DM_KERNEL_HEAD}
# trace slots of one small-segment expert kernel: entry and exit of up to 160 CTAs + CTA 0's detail
Q4_MAX_CTAS = 160
Q4_SLOTS = 2 * Q4_MAX_CTAS + 40
# kernels of the batched step (--batch N): layer is the preset's attention or GDN layer
BKERNELS = {"battn": _lib.DM_BKERNEL_ATTN, "bgdn": _lib.DM_BKERNEL_GDN_REC, "bexperts": _lib.DM_BKERNEL_EXPERTS,
            "brouter": _lib.DM_BKERNEL_ROUTER, "bgemm": _lib.DM_BKERNEL_GEMM_IN}


def batched(a, cfg):
    """N sequences of --ctx tokens of synthetic state (permuted page pool), one batched step,
    then the chosen batched kernel timed alone."""
    pps = (a.ctx + 64 + 15) // 16
    rt = RuntimeConfig(max_seqs=a.batch, max_pages_per_seq=pps, kv_num_pages=a.batch * pps)
    with Engine(cfg, rt) as eng:
        eng.synth_on_device(a.seed)
        rng = np.random.default_rng(a.seed)
        perm = rng.permutation(a.batch * pps).astype(np.int32)
        for s in range(a.batch):
            eng.set_page_table(s, perm[s * pps:(s + 1) * pps])
        eng.synth_state(a.seed, 1.0, 0.1, a.ctx)
        slots = np.arange(a.batch, dtype=np.int32)
        eng.decode_batch(slots, rng.integers(0, cfg.vocab_size, a.batch).astype(np.int32))
        layer = a.layer
        if a.kernel == "battn":
            layer = next(l for l in range(cfg.num_hidden_layers) if cfg.is_attention_layer(l))
        elif a.kernel == "bgdn":
            layer = next(l for l in range(cfg.num_hidden_layers) if not cfg.is_attention_layer(l))
        ms, nbytes = eng.time_batch_kernel(a.batch, BKERNELS[a.kernel], layer, a.iters)
        pipe = None
        if a.trace and a.kernel == "bexperts":
            # CTA 0's first 32 groups of each expert kernel, SM cycles after the kernel's first
            # stamp: B issued, MMAs issued, expand start / stores done / arrived, drain waits /
            # accumulator ready / epilogue done, MMAs issued, commit issued, A ready, B ready
            eng.trace_enable(True)
            eng.time_batch_kernel(a.batch, BKERNELS[a.kernel], layer, 1)
            t = eng.trace_read(64 + 640 + 2 * Q4_SLOTS).astype(np.int64)
            eng.trace_enable(False)
            pipe = {}
            for name, blk in (("gate_up", t[64:384]), ("down", t[384:704])):
                st = blk.reshape(-1, 10)
                base = st[st > 0].min() if (st > 0).any() else 0
                pipe[name] = [[int(v) - int(base) if v else None for v in row] for row in st]
            # small-segment kernels (%globaltimer ns): every CTA's entry and exit, CTA 0's items
            for name, off in (("q4_gate_up", 704), ("q4_down", 704 + Q4_SLOTS)):
                blk = t[off:off + Q4_SLOTS]
                ee = blk[:2 * Q4_MAX_CTAS].reshape(-1, 2)
                ee = ee[(ee > 0).all(axis=1)]
                if not len(ee):
                    continue
                base = int(ee[:, 0].min())
                det = blk[2 * Q4_MAX_CTAS:]
                pipe[name] = {"base_ns": base, "entry_max": int(ee[:, 0].max()) - base, "exit_min": int(ee[:, 1].min()) - base,
                              "exit_med": int(np.median(ee[:, 1])) - base, "exit_max": int(ee[:, 1].max()) - base,
                              "cta0": [int(v) - base if v else None for v in det[:33]]}
        print(json.dumps({"kernel": a.kernel, "batch": a.batch, "ctx": a.ctx, "layer": layer, "us": ms * 1e3,
                          "bytes": nbytes, "GBps": nbytes / (ms * 1e-3) / 1e9, "pipeline_us": pipe}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="layer")
    ap.add_argument("--kernel", default="in_proj", choices=sorted(KERNELS) + sorted(BKERNELS))
    ap.add_argument("--batch", type=int, default=0, help="batched-step kernels: sequences per step")
    ap.add_argument("--layer", type=int, default=0)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--ctx", type=int, default=0, help="tokens already in the KV cache / GDN state")
    ap.add_argument("--warm", action="store_true")
    ap.add_argument("--trace", action="store_true", help="also report the kernel's phase stamps")
    ap.add_argument("--seed", type=int, default=1)
    ap.add_argument("--vocab", type=int, default=0, help="override the preset's vocabulary (e.g. 151936 for the head)")
    a = ap.parse_args()
    cfg = preset(a.preset)
    if a.vocab:
        cfg = dataclasses.replace(cfg, vocab_size=a.vocab)
    if a.kernel in BKERNELS:
        if a.batch <= 0:
            raise SystemExit("--batch N is required for the batched kernels")
        return batched(a, cfg)
    with Engine(cfg, RuntimeConfig.for_context(a.ctx + 64)) as eng:
        eng.synth_on_device(a.seed)
        eng.seq_reset(0)
        if a.ctx:
            n_att = cfg.num_attention_layers()
            rng = np.random.default_rng(a.seed)
            k = rng.integers(0x3000, 0x3F80, (a.ctx, cfg.num_key_value_heads, cfg.head_dim), dtype=np.uint16)
            for att in range(n_att):
                eng.kv_import(att, 0, k, k[::-1].copy())
            eng.seq_set_len(0, a.ctx)
        if a.warm:
            x = np.random.default_rng(a.seed).standard_normal((1, cfg.hidden_size)).astype(np.float32)
            eng.forward_port_block(x, a.layer, a.ctx)
        us_ms, nbytes = eng.time_kernel(KERNELS[a.kernel], a.layer, a.iters)
        phases = None
        ctas = None
        if a.trace:  # one more launch with phase stamps (ns relative to the kernel's start)
            eng.trace_enable(True)
            eng.time_kernel(KERNELS[a.kernel], a.layer, 1)
            t = eng.trace_read(1024).astype(np.int64)
            eng.trace_enable(False)
            base = {"core": 0, "moe": 16}.get(a.kernel, 0)
            cta = t[64:].reshape(-1, 6)
            cta = cta[cta[:, 0] != 0]
            if len(cta):  # per-CTA stamps (decode attention): start, ready, pages done, merged, end, SM
                t0 = cta[:, 0].min()
                rel = lambda c: np.round((cta[:, c] - t0) / 1e3, 2)
                q = lambda v: [float(np.min(v)), float(np.median(v)), float(np.max(v))]
                order = np.argsort(cta[:, 0])
                ctas = {"n": int(len(cta)), "start_us": q(rel(0)), "ready_us": q(rel(1)), "pages_done_us": q(rel(2)),
                        "merged_us": q(rel(3)), "end_us": q(rel(4)),
                        "by_start": [[float(rel(0)[i]), float(rel(2)[i]), float(rel(4)[i]), int(cta[i, 5])]
                                     for i in order]}
            if a.kernel == "moe":
                phases = {"cta0": [int(v - t[16]) if v else None for v in t[16:25]],
                          "last": [int(v - t[26]) if v else None for v in t[26:35]]}
            else:
                phases = [int(v - t[base]) if v else None for v in t[base:base + 10]]
                if a.kernel == "core":  # per-page stamps of the traced attention CTA
                    phases += [int(v - t[0]) if v else None for v in t[40:56]]
    print(json.dumps({"kernel": a.kernel, "preset": a.preset, "layer": a.layer, "ctx": a.ctx,
                      "us": us_ms * 1e3, "bytes": nbytes, "GBps": nbytes / us_ms / 1e6, "phases_ns": phases,
                      "ctas": ctas}))


if __name__ == "__main__":
    main()
