"""Prefill benchmark (its prefill half) behind `bench.py --workload c4`.

Workload: the 40-block Qwen3.6-35B-A3B-shaped model (random-init weights generated on the
device, seed 4), 8 sequences x 8192 random token ids (seed 4), each prompt run through
dm_prefill into its own slot (chunks of dm_prefill_rows tokens through every layer: dense
projections and experts on the tcgen05 tensor cores, the GDN recurrence over the chunk,
causal paged attention over the cache plus the chunk).  W untimed prefills of the first
prompt (slot reset after each), then the K timed ones (K <= 8 sequences: one step = one
sequence's prompt).

  value     prompt tokens/s = K x 8192 / device time of the K dm_prefill calls (CUDA events
            on the library stream around them; each call copies its prompt from host
            memory and reads the next token back, so the copies are inside already)
  e2e       the same tokens over the host wall clock of the K calls
  roofline  tensor-bound: the algorithmic FLOPs of the prompts (dense projections, router,
            the 9 active experts, causal attention scores and P V; computed once, not the
            hi/lo operand doubling the kernels run) over the device time, against the
            measured bf16 GEMM peak
"""
from __future__ import annotations

import json
import time

import numpy as np

C4_SEQS, C4_LEN = 8, 8192


def c4_metric() -> str:
    return "prefill tok/s, 35B-A3B-shape 4-bit, 8 x 8192 tokens"


def c4_workload(B: int, L: int) -> str:
    return (f"config4 prefill: 40-block Qwen3.6-35B-A3B-shape, 4-bit g64 experts, {B} sequences x {L} random "
            "prompt tokens, chunked prefill through dm_prefill")


def prefill_flops(cfg, L: int) -> float:
    """Algorithmic FLOPs of one L-token prompt (multiply-add = 2)."""
    H, I = cfg.hidden_size, cfg.moe_intermediate_size
    D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    n_att, n_gdn, nl = cfg.num_attention_layers(), cfg.num_gdn_layers(), cfg.num_hidden_layers
    gdn_in = cfg.qkv_dim + cfg.z_dim + 2 * cfg.linear_num_value_heads
    per_tok = (n_gdn * 2 * (gdn_in * H + H * cfg.z_dim)
               + n_att * 2 * ((2 * Hq * D + 2 * Hkv * D) * H + H * Hq * D)
               + nl * 2 * (cfg.num_experts + 1) * H
               + nl * (cfg.num_experts_per_tok + 1) * 2 * 3 * H * I
               + n_gdn * 6 * cfg.linear_num_value_heads * cfg.linear_value_head_dim * cfg.linear_key_head_dim)
    # causal attention: token t scores and mixes t + 1 positions
    attn = n_att * 4.0 * Hq * D * (L * (L + 1) / 2)
    head = 2.0 * cfg.vocab_size * H
    return per_tok * L + attn + head


def run(args, rank, local, world):
    import torch

    from . import Engine, RuntimeConfig, build, preset
    from bench import ClockSampler, cpu_baseline_line, measured_peak  # noqa: the repo root is on sys.path

    if world > 1 or rank != 0:
        # one sequence's prefill does not shard here: replicas would only repeat this line
        if rank == 0:
            print(json.dumps({"metric": c4_metric(), "unavailable": "c4 runs on one GPU"}), flush=True)
        return 0
    build.build()
    torch.cuda.set_device(local)
    cfg = preset("full")
    B, L = C4_SEQS, C4_LEN
    K = max(1, min(args.steps, B))
    W = min(max(0, args.warmup), 3)  # each warm-up is a whole 8192-token prefill
    pps = (L + 16 + 15) // 16
    rt = RuntimeConfig(max_seqs=B, max_pages_per_seq=pps, kv_num_pages=B * pps)
    rng = np.random.default_rng(4)
    prompts = rng.integers(0, cfg.vocab_size, (B, L)).astype(np.int32)
    t0 = time.perf_counter()
    with Engine(cfg, rt, device=local) as eng:
        eng.synth_on_device(4)
        perm = np.random.default_rng(4).permutation(B * pps).astype(np.int32)
        for s in range(B):
            eng.set_page_table(s, perm[s * pps:(s + 1) * pps])
        setup_s = time.perf_counter() - t0
        rows, kpc = eng.prefill_rows()
        stream = torch.cuda.ExternalStream(eng.stream(), device=torch.device("cuda", local))
        for _ in range(W):
            eng.seq_reset(0)
            eng.prefill(prompts[0], slot=0, want_logits=False)
        eng.seq_reset(0)
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        nxt = []
        torch.cuda.synchronize()
        with ClockSampler(local) as clocks:
            torch.cuda.nvtx.range_push("dm_timed")  # ncu --nvtx-include dm_timed/ selects the timed launches
            w0 = time.perf_counter()
            ev0.record(stream)
            for s in range(K):
                _, t = eng.prefill(prompts[s], slot=s, want_logits=False)
                nxt.append(int(t))
            ev1.record(stream)
            ev1.synchronize()
            wall = time.perf_counter() - w0
            torch.cuda.nvtx.range_pop()
        ms = ev0.elapsed_time(ev1)
        lens = [eng.seq_len(s) for s in range(K)]
    assert lens == [L] * K, lens
    value = K * L / (ms / 1e3)
    e2e = K * L / wall
    peak, peak_kind = measured_peak("bf16_tflops")
    flops = prefill_flops(cfg, L) * K
    achieved = flops / (ms / 1e3) / 1e12
    chunks = (L + rows - 1) // rows
    cpu = None
    if not args.no_cpu_baseline:
        cpu = cpu_baseline_line(cfg, 4, 4096, args.cpu_sample_steps)
        cpu["sample"] += ("; the CPU restatement runs a prompt token by token (as the reference's full-shape "
                          "blocks do), so its prefill rate is its decode rate")
    line = {
        "metric": c4_metric(), "value": value, "unit": "tokens/s", "n_gpus": 1, "steps": K, "warmup": W,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights generated on the device, random prompt ids, seed 4)",
        "config": {"workload": c4_workload(B, L), "global_batch": K, "seq_len": L, "parallelism": "1 GPU",
                   "prefill_rows_per_chunk": rows, "chunks_per_sequence": chunks,
                   "l2": "inputs larger than L2 (every chunk streams the 20 GB of weights)"},
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 4 * L + 8, "d2h_bytes_per_step": 4},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak if peak else None, "traffic": None, "peak_source": peak_kind,
                     "kernel": "whole prefill: algorithmic FLOPs of the prompts (counted once) over the device time"},
        "flops_per_sequence": prefill_flops(cfg, L),
        "next_tokens": nxt,
        "cpu_baseline": cpu,
        "clocks": clocks.summary(),
        "gpu_launches": K * (chunks * kpc + 4),
        "library_gemms": 0,
        "context_setup_s": round(setup_s, 2),
    }
    print(json.dumps(line), flush=True)
    return 0
