"""Batched decode benchmark behind `bench.py --workload c3`.

Workload: the 40-block Qwen3.6-35B-A3B-shaped model (random-init weights generated on the
device, seed 3), B = 64 sequences each holding 32768 cached tokens in 16-token pages whose
page tables are a random permutation of one shared pool (seed 3), bf16 N(0, 1) K/V and
fp32 N(0, 0.1) GDN states and conv windows, then W warm-up and K timed greedy steps of all
64 sequences at once (one token per sequence per step).

Expert load: the synthetic router alone spreads the 512 (row, expert) choices of a layer
almost uniformly.  Config 3 asks for a Zipf(s = 1.1) skewed load, so every layer gets
per-expert router logit offsets (dm_set_router_bias) drawn for that load: expert ranks
follow a seeded permutation per layer, the target selection frequency of rank r is
min(1, c r^-s) with c such that a row selects top-k experts in total, and the offsets are
calibrated by Monte Carlo against logits of unit spread.  The load actually seen on the
device is reported (`routing`).

  value     tokens/s = B K / (device time of K steps replayed on the device)
  e2e       the same through dm_decode_batch with host token buffers, per step
  roofline  the batched paged attention (the largest byte stream: every cached K/V byte of
            all 64 sequences once per attention layer), timed alone, against the measured
            HBM copy bandwidth
"""
from __future__ import annotations

import json
import time

import numpy as np


def zipf_targets(E: int, k: int, s: float) -> np.ndarray:
    """Selection frequency per rank: min(1, c r^-s), summing to k."""
    w = np.arange(1, E + 1, dtype=np.float64) ** (-s)
    lo, hi = 0.0, 1e6
    for _ in range(200):
        c = 0.5 * (lo + hi)
        if np.minimum(1.0, c * w).sum() > k:
            hi = c
        else:
            lo = c
    return np.minimum(1.0, lo * w)


def calibrate_offsets(E: int, k: int, s: float, seed: int, samples: int = 8192, iters: int = 60) -> np.ndarray:
    """Logit offsets b (rank order) such that top-k of (b + N(0,1)) selects rank r with
    frequency zipf_targets(E, k, s)[r]."""
    target = zipf_targets(E, k, s)
    rng = np.random.default_rng(seed)
    b = np.log(np.maximum(target, 1e-6))
    b -= b.max()
    for _ in range(iters):
        z = rng.standard_normal((samples, E)) + b
        top = np.argpartition(-z, k, axis=1)[:, :k]
        freq = np.bincount(top.ravel(), minlength=E) / samples
        b += 0.5 * (np.log(np.maximum(target, 1e-4)) - np.log(np.maximum(freq, 0.5 / samples)))
        b -= np.median(b)  # only differences matter: keep the offsets anchored
        b = np.minimum(b, 8.0)
    return b.astype(np.float32)


def c3_metric(B: int) -> str:
    return f"decode tok/s, 35B-A3B-shape 4-bit, bs{B}"


def c3_workload(B: int, L: int) -> str:
    name = "config4 long-context decode" if (B, L) == (4, 131072) else "config3"
    return (f"{name}: 40-block Qwen3.6-35B-A3B-shape decode, 4-bit g64 experts, {B} sequences x {L} cached "
            "tokens, paged (16-token pages, permuted pool)")


def c3_config(args, world: int, cfg) -> dict:
    """The config object of a config-3 line (both arms of bench.py print the same one)."""
    B, L = args.batch, args.c3_ctx
    skew = None
    if args.router_skew > 0:
        b = calibrate_offsets(cfg.num_experts, cfg.num_experts_per_tok, args.router_skew, 3)
        skew = {"zipf_s": args.router_skew, "offset_range": [float(b.min()), float(b.max())]}
    return {"workload": c3_workload(B, L), "global_batch": B, "seq_len": L,
            "parallelism": "1 GPU" if world == 1 else
            f"expert-parallel x{world}: {B // world} sequences and {cfg.num_experts // world} experts per GPU, "
            "dense weights replicated, dispatch/combine through peer memory",
            "l2": "inputs larger than L2 (tens of GB of KV per step)", "router_skew": skew}


def apply_router_skew(eng, cfg, s: float, seed: int) -> dict:
    E, k = cfg.num_experts, cfg.num_experts_per_tok
    b = calibrate_offsets(E, k, s, seed)
    rng = np.random.default_rng(seed + 1)
    for layer in range(cfg.num_hidden_layers):
        perm = rng.permutation(E)          # expert id of each rank
        bias = np.empty(E, np.float32)
        bias[perm] = b
        eng.set_router_bias(layer, bias)
    return {"zipf_s": s, "offset_range": [float(b.min()), float(b.max())]}


def step_bytes_c3(cfg, B: int, ctx_mid: int, experts_per_layer: float) -> dict:
    H = cfg.hidden_size
    n_att, n_gdn, L = cfg.num_attention_layers(), cfg.num_gdn_layers(), cfg.num_hidden_layers
    D, Hq, Hkv = cfg.head_dim, cfg.num_attention_heads, cfg.num_key_value_heads
    gdn_w = ((cfg.qkv_dim + cfg.z_dim + 2 * cfg.linear_num_value_heads) * H + cfg.qkv_dim * 4
             + H * cfg.z_dim + cfg.linear_value_head_dim + 2 * H) * 2 + 8 * cfg.linear_num_value_heads
    att_w = ((2 * Hq * D + 2 * Hkv * D) * H + H * Hq * D + 2 * D + 2 * H) * 2
    dense = n_gdn * gdn_w + n_att * att_w + (cfg.num_experts + 1) * H * 2 * L + cfg.vocab_size * H * 2 + H * 2
    kv = B * n_att * (ctx_mid + 1) * 2 * Hkv * D * 2
    state = B * n_gdn * (2 * cfg.linear_num_value_heads * cfg.linear_value_head_dim * cfg.linear_key_head_dim * 4
                         + 5 * cfg.qkv_dim * 4)
    experts = int((experts_per_layer + 1) * cfg.expert_bytes() * L)
    emb = B * H * 2
    return {"total": dense + kv + state + experts + emb, "dense": dense, "kv": kv, "gdn_state": state,
            "experts": experts}


def run(args, rank, local, world):
    import datetime

    import torch

    from . import Engine, RuntimeConfig, _lib, build, ep, preset
    from bench import ClockSampler, cpu_baseline_line, measured_peak  # noqa: the repo root is on sys.path

    build.build()
    torch.cuda.set_device(local)
    dist = None
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    def rank_max(v: float) -> float:
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize()

    cfg = preset("full")
    B, L, K, W = args.batch, args.c3_ctx, args.steps, args.warmup
    rows = ep.rows_of_rank(B, rank, world)   # this rank's sequences
    n = len(rows)
    pps = (L + W + 2 * K + 64 + 15) // 16
    rt = RuntimeConfig(max_seqs=n, max_pages_per_seq=pps, kv_num_pages=n * pps)
    eng = Engine(cfg, rt, device=local)
    t0 = time.perf_counter()
    eng.synth_on_device(3)             # the same weights on every rank
    eng.weights_check()
    skew = apply_router_skew(eng, cfg, args.router_skew, 3) if args.router_skew > 0 else None
    rng = np.random.default_rng(3 + rank)
    perm = rng.permutation(n * pps).astype(np.int32)
    for sl in range(n):
        eng.set_page_table(sl, perm[sl * pps:(sl + 1) * pps])
    eng.synth_state(3 + rank, 1.0, 0.1, L)
    if dist is not None:
        ep.attach_group(eng, dist)
    setup_s = time.perf_counter() - t0
    stream = torch.cuda.ExternalStream(eng.stream(), device=dev)
    slots = np.arange(n, dtype=np.int32)
    toks = rng.integers(0, cfg.vocab_size, n).astype(np.int32)

    eng.enqueue_decode_batch(slots, toks, W)
    eng.sync()
    toks = eng.batch_read_generated(n, W)[-1].copy()
    eng.batch_stats(reset=True)

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(local) as clocks:
        torch.cuda.nvtx.range_push("dm_timed")  # ncu --nvtx-include dm_timed/ selects the timed launches
        ev0.record(stream)
        eng.enqueue_decode_batch(slots, toks, K)
        ev1.record(stream)
        torch.cuda.nvtx.range_pop()
        ev1.synchronize()
    eng.sync()
    barrier()
    ms = rank_max(ev0.elapsed_time(ev1))
    routing = eng.batch_stats(reset=True)
    toks = eng.batch_read_generated(n, K)[-1].copy()
    value = B * K / (ms / 1e3)

    # e2e: one dm_decode_batch call per step, host token buffers in and out
    barrier()
    with ClockSampler(local, 0.02) as clocks_e2e:
        ev0.record(stream)
        for _ in range(K):
            toks, _ = eng.decode_batch(slots, toks)
        ev1.record(stream)
        ev1.synchronize()
    barrier()
    ms_e2e = rank_max(ev0.elapsed_time(ev1))
    e2e = B * K / (ms_e2e / 1e3)

    peak, peak_kind = measured_peak()
    kernels = None
    roofline = None
    if world == 1:  # kernels timed alone (in a group the ranks would not stay in step)
        kernels = {}
        for name, which, layer in (("attn", _lib.DM_BKERNEL_ATTN, 3), ("gdn_rec", _lib.DM_BKERNEL_GDN_REC, 0),
                                   ("experts", _lib.DM_BKERNEL_EXPERTS, cfg.num_hidden_layers - 1)):
            kms, kb = eng.time_batch_kernel(n, which, layer, 5)
            kernels[name] = {"us": round(kms * 1e3, 1), "bytes": kb, "GBps": round(kb / kms / 1e6, 1),
                             "frac": round(kb / kms / 1e6 / peak, 3)}
        dom = kernels["attn"]
        achieved = dom["bytes"] / (dom["us"] * 1e-6) / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                    "traffic": None, "peak_source": peak_kind,
                    "kernel": "attn_decode_warp_kernel<256,8> (layer 3): every cached K/V byte of the "
                              f"{n} sequences, timed alone after an L2 flush"}
    ctx_mid = L + W + K // 2
    # bytes one rank moves per step: its sequences' KV and state, the replicated dense
    # weights, the experts it computes (touched experts counted per rank)
    sb = step_bytes_c3(cfg, n, ctx_mid, routing["experts_touched_per_layer"])
    own, gemms = eng.batch_kernels_per_step(n)
    if world > 1:
        own += cfg.num_hidden_layers  # the cross-rank barrier kernel of every MoE layer
    if dist is not None:
        barrier()
        eng.ep_detach()
    eng.close()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_line(cfg, 3, L, args.cpu_sample_steps)
    line = {
        "metric": c3_metric(B), "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms / K, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights and sequence state on device, seed 3)",
        "config": c3_config(args, world, cfg),
        "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": 8 * B, "d2h_bytes_per_step": 4 * B + 4 * world},
        "roofline": roofline,
        "step_roofline": {"bytes_per_step_per_gpu": sb, "achieved_GBps_per_gpu": sb["total"] / (ms / K / 1e3) / 1e9,
                          "frac": sb["total"] / (ms / K / 1e3) / 1e9 / peak},
        "kernels": kernels,
        "cpu_baseline": cpu,
        "routing": routing,
        "clocks": clocks.summary(),
        "clocks_e2e": clocks_e2e.summary(),
        "gpu_launches": own * K,
        "library_gemms": gemms * K,
        "context_setup_s": round(setup_s, 2),
        "router_skew_applied": skew,
    }
    if dist is not None:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0
