"""Host-spill decode benchmark behind `bench.py --workload spill` (one GPU).

Workload: the config-2 model (40 blocks, 256 experts top-8, random-init weights made on the
device, seed 2) with only `--expert-slots` routed expert records per layer in HBM and all
256 per layer in pinned host memory; seeded synthetic context of `--prompt-len` tokens;
then `--warmup` + `--steps` greedy single-sequence decode steps (dm_decode_step, one-row
batched steps with the residency decided on the host after each layer's router).  The
same steps run on an all-resident context through the same one-row batched path, so the
difference is the spill traffic and the per-layer host round trips.

  value      tokens/s of the spilling context (device-event time of the K steps)
  resident   tokens/s of the resident context, same path
  spill      hit rate, records and bytes copied host -> HBM per token, the copy rate
"""
from __future__ import annotations

import json
import time

import numpy as np


def run(args) -> int:
    import torch

    from . import Engine, RuntimeConfig, build, preset
    from bench import ClockSampler, synthetic_context  # noqa: the repo root is on sys.path (bench.py)

    build.build()
    torch.cuda.set_device(0)
    cfg = preset("full")
    n_ctx = args.prompt_len
    pages = (n_ctx + args.warmup + args.steps + 64 + 15) // 16
    results = {}
    for slots in (args.expert_slots, 0):
        rt = RuntimeConfig(max_seqs=1, max_pages_per_seq=pages, kv_num_pages=pages, expert_cache_slots=slots)
        eng = Engine(cfg, rt)
        t0 = time.perf_counter()
        eng.synth_on_device(args.seed)
        eng.weights_check()
        setup = time.perf_counter() - t0
        tok = synthetic_context(eng, cfg, n_ctx, args.seed)
        one = np.zeros(1, np.int32)
        stream = torch.cuda.ExternalStream(eng.stream())
        for _ in range(args.warmup):
            tok = int(eng.decode_batch(one, np.array([tok], np.int32))[0][0])
        s0 = eng.spill_stats()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        with ClockSampler(0) as clocks:
            ev0.record(stream)
            for _ in range(args.steps):
                tok = int(eng.decode_batch(one, np.array([tok], np.int32))[0][0])
            ev1.record(stream)
            ev1.synchronize()
        wall = time.perf_counter() - w0
        ms = ev0.elapsed_time(ev1)
        s1 = eng.spill_stats()
        d = {k: s1[k] - s0[k] for k in s1 if k != "slots"}
        results[slots] = {"tok_s": args.steps / (ms / 1e3), "ms_per_token": ms / args.steps,
                          "wall_tok_s": args.steps / wall, "setup_s": round(setup, 1), "clocks": clocks.summary(),
                          "device_bytes": eng.device_bytes(), "stats": d}
        eng.close()
    sp, rs = results[args.expert_slots], results[0]
    st = sp["stats"]
    line = {
        "metric": "decode tok/s with a host-spilled expert pool, 35B-A3B-shape 4-bit, bs1",
        "value": sp["tok_s"], "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sp["ms_per_token"], "higher_is_better": True, "dtype": "bf16",
        "data": "synthetic (random-init weights on the device, seeded synthetic context)",
        "config": {"workload": f"config2 with {args.expert_slots} of {cfg.num_experts} routed experts per layer "
                               f"resident in HBM, the rest in pinned host memory; context {n_ctx} tokens",
                   "global_batch": 1, "seq_len": n_ctx},
        "resident_same_path": {"tok_s": rs["tok_s"], "ms_per_token": rs["ms_per_token"]},
        "spill": {"hit_rate": st["hits"] / max(st["accesses"], 1),
                  "records_loaded_per_token": st["loads"] / args.steps,
                  "bytes_h2d_per_token": st["bytes_h2d"] / args.steps,
                  "h2d_GBps": st["bytes_h2d"] / (sp["ms_per_token"] * args.steps / 1e3) / 1e9,
                  "evictions": st["evictions"]},
        "hbm_bytes": {"spilling": sp["device_bytes"], "resident": rs["device_bytes"]},
        "clocks": sp["clocks"], "wall_tok_s": sp["wall_tok_s"],
    }
    print(json.dumps(line), flush=True)
    return 0
