"""Summarises ncu output for profiles/:

* a launch list (`--metrics gpu__time_duration.sum --csv --log-file F`) of `bench.py` into
  per-kernel launches, total time and share of the timed decode steps:

    python -m disk_streaming_moe_engine_b200.ncu_summary launches.csv --warmup 3 --steps 4
    (batched step: --marker b_embed_kernel)

* a full capture (`ncu -i rep --page raw --csv > raw.csv`) into the figures a roofline
  needs, per captured launch, and the top warp stall reasons:

    python -m disk_streaming_moe_engine_b200.ncu_summary --full raw.csv --alg-bytes N

A decode step starts with its embedding kernel, so the launches of the timed steps are
those from the (warmup+1)-th `embed_kernel` up to the (warmup+steps+1)-th.  ncu serialises
the launches and runs each from a cold cache, so absolute times are longer than in the
step; the shares are what compare with the bench's own timeline.
"""
from __future__ import annotations

import argparse
import csv
import io
import re


def read_launches(path: str):
    """[(kernel short name, ns)] in launch order."""
    text = "".join(l for l in open(path) if not l.startswith("=="))
    out = []
    for row in csv.DictReader(io.StringIO(text)):
        if row.get("Metric Name") != "gpu__time_duration.sum":
            continue
        ns = float(row["Metric Value"].replace(",", ""))
        if row.get("Metric Unit") == "us":
            ns *= 1e3
        elif row.get("Metric Unit") == "ms":
            ns *= 1e6
        out.append((short_name(row["Kernel Name"]), ns))
    return out


def short_name(k: str) -> str:
    k = re.sub(r"^void\s+", "", k)
    k = re.sub(r"\(.*$", "", k)  # drop the parameter list
    return k.replace("dm::", "")


def summarise(launches, warmup: int, steps: int, marker: str = "embed_kernel"):
    starts = [i for i, (n, _) in enumerate(launches) if n.startswith(marker)]
    if len(starts) < warmup + steps:
        raise SystemExit(f"only {len(starts)} decode steps in the launch list")
    a = starts[warmup]
    b = starts[warmup + steps] if len(starts) > warmup + steps else len(launches)
    sel = launches[a:b]
    by = {}
    for n, ns in sel:
        d = by.setdefault(n, [0, 0.0])
        d[0] += 1
        d[1] += ns
    total = sum(v[1] for v in by.values())
    rows = sorted(by.items(), key=lambda kv: -kv[1][1])
    return len(sel), total, [(n, c, t, t / total) for n, (c, t) in rows]


FULL_METRICS = [
    "gpu__time_duration.sum", "dram__bytes_read.sum", "dram__bytes_write.sum",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed", "sm__throughput.avg.pct_of_peak_sustained_elapsed",
    "sm__inst_executed_pipe_tensor_subpipe_hmma.avg.pct_of_peak_sustained_active",
    "TPC.TriageCompute.sm__pipe_tensor_cycles_active_realtime.avg.pct_of_peak_sustained_elapsed",
    "sm__ops_path_tensor_op_hmma_src_bf16_dst_fp32_sparsity_off.avg.pct_of_peak_sustained_elapsed",
    "sm__inst_executed_pipe_tmem.avg.pct_of_peak_sustained_active",
    "sm__pipe_alu_cycles_active.avg.pct_of_peak_sustained_active",
    "smsp__issue_active.avg.pct_of_peak_sustained_active", "sm__warps_active.avg.pct_of_peak_sustained_active",
    "l1tex__data_bank_conflicts_pipe_lsu_mem_shared.sum", "launch__registers_per_thread", "launch__grid_size",
    "launch__block_size",
]


def summarise_full(path: str, alg_bytes: float | None):
    """(kernel names, {metric: [value with unit per launch]}, top stall reasons of launch 1)."""
    rows = list(csv.reader(open(path)))
    hdr, units, data = rows[0], rows[1], rows[2:]
    col = {h: i for i, h in enumerate(hdr)}
    names = [short_name(r[col["Kernel Name"]]) for r in data]
    table = {m: [f"{r[col[m]]} {units[col[m]]}".strip() for r in data] for m in FULL_METRICS if m in col}
    stall = []
    pat = re.compile(r"^smsp__average_warps_issue_stalled_(.+)_per_issue_active\.ratio$")
    for h, i in col.items():
        mm = pat.match(h)
        if mm and data:
            try:
                stall.append((float(data[0][i].replace(",", "")), mm.group(1)))
            except ValueError:
                pass
    stall.sort(reverse=True)
    traffic = None
    if "dram__bytes_read.sum" in col and data:
        def to_bytes(v, u):
            v = float(v.replace(",", ""))
            return v * {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}.get(u, 1)
        r = data[0]
        traffic = to_bytes(r[col["dram__bytes_read.sum"]], units[col["dram__bytes_read.sum"]]) + to_bytes(
            r[col["dram__bytes_write.sum"]], units[col["dram__bytes_write.sum"]])
    print(f"kernels: {', '.join(dict.fromkeys(names))}")
    if traffic is not None:
        print(f"\ndram_bytes_per_launch: {traffic:.0f}")
        if alg_bytes:
            print(f"\ntraffic / algorithmic = {traffic / alg_bytes:.3f}")
    print()
    print("| metric | " + " | ".join(f"launch {i + 1}" for i in range(len(data))) + " |")
    print("|---|" + "---|" * len(data))
    for m, vals in table.items():
        print(f"| `{m}` | " + " | ".join(vals) + " |")
    print("\nTop warp stall reasons (cycles per issued instruction, launch 1):\n")
    for v, name in stall[:8]:
        print(f"* {name}: {v:.3f}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("csv")
    ap.add_argument("--warmup", type=int, default=0)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--marker", default="embed_kernel", help="first kernel of a step")
    ap.add_argument("--full", action="store_true", help="csv is a raw page of a full capture")
    ap.add_argument("--alg-bytes", type=float, default=None)
    a = ap.parse_args()
    if a.full:
        summarise_full(a.csv, a.alg_bytes)
        return
    n, total, rows = summarise(read_launches(a.csv), a.warmup, a.steps, a.marker)
    print(f"timed decode steps: {a.steps}; launches: {n} ({n / a.steps:.0f} per step); "
          f"serialised kernel time {total / 1e3 / a.steps:.1f} us per step")
    print()
    print("| kernel | launches | total us | per launch us | share |")
    print("|---|---:|---:|---:|---:|")
    for name, c, t, sh in rows:
        print(f"| `{name}` | {c} | {t / 1e3:.1f} | {t / 1e3 / c:.2f} | {sh:.3f} |")


if __name__ == "__main__":
    main()
