"""Summarises an ncu launch list (`--metrics gpu__time_duration.sum --csv --log-file F`) of
`bench.py` into per-kernel launches, total time and share of the timed decode steps.

    python -m disk_streaming_moe_engine_b200.ncu_summary launches.csv --warmup 3 --steps 4

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


def summarise(launches, warmup: int, steps: int):
    starts = [i for i, (n, _) in enumerate(launches) if n.startswith("embed_kernel")]
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("csv")
    ap.add_argument("--warmup", type=int, required=True)
    ap.add_argument("--steps", type=int, required=True)
    a = ap.parse_args()
    n, total, rows = summarise(read_launches(a.csv), a.warmup, a.steps)
    print(f"timed decode steps: {a.steps}; launches: {n} ({n / a.steps:.0f} per step); "
          f"serialised kernel time {total / 1e3 / a.steps:.1f} us per step")
    print()
    print("| kernel | launches | total us | per launch us | share |")
    print("|---|---:|---:|---:|---:|")
    for name, c, t, sh in rows:
        print(f"| `{name}` | {c} | {t / 1e3:.1f} | {t / 1e3 / c:.2f} | {sh:.3f} |")


if __name__ == "__main__":
    main()
