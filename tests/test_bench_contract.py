"""The reference arm of bench.py on the host: the JSON line the benchmark driver reads.

`bench.py --impl reference` times the CPU restatement of the reference decode step on a
bounded sample and prints one line with the main arm's metric and unit.  It must use every
CPU the process may run on even when the launcher (torchrun) sets OMP_NUM_THREADS=1.
"""
import json
import os
import re
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _main_arm_metric() -> str:
    src = open(os.path.join(ROOT, "bench.py")).read()
    found = set(re.findall(r'"metric": "(decode tok/s[^"]*bs1)"', src))
    assert len(found) == 1, found
    return found.pop()


def test_reference_arm_json_line_uses_every_cpu():
    env = dict(os.environ, OMP_NUM_THREADS="1")
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0"],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["metric"] == _main_arm_metric()
    assert line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["value"] > 0
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["value"] == line["value"]
    assert cpu["cores"] == len(os.sched_getaffinity(0))
