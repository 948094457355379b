"""The reference arm of bench.py on the host: the JSON line the benchmark driver reads.

`bench.py --impl reference` times the CPU restatement of the reference decode step (real
40-block tokens of the config-2 model) and prints one line with the main arm's metric, unit
and config object, as many timed steps as asked.  It must use every CPU the process may
run on even when the launcher (torchrun) sets OMP_NUM_THREADS=1, and it must not load the
CUDA library (its weights come from the oracle's copy of the seeded generator).
"""
import json
import os
import re
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _main_arm_metric() -> str:
    src = open(os.path.join(ROOT, "bench.py")).read()
    found = set(re.findall(r'^C2_METRIC = "(decode tok/s[^"]*bs1)"', src, flags=re.M))
    assert len(found) == 1, found
    return found.pop()


def test_reference_arm_json_line_uses_every_cpu():
    env = dict(os.environ, OMP_NUM_THREADS="1")
    code = ("import runpy, sys; sys.argv = ['bench.py', '--impl', 'reference', '--steps', '2', '--warmup', '0'];"
            "rc = 0\ntry:\n    runpy.run_path('bench.py', run_name='__main__')\n"
            "except SystemExit as e:\n    rc = e.code or 0\n"
            "maps = open('/proc/self/maps').read()\n"
            "print('CUDA_LIB_MAPPED' if 'libdismoen_cuda' in maps else 'CUDA_LIB_NOT_MAPPED')\nsys.exit(rc)")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, env=env, capture_output=True, text=True,
                         timeout=900)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = out.stdout.strip().splitlines()
    assert lines[-1] == "CUDA_LIB_NOT_MAPPED"
    line = json.loads(lines[-2])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["metric"] == _main_arm_metric()
    assert line["unit"] == "tokens/s" and line["higher_is_better"] is True
    assert line["value"] > 0
    assert line["steps"] == 2 and line["warmup"] == 0
    assert line["config"]["workload"].startswith("config2") and line["config"]["seq_len"] == 4096
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["value"] == line["value"]
    assert cpu["cores"] == len(os.sched_getaffinity(0))


def test_workload_resolution(monkeypatch):
    """A plain run measures config 2 (bs1 on one GPU); under torchrun (any world size, 1
    included) or with --gpus > 1 the default is the config-3 expert-parallel step, so the
    1 -> 8 GPU scaling run measures the batch-64 curve."""
    sys.path.insert(0, ROOT)
    import bench
    for var in ("TORCHELASTIC_RUN_ID", "LOCAL_WORLD_SIZE"):
        monkeypatch.delenv(var, raising=False)
    args = lambda gpus, wl=None: type("A", (), {"workload": wl, "gpus": gpus})()
    assert bench.resolve_workload(args(1), 1) == "c2"
    assert bench.resolve_workload(args(2), 2) == "c3"
    assert bench.resolve_workload(args(1, "spill"), 1) == "spill"
    monkeypatch.setenv("TORCHELASTIC_RUN_ID", "x")
    assert bench.resolve_workload(args(1), 1) == "c3"
    assert bench.resolve_workload(args(8, "c2"), 8) == "c2"
