"""Multi-rank host logic on CPU (gloo, world size 2): the benchmark's max-over-ranks timing
and whole-job rate, and a rank that fails before a collective being reported to the
others as an error within the process-group timeout (never as a hang)."""
import datetime
import multiprocessing as mp
import os
import socket

import pytest


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist

    import bench
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
        if mode == "max":
            local_ms = [120.0, 95.5][rank]
            m = bench.max_over_ranks(local_ms, dist)
            q.put((rank, m, bench.whole_job_rate(64, world, m)))
        elif mode == "fail":
            if rank == 1:
                raise RuntimeError("injected host-side failure before the collective")
            try:
                bench.max_over_ranks(1.0, dist)
                q.put((rank, "no-error"))
            except Exception as e:  # the survivor sees an error, not a hang
                q.put((rank, "error:" + type(e).__name__))
        dist.destroy_process_group()
    except RuntimeError as e:
        q.put((rank, "raised:" + str(e)))


def _run(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
    alive = [p for p in ps if p.is_alive()]
    for p in alive:
        p.kill()
    out = {}
    while not q.empty():
        item = q.get()
        out[item[0]] = item[1:]
    return out, alive


def test_max_over_ranks_and_rate():
    out, alive = _run("max")
    assert not alive
    for r in (0, 1):
        m, rate = out[r]
        assert m == 120.0
        assert abs(rate - 2 * 64 / 0.120) < 1e-6


def test_failed_rank_is_reported_not_hung():
    out, alive = _run("fail")
    assert not alive, "a rank hung past the process-group timeout"
    assert out[1][0].startswith("raised:")
    assert out[0][0].startswith("error:")
