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


# ---- expert-parallel group set-up (host side) -------------------------------------------
class _FakeEngine:
    """Stands in for Engine on CPU: a rank-specific handle, records what attach receives."""

    def __init__(self, rank):
        self.rank = rank
        self.attached = None

    def ep_ipc_handle(self):
        return bytes([self.rank]) * 64

    def ep_attach(self, rank, world, handles):
        self.attached = (rank, world, handles)


def _ep_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist

    from disk_streaming_moe_engine_b200 import ep
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    eng = _FakeEngine(rank)
    g = ep.attach_group(eng, dist)
    r, w, handles = eng.attached
    q.put((rank, g.rank, g.world, r, w, [h[0] for h in handles], [len(h) for h in handles]))
    dist.destroy_process_group()


def test_ep_handles_exchanged_in_rank_order():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
    for p in ps:
        if p.is_alive():
            p.kill()
    out = {}
    while not q.empty():
        item = q.get()
        out[item[0]] = item[1:]
    assert sorted(out) == [0, 1]
    for rank in (0, 1):
        g_rank, g_world, r, w, first_bytes, lens = out[rank]
        assert (g_rank, g_world, r, w) == (rank, 2, rank, 2)
        assert first_bytes == [0, 1] and lens == [64, 64]


def test_ep_partitions():
    from disk_streaming_moe_engine_b200 import ep
    owners = [ep.expert_owner(e, 256, 8) for e in range(256)]
    assert owners[:32] == [0] * 32 and owners[32] == 1 and owners[-1] == 7
    assert [len(ep.rows_of_rank(64, r, 8)) for r in range(8)] == [8] * 8
    assert list(ep.rows_of_rank(64, 3, 8)) == list(range(24, 32))
    with pytest.raises(ValueError):
        ep.expert_owner(0, 256, 3)
    with pytest.raises(ValueError):
        ep.rows_of_rank(64, 0, 3)
