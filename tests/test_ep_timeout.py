"""Failure detection of the expert-parallel step: a peer that never enters the step.

Two processes form an expert-parallel group (CUDA IPC handles exchanged over gloo); rank 1
attaches and then never runs a step.  Rank 0's batched step waits at the group's device
barrier for a flag that nothing sets: the bounded wait gives up after 1 s, raises the
timeout bit in the context's error word and the kernels finish without the peer's work;
the host returns DM_ERR_TIMEOUT.  Rank 0 then leaves the group and its context stays
usable: a fresh sequence decodes exactly like the oracle.  Only rank 0 ever has kernels
in flight, so the two processes may share one GPU; no GPU faults or hangs.
"""
import datetime
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, dev, q, done):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    try:
        import time

        import torch
        import torch.distributed as dist

        from disk_streaming_moe_engine_b200 import DmError, Engine, RuntimeConfig, _lib, ep, preset, synth
        torch.cuda.set_device(dev)
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        cfg = preset("mini")
        m = synth.synth_model(cfg, 0)
        eng = Engine(cfg, RuntimeConfig.for_context(64, max_seqs=2), device=dev)
        eng.load_model(m)
        for i in range(2):
            eng.seq_reset(i)
        ep.attach_group(eng, dist)
        result = None
        if rank == 0:
            t0 = time.perf_counter()
            try:
                eng.decode_batch(np.arange(2, dtype=np.int32), np.array([5, 9], np.int32))
                result = ("no error", None, 0.0)
            except DmError as e:
                result = (e.code, e.message, time.perf_counter() - t0)
            eng.ep_detach()
            # the context is usable again: a fresh sequence through the single-sequence and
            # the batched paths
            eng.seq_reset(0)
            _, nxt = eng.forward(np.array([3, 1, 4, 1, 5], np.int32), slot=0, want_logits=False)
            eng.seq_reset(1)
            out, _ = eng.decode_batch(np.arange(2, dtype=np.int32), np.array([nxt, 7], np.int32))
            q.put((rank, "ok", result, int(nxt), [int(v) for v in out]))
            done.set()
        else:
            done.wait(120)  # never enters a step; stays attached until rank 0 is finished
            eng.ep_detach()
            q.put((rank, "ok", None, None, None))
        dist.barrier()  # no rank frees its memory while the other still maps it
        eng.close()
        dist.destroy_process_group()
    except Exception as e:  # reported to the test, never a hang of the parent
        q.put((rank, "error", repr(e), None, None))
        done.set()


def test_peer_that_never_enters_the_step_times_out(lib, oracle_lib):
    import torch

    import oracle
    from disk_streaming_moe_engine_b200 import _lib, preset, synth
    devs = (0, 1) if torch.cuda.device_count() >= 2 else (0, 0)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    done = ctx.Event()
    port = _free_port()
    ps = [ctx.Process(target=_rank_main, args=(r, 2, port, devs[r], q, done)) for r in range(2)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(2):
        item = q.get(timeout=600)
        res[item[0]] = item[1:]
    for p in ps:
        p.join(120)
        if p.is_alive():
            p.kill()
    assert res[1][0] == "ok", res[1]
    assert res[0][0] == "ok", res[0]
    code, msg, secs = res[0][1]
    assert code == _lib.DM_ERR_TIMEOUT, (code, msg)
    assert "DEVICE_TIMEOUT" in msg
    assert secs < 30  # two bounded waits of about 1 s each, no hang
    # after leaving the group the context decodes like the oracle
    cfg = preset("mini")
    om = oracle.OracleModel(synth.synth_model(cfg, 0))
    st = oracle.OracleState(cfg, 64)
    tok = None
    for t in (3, 1, 4, 1, 5):
        tok, _, _ = oracle.decode_step(om, st, t)
    assert res[0][2] == tok
    tok2, _, _ = oracle.decode_step(om, st, tok)
    assert res[0][3][0] == tok2
