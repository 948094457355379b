"""Host-spill streaming of the expert pool (RuntimeConfig.expert_cache_slots).

CPU: the library's residency policy (dm_spill_simulate) against a plain restatement of the
documented rule on random routing traces: every selected expert resident after its layer is
resolved, misses take a free slot or the least recently used unpinned slot the step does
not need, pinned experts are never evicted, pinning stays within 25 % of the slots (the
contract of the reference's expert cache, src/io/lru_cache.mojo:225-610).
GPU: decoding with a spilling pool gives bit for bit the logits of the all-resident context
(the same kernels read the same records, only from cache slots), single-sequence decode
included; statistics count the traffic; capacity and unsupported calls are refused.
"""
import ctypes as C

import numpy as np
import pytest

from disk_streaming_moe_engine_b200 import DmError, Engine, RuntimeConfig, _lib, preset, synth


class PolicyModel:
    """The residency rule, restated."""

    def __init__(self, L, E, Cs):
        self.L, self.E, self.C = L, E, Cs
        self.slot_of = [[-1] * E for _ in range(L)]
        self.exp_in = [[-1] * Cs for _ in range(L)]
        self.stamp = [[0] * Cs for _ in range(L)]
        self.pinned = [[False] * Cs for _ in range(L)]
        self.clock = 0
        self.st = [0] * 6

    def _victim(self, l, in_use):
        for s in range(self.C):
            if self.exp_in[l][s] < 0 and s not in in_use:
                return s
        cand = [s for s in range(self.C) if s not in in_use and not self.pinned[l][s]]
        return min(cand, key=lambda s: (self.stamp[l][s], s)) if cand else -1

    def _place(self, l, e, in_use):
        s = self._victim(l, in_use)
        assert s >= 0
        old = self.exp_in[l][s]
        if old >= 0:
            self.slot_of[l][old] = -1
            self.st[3] += 1
        self.exp_in[l][s] = e
        self.slot_of[l][e] = s
        self.clock += 1
        self.stamp[l][s] = self.clock
        in_use.add(s)
        self.st[4] += 1

    def resolve(self, l, ids):
        u = sorted(set(ids))
        in_use = set()
        for e in u:
            self.st[0] += 1
            s = self.slot_of[l][e]
            if s >= 0:
                self.st[1] += 1
                self.clock += 1
                self.stamp[l][s] = self.clock
                in_use.add(s)
        for e in u:
            if self.slot_of[l][e] < 0:
                self.st[2] += 1
                self._place(l, e, in_use)

    def pin(self, l, e):
        self.st[0] += 1
        if self.slot_of[l][e] < 0:
            self.st[2] += 1
            self._place(l, e, set())
        else:
            self.st[1] += 1
        s = self.slot_of[l][e]
        if self.pinned[l][s]:
            return
        if sum(self.pinned[l]) + 1 > self.C // 4:
            self.st[5] += 1
            return
        self.pinned[l][s] = True


def _simulate(lib, L, E, Cs, ids, pins):
    steps, _, n, topk = ids.shape
    st = (C.c_uint64 * 6)()
    slot_of = np.empty((L, E), np.int32)
    p = np.ascontiguousarray(np.array(pins, np.int32).reshape(-1, 2)) if pins else None
    rc = lib.dm_spill_simulate(L, E, Cs, steps, n, topk, np.ascontiguousarray(ids, np.int32).ctypes.data,
                               None if p is None else p.ctypes.data, len(pins), st, slot_of.ctypes.data)
    return rc, list(st), slot_of


@pytest.mark.parametrize("seed,L,E,Cs,n,topk,skew", [(0, 3, 16, 6, 1, 4, 0.0), (1, 2, 64, 24, 2, 8, 1.1),
                                                     (2, 4, 32, 16, 3, 4, 0.0), (3, 1, 256, 64, 4, 8, 1.1)])
def test_policy_matches_restatement(lib, seed, L, E, Cs, n, topk, skew):
    rng = np.random.default_rng(seed)
    steps = 40
    w = np.arange(1, E + 1, dtype=np.float64) ** (-skew)
    w /= w.sum()
    ids = np.stack([np.stack([np.stack([rng.choice(E, topk, replace=False, p=w) for _ in range(n)])
                              for _ in range(L)]) for _ in range(steps)]).astype(np.int32)
    pins = [(0, int(e)) for e in rng.choice(E, Cs // 4 + 2, replace=False)]
    rc, st, slot_of = _simulate(lib, L, E, Cs, ids, pins)
    assert rc == 0
    m = PolicyModel(L, E, Cs)
    for l, e in pins:
        m.pin(l, e)
    for s in range(steps):
        for l in range(L):
            m.resolve(l, ids[s, l].reshape(-1).tolist())
            assert all(m.slot_of[l][e] >= 0 for e in ids[s, l].reshape(-1))
    assert st == m.st
    assert slot_of.tolist() == m.slot_of
    for e in {e for _, e in pins}:  # pinned experts (within the budget) survived every step
        s = m.slot_of[0][e]
        if s >= 0 and m.pinned[0][s]:
            assert slot_of[0][e] == s
    assert sum(m.pinned[0]) <= Cs // 4 and st[5] >= 2
    assert st[1] + st[2] == st[0] and st[3] <= st[2]


def test_policy_capacity_refused(lib):
    ids = np.arange(8, dtype=np.int32).reshape(1, 1, 2, 4)  # 8 distinct experts, 6 slots
    rc, _, _ = _simulate(lib, 1, 16, 6, ids, [])
    assert rc == _lib.DM_ERR_CAPACITY


def _engines(cfg, m, slots, max_seqs, ctx=96):
    a = Engine(cfg, RuntimeConfig.for_context(ctx, max_seqs=max_seqs))
    b = Engine(cfg, RuntimeConfig(max_seqs=max_seqs, max_pages_per_seq=(ctx + 15) // 16,
                                  kv_num_pages=max_seqs * ((ctx + 15) // 16), expert_cache_slots=slots))
    a.load_model(m)
    b.load_model(m)
    return a, b


def _batched_prefill(eng, prompt, slot):
    out = None
    for t in prompt:
        out, _ = eng.decode_batch(np.array([slot], np.int32), np.array([t], np.int32))
    return int(out[0])


@pytest.mark.gpu
def test_spill_decode_bit_exact_with_resident_pool(lib):
    """3 sequences, 12 slots of 16 experts (top-4): prefill and batched decode give the
    resident pool's ids and logits bit for bit; the device-fed loop too."""
    cfg = preset("mini")
    m = synth.synth_model(cfg, 0)
    a, b = _engines(cfg, m, 12, 3)
    try:
        b.weights_check()
        t = m["layers"][1]
        for e in (0, 7, 15):  # the host pool holds exactly what was uploaded
            for proj, k in ((_lib.DM_PROJ_GATE, "g"), (_lib.DM_PROJ_UP, "u"), (_lib.DM_PROJ_DOWN, "d")):
                q, sc, z = b.expert_download(1, e, proj)
                assert np.array_equal(q, t[k + "q"][e]) and np.array_equal(sc, t[k + "s"][e])
                assert np.array_equal(z, t[k + "z"][e])
        rng = np.random.default_rng(3)
        slots = np.arange(3, dtype=np.int32)
        for i in range(3):  # prefill: the resident pool through one-row batched steps too
            p = rng.integers(0, cfg.vocab_size, 5 + 4 * i).astype(np.int32)
            a.seq_reset(i)
            b.seq_reset(i)
            ta = _batched_prefill(a, p, i)
            _, tb = b.forward(p, slot=i, want_logits=False)
            assert ta == tb
        toks = rng.integers(0, cfg.vocab_size, 3).astype(np.int32)
        for _ in range(6):
            oa, la = a.decode_batch(slots, toks, want_logits=True)
            ob, lb = b.decode_batch(slots, toks, want_logits=True)
            assert np.array_equal(oa, ob) and np.array_equal(la.view(np.uint32), lb.view(np.uint32))
            toks = oa
        assert np.array_equal(a.generate_batch(slots, toks, 4), b.generate_batch(slots, toks, 4))
        st = b.spill_stats()
        assert st["slots"] == 12 and st["misses"] > 0 and st["evictions"] > 0 and st["hits"] > 0
        assert st["bytes_h2d"] == st["loads"] * cfg.expert_bytes()
        assert a.spill_stats()["slots"] == 0
    finally:
        a.close()
        b.close()


@pytest.mark.gpu
def test_spill_single_sequence_pins_and_refusals(lib):
    """Single-sequence decode with 8 slots matches the resident pool; pins are honoured up to
    25 % of the slots; calls that need the whole pool resident are refused, and so is a
    batch the cache cannot hold."""
    cfg = preset("mini")
    m = synth.synth_model(cfg, 0)
    a, b = _engines(cfg, m, 8, 3)
    try:
        assert b.spill_pin(0, 5) and b.spill_pin(0, 9)
        assert not b.spill_pin(0, 11)  # 8 slots: at most 2 pinned
        # a spilling context decodes one sequence through one-row batched steps: bit for bit
        # the resident context's batched path, and within the kernel tolerance of its
        # single-sequence path (other kernels: GEMV vs GEMM, fused MoE vs grouped experts)
        for eng in (a, b):
            eng.seq_reset(0)
            eng.seq_reset(1)
        p = np.random.default_rng(9).integers(0, cfg.vocab_size, 7).astype(np.int32)
        ta = _batched_prefill(a, p, 0)
        ls, ts = a.forward(p, slot=1, want_logits=True)
        lb, tb = b.forward(p, slot=0, want_logits=True)
        assert ta == tb == ts
        assert np.abs(lb - ls).max() / np.abs(ls).max() < 1e-3
        one = np.array([0], np.int32)
        for _ in range(5):
            oa, la = a.decode_batch(one, np.array([ta], np.int32), want_logits=True)
            tb, lb = b.decode_step(tb, slot=0, want_logits=True)
            assert int(oa[0]) == tb and np.array_equal(la[0].view(np.uint32), lb.view(np.uint32))
            ta = tb
        assert a.generate_batch(one, np.array([ta], np.int32), 4)[:, 0].tolist() == b.generate(tb, 4, slot=0).tolist()
        st = b.spill_stats()
        assert st["pins_kept_unpinned"] == 1 and st["misses"] > 0
        for call in (lambda: b.enqueue_decode(1, slot=0),
                     lambda: b.moe_block(np.zeros((1, cfg.hidden_size), np.float32), 0)):
            with pytest.raises(DmError) as ei:
                call()
            assert ei.value.code == _lib.DM_ERR_INVALID_ARG and "SPILL_UNSUPPORTED" in ei.value.message
        # 2 rows x top-4 + 2 pinned > 8 slots
        for i in (1, 2):
            b.seq_reset(i)
        with pytest.raises(DmError) as ei:
            b.decode_batch(np.array([1, 2], np.int32), np.array([3, 4], np.int32))
        assert ei.value.code == _lib.DM_ERR_CAPACITY
    finally:
        a.close()
        b.close()
