"""GPU parity of the batched decode step (B sequences, one token each per step).

Each batch row is checked against the CPU oracle run on its own sequence (same seeded
weights and prompts): identical greedy ids, logits within BATCH_TOL relative (the batched
dense projections use the hi/lo bf16 split of fp32 activations; experts with more than 8
rows of a step run on the tcgen05 tensor cores with each weight rounded once to fp16 and
fp16 hi/lo activations, experts with at most 8 on the integer path: raw nibbles times two
8-bit digits per activation with a unit per 32 elements).  The rows also agree with the
single-sequence decode step of the same context.  rel(a, b) = max|a - b| / max|b|.
"""
import numpy as np
import pytest

from disk_streaming_moe_engine_b200 import DmError, Engine, RuntimeConfig, _lib, preset, synth

pytestmark = pytest.mark.gpu

KERNEL_TOL = 1e-3
# The batched step's experts round each dequantised weight once to fp16, w = fp16(s (q - z))
# (relative error <= 2^-12, finer than the reference's own bf16 dequantisation), so that
# the tensor cores accumulate a whole expert row in one chain; its logits are held to
# BATCH_TOL against the fp32 oracle (greedy ids identical; the north-star bar on hidden
# states is 1e-2).
BATCH_TOL = 3e-3


def rel(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(np.asarray(b)).max(), 1e-30))


def _run_batch_vs_oracle(cfg, m, eng, prompt_lens, steps, seed):
    """Prompts of `prompt_lens` tokens go through the single-sequence path (slot i), then
    `steps` batched steps over all slots; every row is compared with the oracle."""
    import oracle
    om = oracle.OracleModel(m)
    rng = np.random.default_rng(seed)
    n = len(prompt_lens)
    cap = max(prompt_lens) + steps + 16
    states, nxt = [], []
    for i, L in enumerate(prompt_lens):
        eng.seq_reset(i)
        st = oracle.OracleState(cfg, cap)
        prompt = rng.integers(0, cfg.vocab_size, max(L, 1)).astype(np.int32)
        if L == 0:  # empty history: the first batched step decodes at position 0
            nxt.append(int(prompt[0]))
        else:
            tok_o = None
            for t in prompt:
                tok_o, _, _ = oracle.decode_step(om, st, int(t))
            _, tok = eng.forward(prompt, slot=i, want_logits=False)
            assert tok == tok_o
            nxt.append(tok)
        states.append(st)
    slots = np.arange(n, dtype=np.int32)
    toks = np.array(nxt, np.int32)
    for step in range(steps):
        out, lg = eng.decode_batch(slots, toks, want_logits=True)
        for i in range(n):
            tok_o, lg_o, _ = oracle.decode_step(om, states[i], int(toks[i]))
            assert out[i] == tok_o, (step, i)
            assert rel(lg[i], lg_o) < BATCH_TOL, (step, i, rel(lg[i], lg_o))
        toks = out
    for i, L in enumerate(prompt_lens):
        assert eng.seq_len(i) == L + steps
    return toks


def test_batch_mini_ragged_matches_oracle(lib, oracle_lib):
    """Config 0 shape, 12 sequences with ragged histories (0..40 tokens, page edges),
    6 batched steps: the shared expert (12 rows) on the tcgen05 path, routed experts of
    1-8 rows on the integer path (split into pieces of at most 4)."""
    cfg = preset("mini")
    m = synth.synth_model(cfg, 0)
    with Engine(cfg, RuntimeConfig.for_context(128, max_seqs=12)) as eng:
        eng.load_model(m)
        assert eng.batch_capacity() == 12
        _run_batch_vs_oracle(cfg, m, eng, [0, 1, 3, 15, 16, 17, 31, 32, 33, 40, 5, 9], 6, 11)


def test_batch_full_shape_matches_oracle(lib, oracle_lib):
    """Full block shapes (H 2048, 256 experts top-8, attention 16/2 x 256, GDN 16/32 x 128)
    in a 2-block model with a head: 3 sequences, 3 batched steps."""
    cfg = preset("layer")
    m = synth.synth_model(cfg, 1)
    with Engine(cfg, RuntimeConfig.for_context(96, max_seqs=3)) as eng:
        eng.load_model(m)
        _run_batch_vs_oracle(cfg, m, eng, [2, 17, 40], 3, 12)


def test_batch_matches_single_step_and_device_loop(lib):
    """Rows of the batched step equal the single-sequence step of the same context, and
    the device loop (dm_generate_batch) reproduces the host-driven steps."""
    cfg = preset("mini")
    m = synth.synth_model(cfg, 0)
    rt = RuntimeConfig.for_context(128, max_seqs=8)
    with Engine(cfg, rt) as a, Engine(cfg, rt) as b:
        a.load_model(m)
        b.load_model(m)
        rng = np.random.default_rng(5)
        n = 6
        toks = []
        for i in range(n):
            p = rng.integers(0, cfg.vocab_size, 4 + 3 * i).astype(np.int32)
            for e in (a, b):
                e.seq_reset(i)
                _, t = e.forward(p, slot=i, want_logits=False)
            toks.append(t)
        slots = np.arange(n, dtype=np.int32)
        # single-sequence steps on a, batched on b
        cur = np.array(toks, np.int32)
        ref_steps = []
        for _ in range(5):
            nxt = []
            for i in range(n):
                t, lg1 = a.decode_step(int(cur[i]), slot=i, want_logits=True)
                nxt.append(t)
            ref_steps.append(nxt)
            cur = np.array(nxt, np.int32)
        got = b.generate_batch(slots, np.array(toks, np.int32), 5)
        assert got.tolist() == ref_steps
        for i in range(n):
            assert a.seq_len(i) == b.seq_len(i)


def test_batch_rejects_bad_input(lib):
    cfg = preset("mini")
    m = synth.synth_model(cfg, 0)
    with Engine(cfg, RuntimeConfig.for_context(64, max_seqs=4)) as eng:
        eng.load_model(m)
        for i in range(4):
            eng.seq_reset(i)
        with pytest.raises(DmError) as ei:
            eng.decode_batch([0, 0], [1, 2])
        assert ei.value.code == _lib.DM_ERR_INVALID_ARG
        with pytest.raises(DmError) as ei:
            eng.decode_batch([0, 1, 2, 3, 4], [1, 2, 3, 4, 5])
        assert ei.value.code == _lib.DM_ERR_INVALID_ARG
        with pytest.raises(DmError) as ei:
            eng.decode_batch([0, 1], [1, cfg.vocab_size])
        assert ei.value.code == _lib.DM_ERR_INVALID_ARG
        # nothing ran: lengths unchanged, and a valid batch still works
        assert eng.seq_len(0) == 0
        out, _ = eng.decode_batch([2, 0], [7, 9])
        assert out.shape == (2,)
        assert eng.seq_len(2) == 1 and eng.seq_len(0) == 1


@pytest.mark.parametrize("which", ["mini", "layer"])
def test_batched_router_bit_exact(which, lib, oracle_lib):
    """The batched router (rows normalised by one warp each, emulating the canonical
    512-thread reduction order) gives the oracle's ids and probabilities bit for bit, and
    the same bits as the one-row router."""
    import oracle
    cfg = preset(which)
    m = synth.synth_model(cfg, 3, head=False)
    rng = np.random.default_rng(21)
    with Engine(cfg, RuntimeConfig.for_context(64, max_seqs=10)) as eng:
        eng.load_model(m)
        om = oracle.OracleModel(m)
        for layer in range(cfg.num_hidden_layers):
            xs = rng.standard_normal((10, cfg.hidden_size)).astype(np.float32)
            info = eng.router_forward(xs, layer)            # 10 rows: batched kernel
            for t in range(xs.shape[0]):
                ids, probs, sg, _ = oracle.router(om, layer, xs[t])
                np.testing.assert_array_equal(info.selected_experts[t], ids)
                assert np.array_equal(info.routing_weights[t].view(np.uint32), probs.view(np.uint32))
                one = eng.router_forward(xs[t], layer)      # 1 row: the one-token kernel
                np.testing.assert_array_equal(one.selected_experts[0], info.selected_experts[t])
                assert np.array_equal(one.routing_weights[0].view(np.uint32), info.routing_weights[t].view(np.uint32))
