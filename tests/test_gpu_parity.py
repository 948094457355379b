"""GPU parity: libdismoen_cuda.so (through its C ABI) against the CPU oracle on the same
seeded inputs.

Bars: bit-exact nibble unpack, top-k expert ids (ties to the lower
id), page-table gathers and KV append positions; per-layer hidden-state max relative error
<= 1e-2 against the fp32 oracle (each kernel is held to 1e-3 here); identical greedy ids
over 32 decode steps.  rel(a, b) = max|a - b| / max|b|.
"""
import numpy as np
import pytest

from disk_streaming_moe_engine_b200 import DmError, Engine, RuntimeConfig, _lib, preset, synth

pytestmark = pytest.mark.gpu

KERNEL_TOL = 1e-3
HIDDEN_TOL = 1e-2


def rel(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(np.asarray(b)).max(), 1e-30))


@pytest.fixture(scope="module")
def mini(lib, oracle_lib):
    import oracle
    cfg = preset("mini")
    m = synth.synth_model(cfg, 0)
    eng = Engine(cfg, RuntimeConfig.for_context(256))
    eng.load_model(m)
    eng.weights_check()
    yield cfg, m, eng, oracle.OracleModel(m)
    eng.close()


@pytest.fixture(scope="module")
def layer1(lib, oracle_lib):
    """Config 1: one full-shape GDN block (layer 0) and one attention block (layer 1)."""
    import oracle
    cfg = preset("layer")
    m = synth.synth_model(cfg, 1, head=False)
    eng = Engine(cfg, RuntimeConfig.for_context(4096 + 64))
    eng.load_model(m)
    yield cfg, m, eng, oracle.OracleModel(m)
    eng.close()


def _rng(seed):
    return np.random.default_rng(seed)


# ---- quant loader ----------------------------------------------------------------------
def test_dequant_q4_bit_exact(mini):
    import oracle
    cfg, m, eng, om = mini
    rng = _rng(2)
    rows, cols = 96, 512
    q = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    s = np.abs(rng.standard_normal((rows, cols // 64)) * 0.02).astype(np.float16).view(np.uint16)
    z = rng.integers(0, 256, (rows, cols // 64 // 2), dtype=np.uint8)
    got = eng.dequant_q4(q, s, z, rows, cols)
    want = oracle.dequant_q4(q, s, z, rows, cols)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ---- router ------------------------------------------------------------------------------
@pytest.mark.parametrize("which", ["mini", "layer1"])
def test_router_bit_exact(which, request):
    import oracle
    cfg, m, eng, om = request.getfixturevalue(which)
    rng = _rng(3)
    for layer in range(cfg.num_hidden_layers):
        xs = rng.standard_normal((6, cfg.hidden_size)).astype(np.float32)
        info = eng.router_forward(xs, layer)
        for t in range(xs.shape[0]):
            ids, probs, sg, _ = oracle.router(om, layer, xs[t])
            np.testing.assert_array_equal(info.selected_experts[t], ids)
            assert np.array_equal(info.routing_weights[t].view(np.uint32), probs.view(np.uint32))
            assert abs(info.shared_gate[t] - sg) < 1e-6


def test_router_ties_on_gpu(lib, oracle_lib):
    import oracle
    cfg = preset("mini")
    t = synth.synth_layer(cfg, 0, 11, lib, experts=False)
    xn = _rng(0).standard_normal(cfg.hidden_size).astype(np.float32)
    strong = synth.f32_to_bf16(xn / np.linalg.norm(xn) * 0.5)
    for e in (9, 4, 12):
        t["router"][e] = strong
    with Engine(cfg, RuntimeConfig.for_context(64)) as eng:
        eng.upload_tensor(0, _lib.DM_T_ROUTER, t["router"])
        eng.upload_tensor(0, _lib.DM_T_SHARED_GATE, t["shared_gate"])
        info = eng.router_forward(xn, 0)
    om = oracle.OracleModel({"cfg": cfg, "layers": {0: t}})
    ids, probs, _, _ = oracle.router(om, 0, xn)
    assert list(info.selected_experts[0][:3]) == [4, 9, 12]
    np.testing.assert_array_equal(info.selected_experts[0], ids)


# ---- MoE block ---------------------------------------------------------------------------
@pytest.mark.parametrize("which", ["mini", "layer1"])
def test_moe_block(which, request):
    import oracle
    cfg, m, eng, om = request.getfixturevalue(which)
    rng = _rng(4)
    for layer in range(min(2, cfg.num_hidden_layers)):
        xm = (rng.standard_normal((3, cfg.hidden_size)) * 3).astype(np.float32)
        y = eng.moe_block(xm, layer)
        for t in range(3):
            want, _, _ = oracle.moe_block(om, layer, xm[t])
            assert rel(y[t] - xm[t], want - xm[t]) < KERNEL_TOL


# ---- GDN block (config 1) --------------------------------------------------------------
def test_gdn_block_config1_with_state(layer1):
    import oracle
    cfg, m, eng, om = layer1
    rng = _rng(5)
    L0 = 4096
    S = (rng.standard_normal((32, 128, 128)) * 0.1).astype(np.float32)
    conv = rng.standard_normal((3, cfg.qkv_dim)).astype(np.float32)
    eng.seq_reset(0)
    eng.seq_set_len(0, L0)
    eng.gdn_state_import(0, 0, S, conv)
    x = rng.standard_normal((4, cfg.hidden_size)).astype(np.float32)
    y = eng.mixer_block(x, 0, L0)
    S_o, conv_o = S.copy(), conv.copy()
    for t in range(4):
        want = oracle.gdn_block(om, 0, S_o, conv_o, L0 + t, x[t])
        assert rel(y[t] - x[t], want - x[t]) < KERNEL_TOL
    eng.seq_set_len(0, L0 + 4)
    S_g, conv_g = eng.gdn_state_export(0, 0)
    assert rel(S_g, S_o) < KERNEL_TOL
    assert rel(conv_g, conv_o) < KERNEL_TOL


# ---- attention block (config 1, KV 4096) ------------------------------------------------
def _kv(rng, n, cfg):
    k = synth.f32_to_bf16(rng.standard_normal((n, cfg.num_key_value_heads, cfg.head_dim)).astype(np.float32))
    v = synth.f32_to_bf16(rng.standard_normal((n, cfg.num_key_value_heads, cfg.head_dim)).astype(np.float32))
    return k, v


@pytest.mark.parametrize("permuted", [False, True])
def test_attention_block_config1_paged(layer1, permuted):
    import oracle
    cfg, m, eng, om = layer1
    rng = _rng(6)
    n0, T = 4096, 3
    k, v = _kv(rng, n0, cfg)
    eng.seq_reset(0)
    if permuted:  # page tables randomly permuted over the pool (config 3 layout)
        pages = _rng(3).permutation(eng.rt.kv_num_pages)[: eng.rt.max_pages_per_seq]
        eng.set_page_table(0, pages)
    eng.kv_import(0, 0, k, v)
    ke, ve = eng.kv_export(0, 0, n0)
    assert np.array_equal(ke, k) and np.array_equal(ve, v)  # page gather is bit-exact
    x = rng.standard_normal((T, cfg.hidden_size)).astype(np.float32)
    y = eng.mixer_block(x, 1, n0)
    cap = n0 + T
    kc = np.zeros((cap, cfg.num_key_value_heads, cfg.head_dim), np.uint16)
    vc = np.zeros_like(kc)
    kc[:n0], vc[:n0] = k, v
    for t in range(T):
        want = oracle.attn_block(om, 1, kc, vc, n0 + t, x[t])
        assert rel(y[t] - x[t], want - x[t]) < KERNEL_TOL
    ke, ve = eng.kv_export(0, 0, cap)
    assert np.array_equal(ke[:n0], k)
    # appended rows: same positions, values within one bf16 rounding of the oracle's
    kf, kw = synth.bf16_to_f32(ke[n0:]), synth.bf16_to_f32(kc[n0:])
    assert rel(kf, kw) < 1e-2


def test_kv_append_position_contract(layer1):
    cfg, m, eng, om = layer1
    eng.seq_reset(0)
    x = np.zeros((1, cfg.hidden_size), np.float32)
    with pytest.raises(DmError) as ei:
        eng.mixer_block(x, 1, 5)  # current_len is 0
    assert ei.value.code == _lib.DM_ERR_POSITION and "M5_ERR_DECODE" in ei.value.message
    cap = eng.rt.max_pages_per_seq * 16
    with pytest.raises(DmError) as ei:
        eng.seq_set_len(0, cap + 1)
    assert ei.value.code == _lib.DM_ERR_CAPACITY


# ---- full model (config 0) --------------------------------------------------------------
def test_block_forward_per_layer(mini):
    """Per-layer hidden state (same input to both) across the 4 blocks, 6 tokens."""
    import oracle
    cfg, m, eng, om = mini
    st = oracle.OracleState(cfg, 64)
    eng.seq_reset(0)
    rng = _rng(7)
    for t in range(6):
        x = rng.standard_normal(cfg.hidden_size).astype(np.float32)
        for l in range(cfg.num_hidden_layers):
            y = eng.forward_port_block(x[None], l, t)[0]
            want = np.empty_like(x)
            om.lib.or_block_forward(oracle.C.byref(om.model), oracle.C.byref(st.st), l, x.ctypes.data,
                                    want.ctypes.data, None)
            assert rel(y, want) < KERNEL_TOL, (t, l)
            x = want
        st.st.len += 1


def test_decode_32_prompt_32_greedy_matches_oracle(mini):
    """Config 0: 32 prompt tokens + 32 greedy steps; identical ids, close logits."""
    import oracle
    cfg, m, eng, om = mini
    prompt = _rng(0).integers(0, cfg.vocab_size, 32).astype(np.int32)
    st = oracle.OracleState(cfg, 128)
    hid_o = None
    for tok in prompt:
        nxt_o, lg_o, hid_o = oracle.decode_step(om, st, int(tok), hidden=True)
    eng.seq_reset(0)
    lg, nxt = eng.forward(prompt)
    assert nxt == nxt_o
    assert rel(lg, lg_o) < KERNEL_TOL
    greedy_o = [nxt_o]
    tok = nxt_o
    for _ in range(31):
        tok, lg_o, _ = oracle.decode_step(om, st, tok)
        greedy_o.append(tok)
    got = eng.generate(nxt, 31)
    assert [nxt] + list(got) == greedy_o, (list(got), greedy_o)
    assert eng.seq_len(0) == 32 + 31


def test_decode_step_logits_and_determinism(mini):
    import oracle
    cfg, m, eng, om = mini
    outs = []
    for _ in range(2):
        eng.seq_reset(0)
        st = oracle.OracleState(cfg, 64)
        tok, seq, lgs = 3, [], []
        for _ in range(5):
            tok_o, lg_o, _ = oracle.decode_step(om, st, tok)
            nxt, lg = eng.decode_step(tok, want_logits=True)
            assert nxt == tok_o
            assert rel(lg, lg_o) < KERNEL_TOL
            lgs.append(lg)
            tok = nxt
        outs.append(np.stack(lgs))
    assert np.array_equal(outs[0].view(np.uint32), outs[1].view(np.uint32))


def test_nonfinite_logits_reported(lib):
    cfg = preset("mini")
    m = synth.synth_model(cfg, 0)
    m["lm_head"] = m["lm_head"].copy()
    m["lm_head"][:] = 0x7FC0  # NaN
    with Engine(cfg, RuntimeConfig.for_context(64)) as eng:
        eng.load_model(m)
        with pytest.raises(DmError) as ei:
            eng.decode_step(1)
        assert ei.value.code == _lib.DM_ERR_NONFINITE
        # the context stays usable after the error
        m2 = synth.synth_model(cfg, 0)
        eng.upload_tensor(-1, _lib.DM_T_LM_HEAD, m2["lm_head"])
        eng.seq_reset(0)
        eng.decode_step(1)
