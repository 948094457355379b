"""CPU tests of the oracle: pinned to the reference's own fp32 oracle through the committed
golden vectors (tests/golden/make_golden.py), plus known-answer tests of the integer and
tie-breaking rules the GPU path must reproduce bit for bit."""
import json
import math
import os

import numpy as np
import pytest

from disk_streaming_moe_engine_b200 import preset, synth

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
SEED = 11


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN, "reference_oracle_full.npz"))


def _inputs(lib, T, H, stream):
    x = np.empty((T, H), np.float32)
    lib.dm_synth_f32(SEED, stream, x.size, 0.0, 1.0, x.ctypes.data)
    return x


def test_golden_meta_matches_seeds():
    meta = json.load(open(os.path.join(GOLDEN, "reference_oracle_full.json")))
    assert meta["seed"] == SEED and meta["x_stream"] == 0xF100 and meta["s_stream"] == 0xF000


def test_gdn_block_matches_reference_oracle(lib, oracle_lib, golden):
    """Full-shape gated DeltaNet (conv k=4, decay gate, 16 QK / 32 V heads x 128) run token
    by token from a random state equals reference forward_gdn_step (oracle_full.py:209)."""
    import oracle
    c1 = preset("layer")
    t = synth.synth_layer(c1, 0, SEED, lib, experts=False)
    om = oracle.OracleModel({"cfg": c1, "layers": {0: t}})
    x = _inputs(lib, 6, 2048, 0xF100)
    S = np.empty((32, 128, 128), np.float32)
    lib.dm_synth_f32(SEED, 0xF000, S.size, 0.0, 0.1, S.ctypes.data)
    conv = np.zeros((3, c1.qkv_dim), np.float32)
    ys = np.array([oracle.gdn_block(om, 0, S, conv, p, x[p]) - x[p] for p in range(6)])
    assert rel(ys, golden["gdn_full_y"]) < 1e-5
    assert rel(S.reshape(-1)[::97], golden["gdn_full_S_sample"]) < 1e-5


@pytest.mark.parametrize("name,pre,layer,T", [("attn_c0", "mini", 3, 20), ("attn_c1", "layer", 1, 6)])
def test_attention_matches_reference_oracle(lib, oracle_lib, golden, name, pre, layer, T):
    """QK-norm + partial RoPE (theta 1e7, factor 0.25) + GQA + sigmoid gate, decode form
    with an fp32 cache, equals reference forward_attn_step (oracle_full.py:279)."""
    import oracle
    cfg = preset(pre)
    t = synth.synth_layer(cfg, layer, SEED, lib, experts=False)
    om = oracle.OracleModel({"cfg": cfg, "layers": {layer: t}}, kv_bf16=False)
    x = _inputs(lib, T, cfg.hidden_size, 0xF101)
    k = np.zeros((T, cfg.num_key_value_heads, cfg.head_dim), np.float32)
    v = np.zeros_like(k)
    ys = np.array([oracle.attn_block(om, layer, k, v, p, x[p]) - x[p] for p in range(T)])
    assert rel(ys, golden[name + "_y"]) < 1e-5


def test_moe_matches_reference_oracle(lib, oracle_lib, golden):
    """Router softmax/top-k, 4-bit experts, SwiGLU, sigmoid shared gate equal reference
    forward_moe_step (oracle_full.py:361) on dequantised weights; same expert ids."""
    import oracle
    cfg = preset("mini")
    t = synth.synth_layer(cfg, 1, SEED, lib)
    om = oracle.OracleModel({"cfg": cfg, "layers": {1: t}})
    xm = _inputs(lib, 8, 256, 0xF102)
    ys, ids = [], []
    for i in range(8):
        y, idd, _ = oracle.moe_block(om, 1, xm[i])
        ys.append(y - xm[i])
        ids.append(idd)
    assert rel(np.array(ys), golden["moe_c0_y"]) < 1e-5
    np.testing.assert_array_equal(np.array(ids), golden["moe_c0_ids"])


def test_det_exp_accuracy(oracle_lib):
    import oracle
    xs = np.concatenate([np.linspace(-87, 0, 20001), np.linspace(0, 88, 2001)]).astype(np.float32)
    got = np.array([oracle.det_exp(float(v)) for v in xs], np.float64)
    want = np.exp(xs.astype(np.float64))
    ulp = np.abs(got - want) / np.spacing(np.float32(want).astype(np.float32)).astype(np.float64)
    assert ulp.max() <= 2.0
    assert oracle.det_exp(-100.0) == 0.0 and oracle.det_exp(0.0) == 1.0


def test_dequant_all_nibbles_and_zeros(oracle_lib):
    """Known answers for every byte value and every zero point: w = s*(q - z), low
    nibble first (weight 2j in bits 0-3)."""
    import oracle
    rows, cols = 16, 512  # 16 zero points x 256 byte values
    q = np.tile(np.arange(256, dtype=np.uint8), (rows, cols // 2 // 256))
    zero = np.arange(16, dtype=np.uint8)
    z = np.repeat(((zero | (zero << 4)).astype(np.uint8))[:, None], cols // 64 // 2, axis=1)
    s = np.full((rows, cols // 64), 0x3C00, np.uint16)  # fp16 1.0
    s[:, 1] = 0x3800  # 0.5 for the second group
    out = oracle.dequant_q4(q, s, z, rows, cols)
    for r in range(rows):
        for c in range(cols):
            byte = q[r, c // 2]
            qv = (byte >> 4) if (c & 1) else (byte & 15)
            sc = 0.5 if (c // 64) == 1 else 1.0
            assert out[r, c] == sc * (int(qv) - r)


def test_router_ties_go_to_lower_id(lib, oracle_lib):
    """topk.mojo:80-96: equal probabilities select the lower expert id first."""
    import oracle
    cfg = preset("mini")
    t = synth.synth_layer(cfg, 0, SEED, lib, experts=False)
    rng = np.random.default_rng(0)
    xn = rng.standard_normal(cfg.hidden_size).astype(np.float32)
    w = t["router"].copy()
    # make experts 9, 4 and 12 identical and dominant
    strong = synth.f32_to_bf16(xn / np.linalg.norm(xn) * 0.5)
    for e in (9, 4, 12):
        w[e] = strong
    t["router"] = w
    om = oracle.OracleModel({"cfg": cfg, "layers": {0: t}})
    ids, probs, _, logits = oracle.router(om, 0, xn)
    assert list(ids[:3]) == [4, 9, 12]
    assert probs[0] == probs[1] == probs[2]
    assert probs.sum() < 1.0 + 1e-5  # no renormalisation


def test_router_no_renormalisation(lib, oracle_lib):
    import oracle
    cfg = preset("mini")
    t = synth.synth_layer(cfg, 0, SEED, lib, experts=False)
    om = oracle.OracleModel({"cfg": cfg, "layers": {0: t}})
    xn = np.random.default_rng(1).standard_normal(cfg.hidden_size).astype(np.float32)
    ids, probs, sg, logits = oracle.router(om, 0, xn)
    z = logits[: cfg.num_experts].astype(np.float64)
    p = np.exp(z - z.max())
    p /= p.sum()
    assert np.allclose(np.sort(p)[::-1][: cfg.num_experts_per_tok], probs, rtol=1e-5)
    assert probs.sum() < 0.999
    assert 0.0 < sg < 1.0 and math.isclose(sg, 1 / (1 + math.exp(-logits[-1])), rel_tol=1e-6)


def test_oracle_decode_deterministic_across_threads(lib, oracle_lib):
    import oracle
    cfg = preset("mini")
    m = synth.synth_model(cfg, 0)
    om = oracle.OracleModel(m)
    outs = []
    for th in (1, 3):
        oracle.set_threads(th)
        st = oracle.OracleState(cfg, 64)
        tok, toks, lg = 7, [], None
        for _ in range(6):
            tok, lg, _ = oracle.decode_step(om, st, tok)
            toks.append(tok)
        outs.append((toks, lg.copy()))
    oracle.set_threads(0)
    assert outs[0][0] == outs[1][0]
    assert np.array_equal(outs[0][1], outs[1][1])


def test_oracle_generator_matches_library_generator(lib, oracle_lib):
    """The oracle's restatement of the seeded generator (used by the CPU baseline so that
    it never maps the CUDA library) gives the library's host generator's bits: every
    tensor of a config-0 model, and long streams of each distribution."""
    import oracle
    cfg = preset("mini")
    a = synth.synth_model(cfg, 5, lib=lib)
    b = synth.synth_model(cfg, 5, lib=oracle.SynthLib())
    for key in ("embed", "final_norm", "lm_head"):
        assert np.array_equal(a[key], b[key]), key
    for l in a["layers"]:
        for name, arr in a["layers"][l].items():
            assert np.array_equal(arr.view(np.uint8), b["layers"][l][name].view(np.uint8)), (l, name)
    olib = oracle.SynthLib()
    n = 1 << 18
    for seed, sid in ((2, 0x5eed0001), (3, (1 << 40) | 7)):
        x, y = np.empty(n, np.uint16), np.empty(n, np.uint16)
        assert lib.dm_synth_bf16(seed, sid, n, 0.0, 1.0, x.ctypes.data) == 0
        assert olib.dm_synth_bf16(seed, sid, n, 0.0, 1.0, y.ctypes.data) == 0
        assert np.array_equal(x, y)
        f, g = np.empty(n, np.float32), np.empty(n, np.float32)
        assert lib.dm_synth_f32(seed, sid, n, 0.5, 0.1, f.ctypes.data) == 0
        assert olib.dm_synth_f32(seed, sid, n, 0.5, 0.1, g.ctypes.data) == 0
        assert np.array_equal(f.view(np.uint32), g.view(np.uint32))
        assert lib.dm_synth_f16_absnormal(seed, sid, n, 0.02, x.ctypes.data) == 0
        assert olib.dm_synth_f16_absnormal(seed, sid, n, 0.02, y.ctypes.data) == 0
        assert np.array_equal(x, y)
