"""The quant-file loaders: GGUF and the reference's custom 4-bit file.

CPU: the oracle's GGUF dequantisers (oracle/or_formats.c) give the reference oracle's fp32
bits (tests/golden/make_golden_formats.py ran tools/oracle/oracle_port.py) on a synthetic
file of every type and on tensors of the reference fixture fixtures/m9_port_mini.gguf;
the library's native index parsers read those files (directory, metadata, offsets) and
reject what the reference's parsers reject, with its messages; this repository's quant
file writer equals the reference writer; the exact custom-4-bit -> pool conversion and
the re-quantisation rule (oracle) behave as documented.
GPU: the device dequantisers equal the golden bits (fp32; bf16 = its nearest-even
rounding; the gguf.mojo Q4_K reading equals the oracle's), the pool conversions equal the
oracle's bytes, and whole models loaded from a quant file and from a GGUF decode like the
CPU oracle run on the same weights.
"""
import json
import os
import struct

import numpy as np
import pytest

import formats_util as fu
from disk_streaming_moe_engine_b200 import DmError, _lib
from disk_streaming_moe_engine_b200.formats import FormatError, parse_gguf_index, scan_quant_file

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def gold():
    z = np.load(os.path.join(GOLD, "reference_formats.npz"))
    meta = json.load(open(os.path.join(GOLD, "reference_formats.json")))
    return z, meta


def _syn_cases(z, meta):
    data = bytes(z["syn_bytes"])
    idx_meta = meta["syn"]["tensors"]
    return data, idx_meta


def _write(tmp_path, name, data: bytes) -> str:
    p = str(tmp_path / name)
    with open(p, "wb") as f:
        f.write(data)
    return p


# ---------------------------------------------------------------- CPU: oracle vs golden
def test_oracle_gguf_dequant_matches_reference(gold, oracle_lib, tmp_path):
    import oracle
    z, meta = gold
    data, tensors = _syn_cases(z, meta)
    idx = parse_gguf_index(_write(tmp_path, "syn.gguf", data))
    for i, t in enumerate(tensors):
        raw = idx.read_raw(t["name"])
        n = int(np.prod(t["shape"]))
        got = oracle.gguf_dequant(raw, t["type"], n)
        exp = z[f"syn_{i}_expected"]
        assert np.array_equal(got.view(np.uint32), exp.view(np.uint32)), t["name"]
    for i, name in enumerate(meta["fixture"]["picked"]):
        e = next(x for x in meta["fixture"]["listing"] if x["name"] == name)
        got = oracle.gguf_dequant(bytes(z[f"fixture_{i}_raw"]), e["type"], int(np.prod(e["dims"])))
        assert np.array_equal(got.view(np.uint32), z[f"fixture_{i}_expected"].view(np.uint32)), name


def test_q4k_readings_differ_only_where_the_bytes_differ(gold, oracle_lib, tmp_path):
    """gguf.mojo reads Q4_K sub-blocks 4..7 from other scale bytes than the GGUF layout:
    the fixture (all scale bytes equal) decodes the same both ways, random bytes do not."""
    import oracle
    z, meta = gold
    i = meta["fixture"]["picked"].index("blk.0.linear_attn.k.weight")
    raw = bytes(z[f"fixture_{i}_raw"])
    n = raw.__len__() // 144 * 256
    assert np.array_equal(oracle.gguf_dequant(raw, 12, n, q4k_mojo=True), oracle.gguf_dequant(raw, 12, n))
    data, tensors = _syn_cases(z, meta)
    idx = parse_gguf_index(_write(tmp_path, "syn.gguf", data))
    raw = idx.read_raw("q4k.a")
    a, b = oracle.gguf_dequant(raw, 12, 768, q4k_mojo=True), oracle.gguf_dequant(raw, 12, 768)
    blk = np.arange(768) % 256
    assert np.array_equal(a[blk < 128], b[blk < 128]) and not np.array_equal(a[blk >= 128], b[blk >= 128])


# ---------------------------------------------------------------- CPU: native index parsers
def test_gguf_index_synthetic(gold, tmp_path):
    z, meta = gold
    data, tensors = _syn_cases(z, meta)
    idx = parse_gguf_index(_write(tmp_path, "syn.gguf", data))
    assert idx.version == 3 and idx.alignment == 64 and idx.tensor_count == len(tensors)
    assert idx.expected_file_size == len(data) and idx.data_section_offset % 64 == 0
    for t, info in zip(tensors, idx.tensors):
        assert info.name == t["name"] and info.dtype == t["type"]
        assert info.dims == list(reversed(t["shape"])) and info.num_elements == int(np.prod(t["shape"]))
        bs, bpb = fu.BLOCK[t["type"]]
        assert info.raw_bytes == info.num_elements // bs * bpb and info.offset % 64 == 0
    # metadata strings as the reference's index.metadata holds them
    md = idx.metadata
    assert md["general.architecture"] == "qwen3.6" and md["general.alignment"] == "64"
    assert md["t.u8"] == "200" and md["t.i8"] == str(256 - 3) and md["t.u16"] == "65000"
    assert md["t.i16"] == str(65536 - 2) and md["t.u32"] == "4000000000" and md["t.i32"] == str(2 ** 32 - 7)
    assert md["t.f32"] == str(struct.unpack("<I", struct.pack("<f", 1.5))[0]) and md["t.bool"] == "1"
    assert md["t.u64"] == str(2 ** 40) and md["t.f64"] == str(struct.unpack("<Q", struct.pack("<d", 0.25))[0])
    assert md["t.arr_u32"] == "[Array of 3 elements]" and md["t.arr_nested"] == "[Array of 2 elements]"
    assert md["t.i64"] == "5"  # (a negative i64 has its top bit set: the reference reader refuses it)


def test_gguf_index_reference_fixture(gold, tmp_path):
    """The fixture's own header (its tensor data zero-filled to the file's size) parses to
    the fixture's directory."""
    z, meta = gold
    fx = meta["fixture"]
    hdr = bytes(z["fixture_header"])
    p = _write(tmp_path, "fx.gguf", hdr + b"\x00" * (fx["file_size"] - len(hdr)))
    idx = parse_gguf_index(p)
    assert idx.tensor_count == len(fx["listing"]) and idx.data_section_offset == fx["data_start"]
    assert list(idx.metadata.keys()) == fx["meta_keys"]
    assert idx.metadata["qwen3.6.vocab_size"] == "1024"
    for e, info in zip(fx["listing"], idx.tensors):
        assert (info.name, info.dims, info.dtype, info.offset) == (e["name"], e["dims"], e["type"], e["offset"])


def _gguf_err(tmp_path, data: bytes) -> str:
    with pytest.raises(FormatError) as ei:
        parse_gguf_index(_write(tmp_path, "bad.gguf", data))
    assert ei.value.code == _lib.DM_ERR_FORMAT
    return json.loads(ei.value.message)["detail"]


def test_gguf_index_rejects(tmp_path):
    t = [("w", [64], 8, bytes(68))]
    good = fu.write_gguf([("a", 4, 1)], t)
    assert parse_gguf_index(_write(tmp_path, "g.gguf", good)).tensor_count == 1
    assert "too small for header" in _gguf_err(tmp_path, good[:20])
    assert "invalid magic header" in _gguf_err(tmp_path, b"GGUX" + good[4:])
    assert "unsupported version 4" in _gguf_err(tmp_path, good[:4] + struct.pack("<I", 4) + good[8:])
    assert "tensor_count out of bounds" in _gguf_err(tmp_path, good[:8] + struct.pack("<Q", 100001) + good[16:])
    assert "(diff: 1 bytes)" in _gguf_err(tmp_path, good + b"\x00")  # the exact-size check
    assert "tensor extends beyond file boundary" in _gguf_err(tmp_path, good[:-1])
    assert "tensor ndim invalid: 0" in _gguf_err(tmp_path, fu.write_gguf([], [("w", [], 8, b"")]))
    assert "tensor ndim invalid: 9" in _gguf_err(tmp_path, fu.write_gguf([], [("w", [1] * 9, 0, bytes(4))]))
    one_kv = b"GGUF" + struct.pack("<IQQ", 3, 0, 1)
    assert "unknown value type 13" in _gguf_err(tmp_path, one_kv + fu._gstr("a") + struct.pack("<I", 13) + bytes(16))
    assert "string length invalid" in _gguf_err(tmp_path, one_kv + struct.pack("<Q", 70000) + bytes(16))
    neg = good[:8] + b"\x01\x00\x00\x00\x00\x00\x00\x80" + good[16:]
    assert "u64 overflow/negative value" in _gguf_err(tmp_path, neg)
    with pytest.raises(FormatError) as ei:
        parse_gguf_index(str(tmp_path / "missing.gguf"))
    assert ei.value.code == _lib.DM_ERR_IO


def test_quant_file_scan_matches_reference_reader(gold, tmp_path):
    z, meta = gold
    q = meta["quant"]
    idx = scan_quant_file(_write(tmp_path, "q.bin", bytes(z["quant_bytes"])))
    assert idx.header["version"] == 1 and idx.header["model"] == q["model"]
    assert idx.header["total_bytes"] == q["total_bytes"] and idx.header["num_tensors"] == len(q["tensors"])
    for e, t in zip(idx.entries, q["tensors"]):
        assert (e.name, e.shape, e.group_size, e.num_groups) == (t["name"], t["shape"], t["group_size"], t["num_groups"])
        assert (e.record_offset, e.scales_offset, e.data_offset) == (t["record_offset"], t["scales_offset"],
                                                                     t["data_offset"])
        assert e.data_offset + e.weights_bytes == t["end"]
    raw = bytes(z["quant_bytes"])
    e = idx.entries[1]
    assert idx.read_scales(e.name).tobytes() == raw[e.scales_offset:e.scales_offset + e.scales_bytes]
    assert idx.read_packed(e.name).tobytes() == raw[e.data_offset:e.data_offset + e.weights_bytes]


def _quant_err(tmp_path, data: bytes) -> str:
    with pytest.raises(FormatError) as ei:
        scan_quant_file(_write(tmp_path, "bad.bin", data))
    assert ei.value.code == _lib.DM_ERR_FORMAT
    return json.loads(ei.value.message)["detail"]


def test_quant_file_rejects(tmp_path):
    rng = np.random.default_rng(3)
    s, p = fu.sym4_quantize(rng.standard_normal(256).astype(np.float32), 64)
    rec = fu.quant_record("w", [256], s, p, 64)

    def qf(hdr_kw=None, recs=None, total=None):
        recs = [rec] if recs is None else recs
        kw = dict(model="m", num_tensors=len(recs), total_bytes=256 + sum(map(len, recs)), group_size=64)
        kw.update(hdr_kw or {})
        return fu.quant_header(**kw) + b"".join(recs)

    assert scan_quant_file(_write(tmp_path, "ok.bin", qf())).entries[0].num_elements == 256
    assert "file truncated" in _quant_err(tmp_path, b"{}")
    assert "Invalid quant header version: expected 1, got 2" in _quant_err(tmp_path, qf({"version": 2}))
    assert "Group size must be one of {32, 64, 128, 256}, got 48" in _quant_err(tmp_path, qf({"group_size": 48}))
    bad_fmt = qf().replace(b"4-bit per-group", b"4-bit per-grouq")
    assert "Unsupported quantization format" in _quant_err(tmp_path, bad_fmt)
    assert "Unsupported scale dtype" in _quant_err(tmp_path, qf().replace(b'"FP16"', b'"BF16"', 1))
    assert "num_tensors must be positive" in _quant_err(tmp_path, qf({"num_tensors": 0}))
    assert "File size mismatch" in _quant_err(tmp_path, qf({"total_bytes": 999}))
    data = qf()
    assert "tensor payload truncated" in _quant_err(tmp_path, fu.quant_header("m", 1, len(data) - 1) + data[256:-1])
    two = fu.quant_header("m", 2, len(data)) + data[256:]
    assert "framing truncated before meta_len at tensor 1" in _quant_err(tmp_path, two)
    zero = fu.quant_header("m", 1, 260) + b"\x00\x00\x00\x00"
    assert "invalid meta_len (0)" in _quant_err(tmp_path, zero)
    assert "trailing data or size mismatch" in _quant_err(tmp_path, fu.quant_header("m", 1, len(data) + 3) +
                                                          data[256:] + b"abc")
    mism = rec.replace(b'"num_groups":4', b'"num_groups":5')
    assert "num_groups mismatch: meta=5, expected=4" in _quant_err(tmp_path, qf(recs=[mism]))
    noname = rec.replace(b'"name":"w"', b'"name":"" ')
    assert "Tensor name cannot be empty" in _quant_err(tmp_path, qf(recs=[noname]))
    tail = fu.quant_record("w", [96], s[:1], p[:48], 64)
    assert "N % G != 0" in _quant_err(tmp_path, qf(recs=[tail]))


# ---------------------------------------------------------------- CPU: pool conversions
def test_oracle_sym4_to_pool_is_exact(oracle_lib):
    import oracle
    rng = np.random.default_rng(9)
    rows, cols = 8, 256
    for gf in (32, 64, 128, 256):
        w = rng.standard_normal(rows * cols).astype(np.float32)
        s, p = fu.sym4_quantize(w, gf)
        if gf == 32:
            s = np.repeat(s[0::2], 2)  # equal scales inside each pool group: representable
        q, ps, pz, f = oracle.sym4_to_pool(p, s, 0, rows, cols, gf, 64)
        assert f == 0, gf
        pool = oracle.dequant_q4(q, ps, pz, rows, cols, 64)
        assert np.array_equal(pool.reshape(-1).view(np.uint32), fu.sym4_values(s, p, gf).view(np.uint32)), gf
    s, p = fu.sym4_quantize(rng.standard_normal(rows * cols).astype(np.float32), 32)
    assert oracle.sym4_to_pool(p, s, 0, rows, cols, 32, 64)[3] & 4  # different scales: flagged
    p2 = p.copy()
    p2[5] = 0x8F
    assert oracle.sym4_to_pool(p2, s, 0, rows, cols, 32, 64)[3] & 1


def test_oracle_requant_rule(oracle_lib):
    import oracle
    rng = np.random.default_rng(10)
    w = (rng.standard_normal((16, 256)) * rng.uniform(0.01, 3.0, (16, 1))).astype(np.float32)
    w[3, :64] = 0.0
    w[4, 64:128] = 2.5
    q, s, z, f, err = oracle.requant_pool(w, 64)
    assert f == 0
    back = oracle.dequant_q4(q, s, z, 16, 256, 64)
    sf = s.view(np.float16).astype(np.float32)
    assert np.abs(back - w).max() == pytest.approx(err)
    assert np.all(np.abs(back - w).reshape(16, 4, 64).max(axis=2) <= sf * 0.5 * (1 + 1e-6) + 1e-30)
    assert np.all(back[3, :64] == 0.0)           # an all-zero group stays zero
    # the rule restated in numpy (fp16 scale, zero, rint) gives the same codes
    g = w.reshape(16, 4, 64)
    lo, hi = np.minimum(g.min(axis=2), 0), np.maximum(g.max(axis=2), 0)
    s_np = ((hi - lo) / np.float32(15)).astype(np.float32).astype(np.float16)
    s_np = np.where(s_np == 0, np.float16(1.0), s_np).astype(np.float32)
    z_np = np.clip(np.rint(-lo / s_np), 0, 15)
    q_np = np.clip(np.rint(g / s_np[..., None]) + z_np[..., None], 0, 15).astype(np.uint8).reshape(16, 256)
    assert np.array_equal(q, (q_np[:, 0::2] | (q_np[:, 1::2] << 4)))


# ---------------------------------------------------------------- GPU
@pytest.mark.gpu
def test_gguf_dequant_device_bit_exact(gold, lib, oracle_lib, tmp_path):
    import oracle
    from disk_streaming_moe_engine_b200 import Engine, RuntimeConfig, preset
    z, meta = gold
    data, tensors = _syn_cases(z, meta)
    idx = parse_gguf_index(_write(tmp_path, "syn.gguf", data))
    with Engine(preset("mini"), RuntimeConfig.for_context(32, max_seqs=1)) as eng:
        cases = [(idx.read_raw(t["name"]), t["type"], int(np.prod(t["shape"])), z[f"syn_{i}_expected"])
                 for i, t in enumerate(tensors)]
        for i, name in enumerate(meta["fixture"]["picked"]):
            e = next(x for x in meta["fixture"]["listing"] if x["name"] == name)
            cases.append((bytes(z[f"fixture_{i}_raw"]), e["type"], int(np.prod(e["dims"])), z[f"fixture_{i}_expected"]))
        for raw, t, n, exp in cases:
            f32, bf = eng.gguf_dequant(raw, t, n, want_bf16=True)
            assert np.array_equal(f32.view(np.uint32), exp.view(np.uint32)), t
            import torch
            want_bf = torch.from_numpy(exp.copy()).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
            assert np.array_equal(bf, want_bf), t
            if t == 12:
                m, _ = eng.gguf_dequant(raw, t, n, q4k_mojo=True)
                assert np.array_equal(m.view(np.uint32), oracle.gguf_dequant(raw, t, n, q4k_mojo=True).view(np.uint32))
        with pytest.raises(DmError):
            eng.gguf_dequant(bytes(100), 12, 200)  # not whole blocks
        with pytest.raises(DmError):
            eng.gguf_dequant(bytes(100), 14, 256)  # Q6_K: not a supported type


def _mini_quant_file(cfg, m, layers_fused, prefix_lm):
    """The synthetic mini model as a custom 4-bit file by checkpoint names, and the weights
    it decodes to (dense: bf16 of fp32(s) q; experts: the pool codes of s q)."""
    from disk_streaming_moe_engine_b200.engine import Engine as E_
    recs = []
    G = 64
    H, I, E = cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts
    dec = {"layers": {}}

    def dense(name, arr_bf16):
        vals = (arr_bf16.astype(np.uint32) << 16).view(np.float32)
        g = G if vals.size % G == 0 else 32
        s, p = fu.sym4_quantize(vals.reshape(-1), g)
        recs.append(fu.quant_record(name, list(vals.shape), s, p, g))
        v = fu.sym4_values(s, p, g).reshape(vals.shape)
        import torch
        return torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)

    def pref(l):
        return (f"model.language_model.layers.{l}." if prefix_lm else f"model.layers.{l}.")

    dec["embed"] = dense("model.language_model.embed_tokens.weight" if prefix_lm else "model.embed_tokens.weight",
                         m["embed"].reshape(cfg.vocab_size, H))
    dec["final_norm"] = dense("model.language_model.norm.weight" if prefix_lm else "model.norm.weight",
                              m["final_norm"])
    dec["lm_head"] = dense("lm_head.weight", m["lm_head"].reshape(cfg.vocab_size, H))
    for l, t in m["layers"].items():
        table = dict(E_._COMMON)
        table.update(E_._ATT if cfg.is_attention_layer(l) else E_._GDN)
        d = {}
        for key, tid in table.items():
            hf = {_lib.DM_T_INPUT_NORM: "input_layernorm.weight", _lib.DM_T_POST_NORM: "post_attention_layernorm.weight",
                  _lib.DM_T_ROUTER: "mlp.gate.weight", _lib.DM_T_SHARED_GATE: "mlp.shared_expert_gate.weight",
                  _lib.DM_T_GDN_QKV: "linear_attn.in_proj_qkv.weight", _lib.DM_T_GDN_Z: "linear_attn.in_proj_z.weight",
                  _lib.DM_T_GDN_A: "linear_attn.in_proj_a.weight", _lib.DM_T_GDN_B: "linear_attn.in_proj_b.weight",
                  _lib.DM_T_GDN_CONV: "linear_attn.conv1d.weight", _lib.DM_T_GDN_DT_BIAS: "linear_attn.dt_bias",
                  _lib.DM_T_GDN_A_LOG: "linear_attn.A_log", _lib.DM_T_GDN_NORM: "linear_attn.norm.weight",
                  _lib.DM_T_GDN_OUT: "linear_attn.out_proj.weight", _lib.DM_T_ATTN_Q: "self_attn.q_proj.weight",
                  _lib.DM_T_ATTN_K: "self_attn.k_proj.weight", _lib.DM_T_ATTN_V: "self_attn.v_proj.weight",
                  _lib.DM_T_ATTN_Q_NORM: "self_attn.q_norm.weight", _lib.DM_T_ATTN_K_NORM: "self_attn.k_norm.weight",
                  _lib.DM_T_ATTN_O: "self_attn.o_proj.weight"}[tid]
            if t[key].dtype == np.float32:  # dt_bias / A_log (nv = 4 here: below one group): uploaded directly
                d[key] = t[key]
                continue
            d[key] = dense(pref(l) + hf, t[key])
        # experts: signed codes from the model's pool weights
        def proj_vals(kind, idx):
            q, s, zz = t[kind + "q"][idx], t[kind + "s"][idx], t[kind + "z"][idx]
            import oracle
            rows, cols = q.shape[0], q.shape[1] * 2
            return oracle.dequant_q4(q, s, zz, rows, cols, G)
        pools = {k: [] for k in ("gq", "gs", "gz", "uq", "us", "uz", "dq", "ds", "dz")}
        gate_all, up_all, down_all = [], [], []
        for idx in range(E + 1):
            for kind in ("g", "u", "d"):
                v = proj_vals(kind, idx)
                s, p = fu.sym4_quantize(v.reshape(-1), 128)
                rows, cols = v.shape
                import oracle
                q2, s2, z2, f = oracle.sym4_to_pool(p, s, 0, rows, cols, 128, G)
                assert f == 0
                pools[kind + "q"].append(q2)
                pools[kind + "s"].append(s2)
                pools[kind + "z"].append(z2)
                if idx == E:
                    nm = {"g": "gate_proj", "u": "up_proj", "d": "down_proj"}[kind]
                    recs.append(fu.quant_record(pref(l) + f"mlp.shared_expert.{nm}.weight", [rows, cols], s, p, 128))
                elif l in layers_fused:
                    (gate_all if kind == "g" else up_all if kind == "u" else down_all).append((s, p))
                else:
                    nm = {"g": "gate_proj", "u": "up_proj", "d": "down_proj"}[kind]
                    recs.append(fu.quant_record(pref(l) + f"mlp.experts.{idx}.{nm}.weight", [rows, cols], s, p, 128))
        if l in layers_fused:
            s_gu = np.concatenate([np.concatenate([gs, us]) for (gs, _), (us, _) in zip(gate_all, up_all)])
            p_gu = np.concatenate([np.concatenate([gp, up]) for (_, gp), (_, up) in zip(gate_all, up_all)])
            recs.append(fu.quant_record(pref(l) + "mlp.experts.gate_up_proj", [E, 2 * I, H], s_gu, p_gu, 128))
            s_d = np.concatenate([s for s, _ in down_all])
            p_d = np.concatenate([p for _, p in down_all])
            recs.append(fu.quant_record(pref(l) + "mlp.experts.down_proj", [E, H, I], s_d, p_d, 128))
        for k, v in pools.items():
            d[k] = np.stack(v)
        dec["layers"][l] = d
    return fu.quant_file("mini", recs, 64), dec


@pytest.mark.gpu
def test_quant_file_full_model_matches_oracle(lib, oracle_lib, tmp_path):
    """A whole config-0 model from a custom 4-bit file (fused experts in two layers,
    per-expert tensors in the others; both name prefixes) loads exactly: every dense weight
    equals dequant_kernel_simd's bf16 of the file, every expert projection the exact pool
    conversion; then greedy decoding matches the CPU oracle on those weights."""
    import oracle
    from disk_streaming_moe_engine_b200 import Engine, RuntimeConfig, preset, synth
    cfg = preset("mini")
    m = synth.synth_model(cfg, 0)
    for prefix_lm, fused in ((True, {0, 1}), (False, {2})):
        data, dec = _mini_quant_file(cfg, m, fused, prefix_lm)
        path = _write(tmp_path, "mini.q4", data)
        with Engine(cfg, RuntimeConfig.for_context(64, max_seqs=1)) as eng:
            with pytest.raises(DmError) as ei:   # dt_bias / A_log are not in the file
                eng.load_quant_file(path)
            assert ei.value.code == _lib.DM_ERR_NOT_READY and "linear_attn.dt_bias" in ei.value.message
            for l, t in m["layers"].items():
                if not cfg.is_attention_layer(l):
                    eng.upload_tensor(l, _lib.DM_T_GDN_DT_BIAS, t["dt_bias"])
                    eng.upload_tensor(l, _lib.DM_T_GDN_A_LOG, t["a_log"])
            eng.load_quant_file(path)
            eng.weights_check()
            for l, d in dec["layers"].items():
                table = dict(Engine._COMMON)
                table.update(Engine._ATT if cfg.is_attention_layer(l) else Engine._GDN)
                for key, tid in table.items():
                    got = eng.tensor_download(l, tid, d[key].size)
                    assert np.array_equal(got.reshape(-1).view(np.uint32 if got.dtype == np.float32 else np.uint16),
                                          d[key].reshape(-1).view(np.uint32 if got.dtype == np.float32 else np.uint16)), (l, key)
                for e in (0, 5, cfg.num_experts - 1, -1):
                    idx = e if e >= 0 else cfg.num_experts
                    for proj, kind in ((_lib.DM_PROJ_GATE, "g"), (_lib.DM_PROJ_UP, "u"), (_lib.DM_PROJ_DOWN, "d")):
                        q, s, zz = eng.expert_download(l, e, proj)
                        assert np.array_equal(q, d[kind + "q"][idx]) and np.array_equal(s, d[kind + "s"][idx])
                        assert np.array_equal(zz, d[kind + "z"][idx]), (l, e, kind)
            om = oracle.OracleModel({"cfg": m["cfg"], "layers": dec["layers"], "embed": dec["embed"].reshape(-1),
                                     "final_norm": dec["final_norm"], "lm_head": dec["lm_head"].reshape(-1)})
            st = oracle.OracleState(cfg, 64)
            eng.seq_reset(0)
            toks = np.random.default_rng(1).integers(0, cfg.vocab_size, 6)
            tok = None
            for t in toks:
                tok_o, lg_o, _ = oracle.decode_step(om, st, int(t))
                tok, lg = eng.decode_step(int(t), slot=0, want_logits=True)
                assert tok == tok_o
                assert np.abs(lg - lg_o).max() / np.abs(lg_o).max() < 1e-3


@pytest.mark.gpu
def test_gguf_experts_requantised_like_oracle(lib, oracle_lib, tmp_path):
    """GGUF expert tensors (Q4_K, Q8_0, Q3_K; a stacked 3-D tensor) load into the pool only
    with re-quantisation; the device's codes equal the oracle's rule applied to the
    oracle's dequantisation; dense GGUF tensors land as the bf16 of their fp32 values."""
    import oracle
    import torch
    from disk_streaming_moe_engine_b200 import Engine, RuntimeConfig, preset
    cfg = preset("mini")
    H, I, E = cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts
    rng = np.random.default_rng(5)
    stacked = fu.random_blocks(12, E * I * H, rng)
    down = fu.random_blocks(11, H * I, rng)
    up = fu.random_blocks(8, I * H, rng)
    norm = fu.random_blocks(0, H, rng)
    router = fu.random_blocks(8, E * H, rng)
    data = fu.write_gguf([("general.architecture", 8, "qwen3.6")],
                         [("blk.0.ffn_gate_exps.weight", [H, I, E], 12, stacked), ("d", [I, H], 11, down),
                          ("u", [H, I], 8, up), ("n", [H], 0, norm), ("r", [H, E], 8, router)])
    idx = parse_gguf_index(_write(tmp_path, "e.gguf", data))
    with Engine(cfg, RuntimeConfig.for_context(32, max_seqs=1)) as eng:
        with pytest.raises(DmError) as ei:
            eng.load_gguf_expert(idx, "u", 0, 3, _lib.DM_PROJ_UP)
        assert "DM_LOAD_REQUANT" in ei.value.message
        for name, slab, expert, proj, t, raw_all, n_all in (
                ("blk.0.ffn_gate_exps.weight", 7, 7, _lib.DM_PROJ_GATE, 12, stacked, E * I * H),
                ("u", 0, 3, _lib.DM_PROJ_UP, 8, up, I * H), ("d", 0, -1, _lib.DM_PROJ_DOWN, 11, down, H * I)):
            err = eng.load_gguf_expert(idx, name, 0, expert, proj, slab=slab, requant=True)
            vals = oracle.gguf_dequant(raw_all, t, n_all)
            rows, cols = (H, I) if proj == _lib.DM_PROJ_DOWN else (I, H)
            w = vals[slab * rows * cols:(slab + 1) * rows * cols].reshape(rows, cols)
            q, s, zz, f, err_o = oracle.requant_pool(w, 64)
            gq, gs, gz = eng.expert_download(0, expert, proj)
            assert np.array_equal(gq, q) and np.array_equal(gs, s) and np.array_equal(gz, zz), name
            assert err == err_o
        eng.load_gguf_tensor(idx, "n", 0, _lib.DM_T_INPUT_NORM)
        eng.load_gguf_tensor(idx, "r", 0, _lib.DM_T_ROUTER)
        for name, tid, t, raw, n in (("n", _lib.DM_T_INPUT_NORM, 0, norm, H), ("r", _lib.DM_T_ROUTER, 8, router, E * H)):
            want = torch.from_numpy(oracle.gguf_dequant(raw, t, n)).to(torch.bfloat16).view(torch.int16).numpy()
            assert np.array_equal(eng.tensor_download(0, tid, n), want.view(np.uint16)), name
        with pytest.raises(DmError):
            eng.load_gguf_tensor(idx, "n", 0, _lib.DM_T_ROUTER)  # wrong element count
        with pytest.raises(DmError):
            eng.load_gguf_tensor(idx, "absent", 0, _lib.DM_T_ROUTER)
