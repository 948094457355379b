"""CPU tests of the C-ABI library: it loads without a GPU, exports every symbol declared
in include/dismoen_cuda.h, validates configs like reference ModelConfig, and its
synthetic generator is deterministic.  No device compute is called here."""
import ctypes as C
import json
import os
import re

import numpy as np
import pytest

from disk_streaming_moe_engine_b200 import _lib, preset

HEADER = os.path.join(os.path.dirname(os.path.dirname(__file__)), "include", "dismoen_cuda.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*int32_t\s+(dm_\w+)\s*\(", src, flags=re.M)))


def test_every_declared_symbol_is_exported(lib):
    syms = declared_symbols()
    assert len(syms) >= 30
    for s in syms:
        assert hasattr(lib, s), s
        assert s in _lib.SIGNATURES, f"{s} missing from the ctypes binding"


def test_abi_version(lib):
    assert lib.dm_abi_version() == 2


def _validate(lib, cfg):
    buf = C.create_string_buffer(512)
    rc = lib.dm_config_validate(C.byref(cfg.to_c()), buf, 512)
    return rc, buf.value.decode()


@pytest.mark.parametrize("name", ["mini", "layer", "full"])
def test_presets_validate(lib, name):
    rc, msg = _validate(lib, preset(name))
    assert rc == 0, msg


def test_config_errors_use_reference_json_shape(lib):
    cfg = preset("mini")
    cfg.num_experts_per_tok = 17
    rc, msg = _validate(lib, cfg)
    assert rc == _lib.DM_ERR_INVALID_ARG
    err = json.loads(msg)
    assert set(err) == {"error_type", "detail", "stage", "layer"}
    assert err["error_type"] == "CONFIG_ERROR"
    cfg = preset("mini")
    cfg.norm_topk_prob = True
    rc, msg = _validate(lib, cfg)
    assert rc != 0 and json.loads(msg)["error_type"] == "ROUTER_ERROR"
    cfg = preset("mini")
    cfg.rms_norm_eps = 0.0
    assert _validate(lib, cfg)[0] != 0
    cfg = preset("mini")
    cfg.num_key_value_heads = 3
    assert _validate(lib, cfg)[0] != 0


def test_synth_is_counter_based(lib):
    a = np.empty(1000, np.uint16)
    b = np.empty(400, np.uint16)
    lib.dm_synth_bf16(5, 77, a.size, 0.0, 1.0, a.ctypes.data)
    lib.dm_synth_bf16(5, 77, b.size, 0.0, 1.0, b.ctypes.data)
    assert np.array_equal(a[:400], b)
    f = (a.astype(np.uint32) << 16).view(np.float32)
    assert abs(f.mean()) < 0.15 and 0.85 < f.std() < 1.15
    u = np.empty(1 << 16, np.uint8)
    lib.dm_synth_u8(5, 78, u.size, u.ctypes.data)
    counts = np.bincount(u & 15, minlength=16)
    assert counts.min() > 0.8 * counts.mean()
    s = np.empty(4096, np.uint16)
    lib.dm_synth_f16_absnormal(5, 79, s.size, 0.02, s.ctypes.data)
    sf = s.view(np.float16).astype(np.float32)
    assert (sf >= 0).all() and 0.012 < sf.mean() < 0.02


def test_expert_bytes_match_baseline_figure():
    # 4.3125 bits/weight: 1,695,744 B per full-shape expert (gate + up + down)
    assert preset("full").expert_bytes() == 1695744


def test_plain_c_host_links_and_calls(tmp_path, lib):
    """The library as a plain C host links it (gcc, the header only): config validation,
    SHA-256, the GGUF and quant-file parsers and the spill policy answer without a device."""
    import hashlib
    import json as _json
    import shutil
    import subprocess

    import numpy as np

    import formats_util as fu
    from disk_streaming_moe_engine_b200 import _lib as L
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = str(tmp_path / "harness")
    libdir = os.path.dirname(L.LIB_PATH)
    subprocess.run([gcc, "-O1", "-std=c11", "-I", os.path.join(repo, "include"),
                    os.path.join(repo, "tests", "c_abi", "harness.c"), "-o", exe, "-L", libdir, "-ldismoen_cuda",
                    f"-Wl,-rpath,{libdir}", "-Wl,-rpath,/usr/local/cuda/lib64"], check=True)
    gg = tmp_path / "m.gguf"
    gg.write_bytes(fu.write_gguf([("general.architecture", 8, "qwen3.6")],
                                 [("tok", [32, 4], 8, fu.random_blocks(8, 128, np.random.default_rng(0)))]))
    s, p = fu.sym4_quantize(np.linspace(-1, 1, 128, dtype=np.float32), 64)
    qf = tmp_path / "m.q4"
    qf.write_bytes(fu.quant_file("m", [fu.quant_record("w", [2, 64], s, p, 64)]))
    out = subprocess.run([exe, str(gg), str(qf)], check=True, capture_output=True, text=True).stdout
    r = _json.loads(out)
    assert r["abi"] == 2 and r["cfg_ok"] == 0 and r["cfg_bad"] != 0
    assert r["sha_abc"] == hashlib.sha256(b"abc").hexdigest()
    assert r["gguf"][:3] == [0, 3, 1] and r["gguf"][5:] == ["tok", 8]
    assert r["quant"] == [0, 1, 64, 1]
    # 4 slots: step 1 {0,1,2,3} misses 4; step 2 {2,3,4,5} hits 2, misses 2, evicts 0 and 1
    assert r["spill"] == [0, 8, 2, 6, 2]


@pytest.mark.gpu
def test_c_host_drives_the_decode_path(lib, oracle_lib, tmp_path):
    """tests/c_abi/decode.c: a plain C program creates a context, synthesises the config-0
    model on the device and runs dm_forward, dm_generate, dm_prefill and dm_decode_batch;
    its ids equal the oracle's on the host generator's weights (the device generator is the
    same), and a bad token comes back as an error status with the reference's error type."""
    import json as _json
    import shutil
    import subprocess

    import numpy as np

    import oracle
    from disk_streaming_moe_engine_b200 import _lib as L, preset, synth
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    exe = str(tmp_path / "decode")
    libdir = os.path.dirname(L.LIB_PATH)
    subprocess.run([gcc, "-O1", "-std=c11", "-I", os.path.join(repo, "include"),
                    os.path.join(repo, "tests", "c_abi", "decode.c"), "-o", exe, "-L", libdir, "-ldismoen_cuda",
                    f"-Wl,-rpath,{libdir}", "-Wl,-rpath,/usr/local/cuda/lib64"], check=True)
    cfg = preset("mini")
    prompt = [int(t) for t in np.random.default_rng(7).integers(0, cfg.vocab_size, 11)]
    out = subprocess.run([exe] + [str(t) for t in prompt], check=True, capture_output=True, text=True).stdout
    r = _json.loads(out)
    om = oracle.OracleModel(synth.synth_model(cfg, 0))
    st = oracle.OracleState(cfg, 64)
    tok = None
    for t in prompt:
        tok, _, _ = oracle.decode_step(om, st, t)
    assert r["next_forward"] == tok and r["next_prefill"] == tok
    gen = []
    for _ in range(8):
        tok, _, _ = oracle.decode_step(om, st, tok)
        gen.append(tok)
    assert r["generate"] == gen
    assert r["len"] == [len(prompt) + 8, len(prompt)]
    nxt, _, _ = oracle.decode_step(om, st, gen[7])
    assert r["batch"] == [nxt, gen[0]]
    assert r["bad_rc"] != 0 and "M4_ERR_INPUT" in r["bad_msg"]
