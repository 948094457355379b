"""Session files in the reference's KMSS v1 format (reference src/format/kmss.mojo).

CPU: the library's SHA-256 (the files' trailer) against hashlib.  GPU: the bytes the
library writes equal the restatement of write_kmss_v1 in oracle/kmss.py for the slot's
exported KV cache, GDN states and tokens (fp32 and bf16 KV); a file loads back into another
slot with identical KV, states and tokens; the reader's checks reject what
read_kmss_v1 rejects, with its error types (the reference unit test
tests/unit/test_m9_w2_kmss.mojo corrupts byte 130).
"""
import hashlib
import json
import os

import numpy as np
import pytest

from disk_streaming_moe_engine_b200 import DmError, Engine, RuntimeConfig, _lib, preset, synth


def test_sha256_matches_hashlib(lib):
    import ctypes as C
    rng = np.random.default_rng(0)
    for n in (0, 1, 55, 56, 63, 64, 65, 119, 120, 1000, 65537):
        data = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        buf = C.create_string_buffer(data, max(n, 1))
        out = C.create_string_buffer(32)
        assert lib.dm_sha256(buf, n, out) == 0
        assert out.raw == hashlib.sha256(data).digest(), n


def _state(eng, cfg, slot, n):
    k = np.stack([eng.kv_export(a, slot, n)[0] for a in range(cfg.num_attention_layers())], axis=1)
    v = np.stack([eng.kv_export(a, slot, n)[1] for a in range(cfg.num_attention_layers())], axis=1)
    S = np.stack([eng.gdn_state_export(g, slot)[0] for g in range(cfg.num_gdn_layers())])
    return k, v, S


def _bf16_to_f32(u16):
    return (u16.astype(np.uint32) << 16).view(np.float32)


@pytest.mark.gpu
def test_kmss_bytes_roundtrip_and_rejects(lib, tmp_path):
    import oracle.kmss as ok
    cfg = preset("mini")
    m = synth.synth_model(cfg, 0)
    with Engine(cfg, RuntimeConfig.for_context(128, max_seqs=2)) as eng:
        eng.load_model(m)
        eng.seq_reset(0)
        prompt = np.random.default_rng(4).integers(0, cfg.vocab_size, 21).astype(np.int32)
        eng.forward(prompt, slot=0, want_logits=False)
        n = eng.seq_len(0)
        k, v, S = _state(eng, cfg, 0, n)
        gdn = S.reshape(cfg.num_gdn_layers(), -1, cfg.linear_key_head_dim)  # [layers][nv dv][dk]
        mh = hashlib.sha256(b"manifest").digest()
        for kv_dtype in (1, 2):
            path = str(tmp_path / f"s{kv_dtype}.kmss")
            eng.save_session(path, prompt, slot=0, kv_dtype=kv_dtype, manifest_hash=mh)
            kk, vv = (_bf16_to_f32(k), _bf16_to_f32(v)) if kv_dtype == 1 else (k, v)
            want = ok.kmss_bytes(kk, vv, gdn, prompt, cfg.vocab_size, kv_dtype, mh)
            got = open(path, "rb").read()
            assert got == want, kv_dtype
            # load into the other slot: same KV, states and tokens
            toks = eng.load_session(path, slot=1)
            assert toks.tolist() == prompt.tolist()
            assert eng.seq_len(1) == n
            k1, v1, S1 = _state(eng, cfg, 1, n)
            assert np.array_equal(k1, k) and np.array_equal(v1, v)
            assert np.array_equal(S1.view(np.uint32), S.view(np.uint32))
            eng.decode_step(int(prompt[-1]), slot=1)  # the loaded slot decodes
            assert os.path.exists(path) and not os.path.exists(path + ".tmp")
        # the reader's checks, in read_kmss_v1's order
        good = open(str(tmp_path / "s1.kmss"), "rb").read()

        def expect(data: bytes, err_type: str):
            p = str(tmp_path / "bad.kmss")
            open(p, "wb").write(data)
            with pytest.raises(DmError) as ei:
                eng.load_session(p, slot=1)
            assert ei.value.code == _lib.DM_ERR_FORMAT
            assert json.loads(eng.last_error())["error_type"] == err_type

        corrupt = bytearray(good)
        corrupt[130] ^= 0xFF
        expect(bytes(corrupt), "CORRUPT_SESSION_CHECKSUM")
        expect(good[:100], "CORRUPT_SESSION_CHECKSUM")
        expect(b"XMSS" + good[4:], "FORMAT_MISMATCH")
        expect(good[:4] + (2).to_bytes(4, "little") + good[8:], "VERSION_MISMATCH")
        expect(good[:8] + (3).to_bytes(4, "little") + good[12:], "CONFIG_MISMATCH")
        expect(good[:-1], "LAYOUT_MISMATCH")
        with pytest.raises(DmError) as ei:
            eng.load_session(str(tmp_path / "missing.kmss"), slot=1)
        assert ei.value.code == _lib.DM_ERR_IO
