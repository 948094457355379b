"""The reference's custom 4-bit format (dequant_kernel_simd, reference
src/quant/dequant_kernel.mojo:22-121): the CPU oracle and the device kernel against golden
vectors made by the reference's own Python oracle (tests/golden/make_golden_sym4.py):
the tensor of the reference fixture fixtures/m10_quant_mini.bin and seeded tensors for every
allowed group size, bit-exact in bf16; plus the reference's rejections."""
import json
import os

import numpy as np
import pytest

from disk_streaming_moe_engine_b200 import DmError, Engine, RuntimeConfig, _lib, preset

GOLD = os.path.join(os.path.dirname(__file__), "golden")
CASES = ["m10", "g32", "g64", "g128", "g256"]


@pytest.fixture(scope="module")
def gold():
    z = np.load(os.path.join(GOLD, "reference_sym4.npz"))
    meta = json.load(open(os.path.join(GOLD, "reference_sym4.json")))
    return z, meta


def _case(z, k):
    g = int(z["m10_group"]) if k == "m10" else int(k[1:])
    return z[k + "_scales"], z[k + "_packed"], z[k + "_expected_bf16"], g


def _f32_ref(scales, packed, group):
    """fp32(s_g) * q from first principles (numpy), for the fp32 output."""
    lo = (packed & 0xF).astype(np.int8)
    hi = (packed >> 4).astype(np.int8)
    q = np.empty(packed.size * 2, np.int8)
    q[0::2], q[1::2] = lo, hi
    q = np.where(q >= 8, q - 16, q).astype(np.float32)
    s = scales.view(np.float16).astype(np.float32)
    return np.repeat(s, group) * q


@pytest.mark.parametrize("k", CASES)
def test_oracle_matches_reference_bf16(gold, oracle_lib, k):
    import oracle
    z, _ = gold
    sc, pk, exp, g = _case(z, k)
    ob, of, rc = oracle.dequant_sym4(pk, sc, exp.size, g)
    assert rc == 0
    assert np.array_equal(ob, exp)
    assert np.array_equal(of.view(np.uint32), _f32_ref(sc, pk, g).view(np.uint32))


def test_oracle_rejects_like_reference(gold, oracle_lib):
    import oracle
    z, meta = gold
    for i, r in enumerate(meta["reject"]):
        sc, pk = z[f"rej{i}_scales"], z[f"rej{i}_packed"]
        _, _, rc = oracle.dequant_sym4(pk, sc, pk.size * 2, 32)
        assert rc == (-1 if r["name"].startswith("nibble") else -2), r


@pytest.fixture(scope="module")
def eng(lib):
    e = Engine(preset("mini"), RuntimeConfig.for_context(64))
    yield e
    e.close()


@pytest.mark.gpu
@pytest.mark.parametrize("k", CASES)
def test_device_matches_reference_bf16(gold, eng, k):
    z, _ = gold
    sc, pk, exp, g = _case(z, k)
    ob, of = eng.dequant_sym4(pk, sc, exp.size, g)
    assert np.array_equal(ob, exp)
    assert np.array_equal(of.view(np.uint32), _f32_ref(sc, pk, g).view(np.uint32))
    ob2, none = eng.dequant_sym4(pk, sc, exp.size, g, want_f32=False)
    assert none is None and np.array_equal(ob2, exp)


@pytest.mark.gpu
def test_device_rejects_like_reference(gold, eng):
    z, meta = gold
    for i, r in enumerate(meta["reject"]):
        sc, pk = z[f"rej{i}_scales"], z[f"rej{i}_packed"]
        with pytest.raises(DmError) as e:
            eng.dequant_sym4(pk, sc, pk.size * 2, 32)
        assert e.value.code == _lib.DM_ERR_INVALID_ARG
        want = "reserved nibble" if r["name"].startswith("nibble") else (
            "NaN or Inf" if r["name"] in ("scale_nan", "scale_inf") else "non-positive")
        assert want in e.value.message, (r, e.value.message)
    sc, pk, exp, g = _case(z, "g64")
    for bad_group in (16, 48, 512):
        with pytest.raises(DmError):
            eng.dequant_sym4(pk, sc, exp.size, bad_group)
    with pytest.raises(DmError) as e:  # N % G != 0
        eng.dequant_sym4(pk[:24], sc[:1], 48, 32)
    assert "N % G" in e.value.message
