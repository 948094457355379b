"""The integer arithmetic of the small-segment batched experts, restated in numpy (CPU).

The batched kernels for segments of at most 8 rows (csrc/dm_expert_q4.cu, helpers in
csrc/dm_q4mma.cuh) multiply raw 4-bit weights q by activations carried as two signed 8-bit
digits per element with one unit per 32 elements (a half scale group):

    S = max |x| over the half,  u = 127 x / S,  d0 = rint(u),  d1 = rint(254 (u - d0)),
    x ~= unit (254 d0 + d1),    unit = S / (127 * 254),
    row += s * sum_halves unit_h ((C0_h - z D0_h) * 254 + (C1_h - z D1_h)),
    C_i = sum q d_i (integer MMA),  D_i = sum d_i.

These tests check the two facts the kernels rely on, on the same formulas: the zero point
enters exactly (C - z D = sum (q - z) d), and the encoding error of an element is at most
unit / 2 = S / 64516 (1.55e-5 of its half's largest magnitude), which bounds the row error by
s * sum |q - z| * unit / 2 per half.  The GPU tests compare the kernels themselves with the
oracle (tests/test_batch.py).
"""
import numpy as np

GROUP = 64
HALF = 32


def rint_even(v):
    """Round half to even, as the kernels' 1.5 * 2^23 addition does in fp32."""
    return np.rint(v)


def encode_half(x):
    """Digits (d0, d1) and the unit of one half group (32 values), fp32 as on the GPU."""
    x = x.astype(np.float32)
    S = np.float32(np.max(np.abs(x)))
    inv = np.float32(127.0) / S if (S > 0 and S <= 3.0e38) else np.float32(0.0)
    u = (x * inv).astype(np.float32)
    d0 = rint_even(u).astype(np.int32)
    d1 = rint_even(((u - d0.astype(np.float32)) * np.float32(254.0)).astype(np.float32)).astype(np.int32)
    unit = np.float32(S * np.float32(1.0 / (127.0 * 254.0)))
    return d0, d1, unit


def row_dot(q, z, s, x):
    """One weight row (K nibbles q, per-group zero z and scale s) times x, the kernels' way."""
    K = q.size
    acc = np.float64(0.0)
    for g in range(K // GROUP):
        part = 0.0
        for h in range(2):
            sl = slice(g * GROUP + h * HALF, g * GROUP + (h + 1) * HALF)
            d0, d1, unit = encode_half(x[sl])
            qq = q[sl].astype(np.int64)
            C0, C1 = int(qq @ d0), int(qq @ d1)
            D0, D1 = int(d0.sum()), int(d1.sum())
            T = (C0 - int(z[g]) * D0) * 254 + (C1 - int(z[g]) * D1)
            # the zero point enters exactly
            assert T == int(((qq - int(z[g])) * (254 * d0 + d1)).sum())
            assert abs(T) < 2 ** 24  # exact in fp32
            part += float(unit) * T
        acc += float(s[g]) * part
    return acc


def test_digit_encoding_error_within_half_unit():
    rng = np.random.default_rng(0)
    for scale in (1e-3, 1.0, 37.0, 6.0e4):
        x = (rng.standard_normal(HALF) * scale).astype(np.float32)
        d0, d1, unit = encode_half(x)
        assert np.all(np.abs(d0) <= 127) and np.all(np.abs(d1) <= 127)
        err = np.abs(unit * (254.0 * d0 + d1) - x.astype(np.float64))
        assert err.max() <= 0.5 * unit * (1 + 1e-5) + 1e-12 * scale
        assert abs(unit - np.abs(x).max() / (127.0 * 254.0)) <= 1e-6 * unit


def test_zero_half_gives_zero_digits():
    d0, d1, unit = encode_half(np.zeros(HALF, np.float32))
    assert not d0.any() and not d1.any() and unit == 0.0


def test_row_product_matches_float_within_bound():
    rng = np.random.default_rng(1)
    K = 512
    for trial in range(20):
        q = rng.integers(0, 16, K)
        z = rng.integers(0, 16, K // GROUP)
        s = np.abs(rng.standard_normal(K // GROUP) * 0.02).astype(np.float16).astype(np.float32)
        x = rng.standard_normal(K).astype(np.float32)
        if trial % 5 == 0:
            x[: HALF] *= 1e-4  # halves of very different magnitude keep their own units
        exact = float(sum(s[g] * ((q[g * GROUP:(g + 1) * GROUP] - z[g]) @ x[g * GROUP:(g + 1) * GROUP].astype(np.float64))
                          for g in range(K // GROUP)))
        bound = 0.0
        for g in range(K // GROUP):
            for h in range(2):
                sl = slice(g * GROUP + h * HALF, g * GROUP + (h + 1) * HALF)
                _, _, unit = encode_half(x[sl])
                bound += float(s[g]) * np.abs(q[sl] - z[g]).sum() * 0.5 * float(unit)
        got = row_dot(q, z, s, x)
        assert abs(got - exact) <= bound * (1 + 1e-4) + 1e-9
