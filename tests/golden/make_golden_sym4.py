"""Golden vectors for the reference's custom 4-bit format (dequant_kernel_simd), made by the
reference's own Python oracle `tools/oracle/oracle_dequant.py:dequant_kernel_oracle` (and
its nibble unpacker `tools/quant/quant_format.py:unpack_4bit_pair`), imported from a
reference checkout.  Run once where the checkout exists:

    python tests/golden/make_golden_sym4.py /path/to/reference

Cases (all stored with their inputs, so the tests need no reference at run time):
  m10      the tensor of the reference fixture fixtures/m10_quant_mini.bin (64 x 64, G 64),
           parsed from the file's header / tensor record layout
  g<G>     seeded tensors for G in {32, 64, 128, 256}; scales are random finite positive
           fp16 bit patterns with the smallest subnormal (0x0001) and the largest finite
           value (0x7BFF = 65504) forced in; nibbles cover all 15 valid values [-7, 7]
  reject   inputs the reference rejects: reserved nibble 0b1000 (low and high position),
           NaN, +Inf, zero and negative scales
Outputs: tests/golden/reference_sym4.npz (+ .json with the per-case SHA-256 of the expected
bf16 bytes).
"""
import hashlib
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def parse_m10(path):
    d = open(path, "rb").read()
    header = json.loads(d[:256].rstrip(b" \x00").decode())
    n = struct.unpack_from("<I", d, 256)[0]
    meta = json.loads(d[260:260 + n].decode())
    base = 260 + n
    rows, cols = meta["shape"]
    ng = meta["num_groups"]
    scales = np.frombuffer(d, np.uint16, ng, base + meta["scale_offset"]).copy()
    packed = np.frombuffer(d, np.uint8, rows * cols // 2, base + meta["data_offset"]).copy()
    return header, meta, scales, packed


def seeded(group, groups, seed):
    rng = np.random.default_rng(seed)
    scales = rng.integers(0x0001, 0x7BFF + 1, groups).astype(np.uint16)
    scales[0] = 0x0001
    scales[min(1, groups - 1)] = 0x7BFF
    n = group * groups
    q = rng.integers(-7, 8, n)
    q[:15] = np.arange(-7, 8)
    u = (q & 0xF).astype(np.uint8)
    packed = (u[0::2] | (u[1::2] << 4)).astype(np.uint8)
    return scales, packed


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DISMOEN_REFERENCE", "")
    if not ref or not os.path.isdir(ref):
        raise SystemExit("usage: make_golden_sym4.py <reference checkout>")
    sys.path.insert(0, ref)
    from tools.oracle.oracle_dequant import dequant_kernel_oracle  # noqa: E402

    def oracle(scales, packed, group):
        raw = dequant_kernel_oracle(scales.tobytes(), packed.tobytes(), group)
        return np.frombuffer(raw, np.uint16).copy()

    out, meta_out = {}, {"generator": "tools/oracle/oracle_dequant.py:dequant_kernel_oracle", "cases": {}}
    header, meta, sc, pk = parse_m10(os.path.join(ref, "fixtures", "m10_quant_mini.bin"))
    g = meta["group_size"]
    exp = oracle(sc, pk, g)
    out.update(m10_scales=sc, m10_packed=pk, m10_expected_bf16=exp, m10_group=np.int32(g))
    meta_out["cases"]["m10"] = {"source": "fixtures/m10_quant_mini.bin", "tensor": meta["name"],
                                "shape": meta["shape"], "group": g, "model": header["model"],
                                "sha256_bf16": hashlib.sha256(exp.tobytes()).hexdigest()}
    for group, groups in ((32, 256), (64, 128), (128, 512), (256, 64)):
        sc, pk = seeded(group, groups, 42 + group)
        exp = oracle(sc, pk, group)
        k = f"g{group}"
        out.update({k + "_scales": sc, k + "_packed": pk, k + "_expected_bf16": exp})
        meta_out["cases"][k] = {"group": group, "groups": groups, "seed": 42 + group,
                                "sha256_bf16": hashlib.sha256(exp.tobytes()).hexdigest()}
    # rejection cases: (name, scales, packed, group); the reference oracle must raise
    rej = []
    sc, pk = seeded(32, 2, 7)
    bad_lo = pk.copy(); bad_lo[5] = (bad_lo[5] & 0xF0) | 0x8
    bad_hi = pk.copy(); bad_hi[9] = (bad_hi[9] & 0x0F) | 0x80
    for name, s_, p_ in (("nibble_lo_0x8", sc, bad_lo), ("nibble_hi_0x8", sc, bad_hi)):
        rej.append((name, s_, p_))
    for name, bits in (("scale_nan", 0x7E00), ("scale_inf", 0x7C00), ("scale_zero", 0x0000), ("scale_neg", 0xBC00)):
        s_ = sc.copy(); s_[1] = bits
        rej.append((name, s_, pk))
    meta_out["reject"] = []
    for i, (name, s_, p_) in enumerate(rej):
        try:
            oracle(s_, p_, 32)
            raise SystemExit(f"reference accepted reject case {name}")
        except ValueError as e:
            meta_out["reject"].append({"name": name, "reference_error": str(e)})
        out[f"rej{i}_scales"] = s_
        out[f"rej{i}_packed"] = p_
    np.savez_compressed(os.path.join(HERE, "reference_sym4.npz"), **out)
    with open(os.path.join(HERE, "reference_sym4.json"), "w") as f:
        json.dump(meta_out, f, indent=1)
    print(json.dumps(meta_out, indent=1))


if __name__ == "__main__":
    main()
