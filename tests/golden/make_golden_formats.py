"""Golden vectors for the reference's on-disk weight formats, made by the reference's own
Python code imported from a reference checkout:

  GGUF dequantisation   tools/oracle/oracle_port.py:parse_gguf_tensors (its block
                        dequantisers dequantize_q8_0 / _q4_k / _q3_k, :68-159)
  custom 4-bit file     tools/quant/quant_format.py:make_quant_header / make_tensor_record
                        (writer) and parse_quant_header / read_tensor_record (reader)

Run once where the checkout exists:

    python tests/golden/make_golden_formats.py /path/to/reference

Cases (inputs stored with the outputs, so the tests need no reference at run time):
  syn        a GGUF v3 file written by tests/formats_util.write_gguf: alignment 64, every
             metadata value type (arrays, nested arrays), seeded tensors of F32, F16, BF16,
             Q8_0, Q4_K (random scale bytes: the sub-blocks 4..7 where gguf.mojo and the
             GGUF layout disagree) and Q3_K; expected fp32 of every tensor
  fixture    the reference fixture fixtures/m9_port_mini.gguf: its header bytes (up to the
             data section), size and tensor directory, and four of its tensors (Q8_0, Q4_K,
             Q3_K, F32) with their expected fp32
  quant      a three-tensor custom 4-bit file written by the reference writer (groups 64,
             128, 32; 2-D, 3-D, 1-D), with what the reference reader returns for it
Outputs: tests/golden/reference_formats.npz (+ .json).
"""
import hashlib
import json
import os
import struct
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import formats_util as fu  # noqa: E402

SYN_TENSORS = [("f32.a", (8, 4), 0), ("f16.a", (16, 4), 1), ("bf16.a", (64,), 30), ("q8.a", (64, 3), 8),
               ("q4k.a", (256, 3), 12), ("q4k.b", (512, 2), 12), ("q3k.a", (256, 2), 11), ("q3k.b", (768,), 11)]
SYN_META = [
    ("general.architecture", 8, "qwen3.6"),
    ("t.u8", 0, 200), ("t.i8", 1, -3), ("t.u16", 2, 65000), ("t.i16", 3, -2),
    ("t.u32", 4, 4000000000), ("t.i32", 5, -7), ("t.f32", 6, 1.5), ("t.bool", 7, 1),
    ("t.u64", 10, 2 ** 40), ("t.i64", 11, 5), ("t.f64", 12, 0.25),
    ("t.arr_u32", 9, (4, [1, 2, 3])), ("t.arr_str", 9, (8, ["a", "bc"])),
    ("t.arr_nested", 9, (9, [(0, [1, 2]), (0, [])])),
]
FIXTURE_PICK = ["blk.0.ffn_gate_exps.weight", "blk.0.linear_attn.k.weight", "blk.0.ffn_gate.0.weight",
                "blk.0.attn_norm.weight"]


def gguf_listing(data: bytes):
    """(tensor directory, metadata keys, data start) of a GGUF file (plain restatement)."""
    pos = 24
    tc, kc = struct.unpack_from("<QQ", data, 8)
    alignment = 32
    keys = []

    def skip(pos, vt):
        if vt in (0, 1, 7):
            return pos + 1
        if vt in (2, 3):
            return pos + 2
        if vt in (4, 5, 6):
            return pos + 4
        if vt in (10, 11, 12):
            return pos + 8
        if vt == 8:
            return pos + 8 + struct.unpack_from("<Q", data, pos)[0]
        et, n = struct.unpack_from("<IQ", data, pos)
        pos += 12
        for _ in range(n):
            pos = skip(pos, et)
        return pos

    for _ in range(kc):
        n = struct.unpack_from("<Q", data, pos)[0]
        k = data[pos + 8:pos + 8 + n].decode()
        pos += 8 + n
        vt = struct.unpack_from("<I", data, pos)[0]
        pos += 4
        if k == "general.alignment" and vt == 4:
            alignment = struct.unpack_from("<I", data, pos)[0]
        keys.append(k)
        pos = skip(pos, vt)
    out = []
    for _ in range(tc):
        n = struct.unpack_from("<Q", data, pos)[0]
        name = data[pos + 8:pos + 8 + n].decode()
        pos += 8 + n
        nd = struct.unpack_from("<I", data, pos)[0]
        pos += 4
        dims = list(struct.unpack_from(f"<{nd}Q", data, pos))
        pos += 8 * nd
        t, off = struct.unpack_from("<IQ", data, pos)
        pos += 12
        out.append({"name": name, "dims": dims, "type": t, "offset": off})
    return out, keys, (pos + alignment - 1) // alignment * alignment


def main(ref_root: str):
    sys.path.insert(0, os.path.join(ref_root, "tools", "oracle"))
    sys.path.insert(0, os.path.join(ref_root, "tools", "quant"))
    import oracle_port  # the reference's own GGUF reader and dequantisers
    import quant_format  # the reference's own custom-format writer and reader
    import tempfile

    arrays, meta = {}, {}

    # --- synthetic GGUF
    rng = np.random.default_rng(2026)
    tensors = []
    for name, shape, t in SYN_TENSORS:
        n = int(np.prod(shape))
        tensors.append((name, list(reversed(shape)), t, fu.random_blocks(t, n, rng)))
    syn = fu.write_gguf(SYN_META, tensors, alignment=64)
    with tempfile.NamedTemporaryFile(suffix=".gguf", delete=False) as f:
        f.write(syn)
        path = f.name
    ref = oracle_port.parse_gguf_tensors(path)
    os.unlink(path)
    arrays["syn_bytes"] = np.frombuffer(syn, np.uint8)
    for i, (name, shape, t) in enumerate(SYN_TENSORS):
        exp = ref[name].numpy().reshape(-1).astype(np.float32)
        arrays[f"syn_{i}_expected"] = exp
        assert exp.size == int(np.prod(shape))
    meta["syn"] = {"tensors": [{"name": n, "shape": list(s), "type": t} for n, s, t in SYN_TENSORS],
                   "alignment": 64, "sha256": hashlib.sha256(syn).hexdigest()}

    # --- the reference fixture
    fpath = os.path.join(ref_root, "fixtures", "m9_port_mini.gguf")
    data = open(fpath, "rb").read()
    listing, keys, data_start = gguf_listing(data)
    ref = oracle_port.parse_gguf_tensors(fpath)
    arrays["fixture_header"] = np.frombuffer(data[:data_start], np.uint8)
    meta["fixture"] = {"file_size": len(data), "data_start": data_start, "listing": listing, "meta_keys": keys,
                       "sha256": hashlib.sha256(data).hexdigest(), "picked": FIXTURE_PICK}
    by_name = {e["name"]: e for e in listing}
    for i, name in enumerate(FIXTURE_PICK):
        e = by_name[name]
        n = int(np.prod(e["dims"]))
        bs, bpb = fu.BLOCK[e["type"]]
        raw = data[data_start + e["offset"]:data_start + e["offset"] + n // bs * bpb]
        arrays[f"fixture_{i}_raw"] = np.frombuffer(raw, np.uint8)
        arrays[f"fixture_{i}_expected"] = ref[name].numpy().reshape(-1).astype(np.float32)

    # --- custom 4-bit quant file through the reference writer and reader
    qrng = np.random.default_rng(77)
    specs = [("model.layers.0.a.weight", [64, 128], 64), ("model.layers.0.b.weight", [2, 32, 128], 128),
             ("c.weight", [256], 32)]
    recs, qmeta = [], []
    for name, shape, g in specs:
        n = int(np.prod(shape))
        ng = n // g
        s_bits = qrng.integers(0x1000, 0x5000, ng).astype(np.uint16)
        scales = [float(v) for v in s_bits.view(np.float16)]
        weights = [int(v) for v in qrng.integers(-7, 8, n)]
        recs.append(quant_format.make_tensor_record(name, shape, scales, weights, dtype="BF16", group_size=g))
        # this repository's writer must produce the same bytes
        packed = np.array([(weights[i] & 0xF) | ((weights[i + 1] & 0xF) << 4) for i in range(0, n, 2)], np.uint8)
        assert fu.quant_record(name, shape, s_bits, packed, g) == recs[-1], name
    total = 256 + sum(len(r) for r in recs)
    hdr = quant_format.make_quant_header("golden-mini", len(recs), total, group_size=64)
    assert fu.quant_header("golden-mini", len(recs), total, 64) == hdr
    qbytes = hdr + b"".join(recs)
    quant_format.parse_quant_header(qbytes[:256])
    off = 256
    for name, shape, g in specs:
        m, sc, w, new = quant_format.read_tensor_record(qbytes, off)
        meta_len = struct.unpack_from("<I", qbytes, off)[0]
        payload = off + 4 + meta_len
        qmeta.append({"name": m["name"], "shape": m["shape"], "group_size": m["group_size"],
                      "num_groups": m["num_groups"], "record_offset": off, "scales_offset": payload + m["scale_offset"],
                      "data_offset": payload + m["data_offset"], "end": new})
        off = new
    assert off == len(qbytes)
    arrays["quant_bytes"] = np.frombuffer(qbytes, np.uint8)
    meta["quant"] = {"tensors": qmeta, "total_bytes": total, "model": "golden-mini"}

    np.savez_compressed(os.path.join(HERE, "reference_formats.npz"), **arrays)
    with open(os.path.join(HERE, "reference_formats.json"), "w") as f:
        json.dump(meta, f, indent=1)
    print("wrote", sum(a.nbytes for a in arrays.values()), "bytes of arrays")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden_formats.py <reference checkout>")
    main(sys.argv[1])
