"""Test infrastructure (never on the product path): a restatement of the reference's session
writer, KMSS v1 (reference src/format/kmss.mojo), used to pin the bytes the library writes.

Layout (kmss.mojo:6-27, write_kmss_v1 :90-170): 128-byte header — magic "KMSS", version 1,
architecture 2, 32-byte manifest hash, seq_len, vocab_size, kv_layers, kv_heads, head_dim,
kv_dtype (1 fp32, 2 bf16), gdn_layers, gdn_dv, gdn_dk, gdn_dtype 1 (u32 LE each), kv_bytes,
gdn_bytes, token_bytes (u64 LE), 20 zero bytes; payload: KV in the order kv index,
position, attention layer, head, dim (:172-199), GDN states as stored (:201-207), token ids
u32 LE zero-padded to seq_len (:209-215); trailer: SHA-256 of header || payload (:226-240).
"""
from __future__ import annotations

import hashlib
import struct

import numpy as np


def kmss_bytes(k: np.ndarray, v: np.ndarray, gdn: np.ndarray, tokens, vocab_size: int, kv_dtype: int = 1,
               manifest_hash: bytes = b"") -> bytes:
    """k, v: [seq, kv_layers, kv_heads, head_dim] float32 values (bf16 bit patterns as uint16
    for kv_dtype 2); gdn: [gdn_layers, gdn_dv, gdn_dk] float32; tokens: ids (<= seq)."""
    seq, kv_layers, kv_heads, head_dim = k.shape
    gdn_layers, gdn_dv, gdn_dk = gdn.shape
    b_kv = 4 if kv_dtype == 1 else 2
    kv_bytes = 2 * seq * kv_layers * kv_heads * head_dim * b_kv
    gdn_bytes = gdn_layers * gdn_dv * gdn_dk * 4
    token_bytes = seq * 4
    mh = (bytes(manifest_hash) + bytes(32))[:32]
    hdr = b"KMSS" + struct.pack("<II", 1, 2) + mh
    hdr += struct.pack("<10I", seq, vocab_size, kv_layers, kv_heads, head_dim, kv_dtype, gdn_layers, gdn_dv, gdn_dk, 1)
    hdr += struct.pack("<3Q", kv_bytes, gdn_bytes, token_bytes)
    hdr += bytes(128 - len(hdr))
    assert len(hdr) == 128
    dt = np.float32 if kv_dtype == 1 else np.uint16
    kv = np.stack([k, v]).astype(dt).tobytes()
    tok = np.zeros(seq, np.uint32)
    tok[:len(tokens)] = np.asarray(tokens, np.uint32)
    body = hdr + kv + np.ascontiguousarray(gdn, np.float32).tobytes() + tok.tobytes()
    return body + hashlib.sha256(body).digest()
