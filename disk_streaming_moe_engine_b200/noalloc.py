"""Python side of dm_moe_layer_noalloc: the MoE mixer of one layer over caller-owned
device buffers, with its scratch in the library's fixed 64 KiB device array (nothing is
allocated by the call).  `pack_expert_record` lays one expert out in the chunked 4-bit
record format the kernel reads (the format dm_expert_upload writes into a context)."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib

SCRATCH_BYTES = 65536


def scratch_bytes(H: int, I: int, topk: int) -> int:
    """Scratch a layer needs: control block, logits, top-k, x_norm [H], h [(k+1) I]."""
    return 512 + 4096 + 256 + 4 * H + 4 * (topk + 1) * I


def _chunks(q, s, z, cols, G):
    """q, s, z as [n chunks][16 rows][...] -> [n][chunk bytes]: nibbles, scales, zeros."""
    n = q.shape[0]
    ng = cols // G
    return np.concatenate([q.reshape(n, 16 * (cols // 2)),
                           s.reshape(n, 16 * ng).astype("<u2").view(np.uint8),
                           z.reshape(n, 16 * (ng // 2))], axis=1)


def pack_expert_record(gq, gs, gz, uq, us, uz, dq, ds, dz, H: int, I: int, G: int = 64) -> np.ndarray:
    """Canonical per-projection arrays (q [rows][cols/2] nibble pairs, s [rows][cols/G] fp16
    bits, z [rows][cols/G/2] zero pairs; gate/up [I][H], down [H][I]) -> record bytes.
    Gate/up chunk c holds gate rows 8c..8c+7 then up rows 8c..8c+7; the down projection
    follows in chunks of 16 output rows; each chunk is [nibbles][scales][zeros]."""
    assert G == 64
    n = I // 8

    def inter(g, u):  # [I][w] x2 -> [I/8][16][w] with gate rows first
        g = g.reshape(n, 8, -1)
        u = u.reshape(n, 8, -1)
        return np.concatenate([g, u], axis=1)

    gu = _chunks(inter(gq, uq), inter(gs, us), inter(gz, uz), H, G)
    nd = H // 16
    dn = _chunks(dq.reshape(nd, 16, -1), ds.reshape(nd, 16, -1), dz.reshape(nd, 16, -1), I, G)
    return np.concatenate([gu.ravel(), dn.ravel()])


def moe_layer_noalloc(H: int, I: int, E: int, topk: int, eps: float, router_ptr: int, post_norm_ptr: int,
                      experts_ptr: int, shared_ptr: int, x_mid_ptr: int, x_out_ptr: int,
                      ids_ptr: int = 0, probs_ptr: int = 0, stream: int = 0) -> None:
    """Calls dm_moe_layer_noalloc with raw device addresses; raises DmError on failure."""
    lib = _lib.load()
    buf = C.create_string_buffer(768)
    rc = lib.dm_moe_layer_noalloc(H, I, E, topk, eps, router_ptr, post_norm_ptr, experts_ptr, shared_ptr,
                                  x_mid_ptr, x_out_ptr, ids_ptr or None, probs_ptr or None, stream or None,
                                  buf, 768)
    if rc != _lib.DM_OK:
        raise _lib.DmError(rc, buf.value.decode())
