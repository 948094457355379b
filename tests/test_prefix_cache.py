"""The longest-prefix session cache (reference src/core/prefix_cache.mojo) and lossless
session resume.

CPU: the policy with host-object entries, case by case as the reference's unit test
tests/unit/test_m12_prefix_cache.mojo states it (longest exact prefix, mid-history
divergence, domain and session isolation, clean-completion-only insertion, bounded LRU
eviction, directory persistence with the manifest format).
GPU: entries held in engine slots (device copies of the whole sequence state): a cache hit
plus delta prefill gives bit-identical logits to the same operations without the cache;
entries persisted to a directory (KMSS v1 + conv-window sidecar) and loaded into another
cache decode the same; a session file with its sidecar resumes decoding exactly as the
uninterrupted sequence over 8 steps, and without the sidecar starts from a zero conv window.
"""
import json
import os

import numpy as np
import pytest

from disk_streaming_moe_engine_b200.prefix_cache import (HostStore, PrefixCache, compute_domain_key,
                                                          domain_key_to_bytes)

DOMAIN = compute_domain_key("qwen3.6", "pin_v1", "m12_v1")


def test_domain_key_is_sha256_hex():
    import hashlib
    assert DOMAIN == hashlib.sha256(b"qwen3.6:pin_v1:m12_v1").hexdigest()
    assert domain_key_to_bytes(DOMAIN) == hashlib.sha256(b"qwen3.6:pin_v1:m12_v1").digest()
    assert compute_domain_key("a", "b", "c") != compute_domain_key("a", "b", "d")
    assert domain_key_to_bytes("ab") == bytes([0xAB]) + bytes(31)


def test_exact_longest_prefix_match():
    c = PrefixCache(capacity=4)
    assert c.insert(DOMAIN, [1, 2, 3], "s3", "stop")
    assert c.insert(DOMAIN, [1, 2, 3, 4, 5], "s5", "stop")
    r = c.lookup(DOMAIN, [1, 2, 3, 4, 5, 6, 7])
    assert (r.hit, r.prefix_len, r.delta_tokens_len) == (True, 5, 2)
    assert c.restore(r, None) == "s5"
    r = c.lookup(DOMAIN, [1, 2, 3, 9, 9])
    assert (r.hit, r.prefix_len, r.delta_tokens_len) == (True, 3, 2)
    assert c.restore(r, None) == "s3"
    r = c.lookup(DOMAIN, [7, 8])
    assert (r.hit, r.prefix_len, r.delta_tokens_len) == (False, 0, 2)
    r = c.lookup(DOMAIN, [])
    assert (r.hit, r.prefix_len, r.delta_tokens_len) == (False, 0, 0)
    # an entry longer than the request is no prefix of it
    assert not c.lookup(DOMAIN, [1, 2]).hit


def test_mid_history_divergence():
    c = PrefixCache(capacity=4)
    assert c.insert(DOMAIN, [100, 101, 102], "t1", "stop")
    assert c.insert(DOMAIN, [100, 101, 102, 200, 201], "t2", "stop")
    r = c.lookup(DOMAIN, [100, 101, 102, 301, 302])  # turn 2 edited: reuse up to the divergence
    assert (r.hit, r.prefix_len, r.delta_tokens_len) == (True, 3, 2)


def test_domain_and_session_isolation():
    other = compute_domain_key("qwen3.6", "pin_v2", "m12_v1")
    c = PrefixCache(capacity=4)
    assert c.insert(DOMAIN, [5, 6, 7], "a", "stop")
    assert not c.lookup(other, [5, 6, 7]).hit
    c2 = PrefixCache(capacity=4)
    assert c2.insert(DOMAIN, [1, 2, 3, 4], "a", "stop")
    r = c2.lookup(DOMAIN, [1, 2, 3, 5])  # same length, one token differs
    assert (r.hit, r.prefix_len, r.delta_tokens_len) == (False, 0, 4)


def test_insertion_policy_clean_vs_abort():
    c = PrefixCache(capacity=4)
    for reason in ("abort", "error", "timeout"):
        assert not c.insert(DOMAIN, [1, 2], "x", reason)
        assert c.size() == 0
    assert not c.insert(DOMAIN, [], "x", "stop")
    assert c.insert(DOMAIN, [1, 2], "x", "stop") and c.size() == 1
    assert c.insert(DOMAIN, [1, 2, 3], "y", "length") and c.size() == 2
    # the same tokens again refresh the entry in place
    assert c.insert(DOMAIN, [1, 2], "x2", "stop") and c.size() == 2
    assert c.restore(c.lookup(DOMAIN, [1, 2]), None) == "x2"


def test_bounded_lru_eviction():
    c = PrefixCache(capacity=2)
    t1, t2, t3 = [1, 1, 1], [2, 2, 2], [3, 3, 3]
    assert c.insert(DOMAIN, t1, "1", "stop") and c.insert(DOMAIN, t2, "2", "stop")
    assert c.lookup(DOMAIN, t1).hit  # t1 becomes the most recently used
    assert c.insert(DOMAIN, t3, "3", "stop")
    assert c.size() == 2
    assert c.lookup(DOMAIN, t1).hit and c.lookup(DOMAIN, t3).hit
    assert not c.lookup(DOMAIN, t2).hit
    # entry ids follow the access clock
    assert [e.entry_id for e in c.entries] == ["entry_1", "entry_4"]


class _FileStore(HostStore):
    """Host entries persisted as JSON token lists (the engine store writes KMSS files)."""

    def save(self, i, path, tokens, manifest_hash):
        json.dump({"tokens": list(tokens), "state": self.states[i], "mh": manifest_hash.hex()}, open(path, "w"))

    def load(self, i, path):
        d = json.load(open(path))
        self.states[i] = d["state"]
        return d["tokens"]


def test_dir_persistence_roundtrip(tmp_path):
    c = PrefixCache(capacity=4, store=_FileStore(4))
    assert c.insert(DOMAIN, [1, 2, 3], "s1", "stop")
    assert c.insert(DOMAIN, [9, 8, 7, 6], "s2", "stop")
    c.save_to_dir(str(tmp_path))
    lines = open(tmp_path / "manifest.txt").read().splitlines()
    assert lines == [f"entry_1 1 {DOMAIN} entry_1.kmss", f"entry_2 2 {DOMAIN} entry_2.kmss"]
    assert json.load(open(tmp_path / "entry_1.kmss"))["mh"] == domain_key_to_bytes(DOMAIN).hex()
    # a malformed line and a missing file are skipped
    with open(tmp_path / "manifest.txt", "a") as f:
        f.write("broken\nentry_9 9 x missing.kmss\n")
    c2 = PrefixCache(capacity=4, store=_FileStore(4))
    c2.load_from_dir(str(tmp_path))
    assert c2.size() == 2 and c2.access_clock == 2
    r = c2.lookup(DOMAIN, [1, 2, 3, 4])
    assert (r.hit, r.prefix_len, r.delta_tokens_len) == (True, 3, 1)
    assert c2.restore(r, None) == "s1"
    c3 = PrefixCache(capacity=4, store=_FileStore(4))
    c3.load_from_dir(str(tmp_path / "nowhere"))  # no manifest: nothing loaded, no error
    assert c3.size() == 0


# ---------------------------------------------------------------------------------------
@pytest.mark.gpu
def test_cache_hit_delta_prefill_is_bit_identical(lib, tmp_path):
    """Turn 1 (prompt A + 5 greedy steps) inserted from slot 0; turn 2 (the history + the
    pending token + B) through the cache into slot 0 equals, bit for bit, the same prompt,
    steps and delta prefill run in slot 3 without any cache; also after the cache went to a
    directory and back into another cache."""
    from disk_streaming_moe_engine_b200 import Engine, RuntimeConfig, preset, synth
    from disk_streaming_moe_engine_b200.prefix_cache import EngineSlotStore, prefill_with_cache
    cfg = preset("mini")
    m = synth.synth_model(cfg, 0)
    rng = np.random.default_rng(12)
    a = rng.integers(0, cfg.vocab_size, 30).astype(np.int32)
    b = rng.integers(0, cfg.vocab_size, 12).astype(np.int32)
    with Engine(cfg, RuntimeConfig.for_context(96, max_seqs=8)) as eng:
        eng.load_model(m)
        for s in range(8):
            eng.seq_reset(s)
        cache = PrefixCache(capacity=4, store=EngineSlotStore(eng, [4, 5, 6, 7]))
        _, n0 = eng.prefill(a, slot=0, want_logits=False)
        g = eng.generate(n0, 5, slot=0)
        hist = np.concatenate([a, [n0], g[:4]]).astype(np.int32)  # the tokens slot 0 has consumed
        assert eng.seq_len(0) == len(hist)
        assert cache.insert(DOMAIN, hist, 0, "stop", next_token=int(g[4]))
        eng.seq_reset(0)  # the working slot is reused for something else meanwhile
        eng.prefill(b, slot=0, want_logits=False)
        req = np.concatenate([hist, [g[4]], b]).astype(np.int32)
        lg, nx, res = prefill_with_cache(eng, cache, DOMAIN, req, slot=0, want_logits=True)
        assert res.hit and res.prefix_len == len(hist) and res.delta_tokens_len == 13
        assert eng.seq_len(0) == len(req)
        # the same kernels on the same state without the cache
        _, n3 = eng.prefill(a, slot=3, want_logits=False)
        g3 = eng.generate(n3, 5, slot=3)
        assert n3 == n0 and list(g3) == list(g)
        lg3, nx3 = eng.prefill(np.concatenate([[g3[4]], b]).astype(np.int32), slot=3)
        assert nx3 == nx and np.array_equal(lg3, lg)
        # a request equal to the entry needs no prefill: the stored next token
        _, nx4, res4 = prefill_with_cache(eng, cache, DOMAIN, hist, slot=0)
        assert res4.hit and res4.delta_tokens_len == 0 and nx4 == int(g[4]) and eng.seq_len(0) == len(hist)
        # persisted (KMSS v1 + conv sidecar) and loaded into another cache on other slots
        cache.save_to_dir(str(tmp_path))
        assert os.path.exists(tmp_path / "entry_1.kmss") and os.path.exists(tmp_path / "entry_1.kmss.conv")
        c2 = PrefixCache(capacity=2, store=EngineSlotStore(eng, [6, 7]))
        c2.load_from_dir(str(tmp_path))
        assert c2.size() == 1
        lg5, nx5, res5 = prefill_with_cache(eng, c2, DOMAIN, req, slot=0, want_logits=True)
        assert res5.hit and nx5 == nx and np.array_equal(lg5, lg)


@pytest.mark.gpu
def test_session_resume_is_lossless_with_the_conv_sidecar(lib, tmp_path):
    from disk_streaming_moe_engine_b200 import DmError, Engine, RuntimeConfig, preset, synth
    cfg = preset("mini")
    m = synth.synth_model(cfg, 0)
    prompt = np.random.default_rng(21).integers(0, cfg.vocab_size, 21).astype(np.int32)
    path = str(tmp_path / "s.kmss")
    with Engine(cfg, RuntimeConfig.for_context(64, max_seqs=3)) as eng:
        eng.load_model(m)
        for s in range(3):
            eng.seq_reset(s)
        _, nxt = eng.forward(prompt, slot=0, want_logits=False)
        eng.save_session(path, prompt, slot=0, kv_dtype=1)
        toks = eng.load_session(path, slot=1)
        assert list(toks) == list(prompt)
        # 8 steps from the original and from the resumed slot: identical ids and logits
        t0 = t1 = nxt
        for _ in range(8):
            t0, lg0 = eng.decode_step(t0, slot=0, want_logits=True)
            t1, lg1 = eng.decode_step(t1, slot=1, want_logits=True)
            assert t0 == t1 and np.array_equal(lg0, lg1)
        # without the sidecar the window starts at zero (the reference's port semantics)
        os.rename(path + ".conv", path + ".conv.bak")
        eng.load_session(path, slot=2)
        for g in range(cfg.num_gdn_layers()):
            S1, c1 = eng.gdn_state_export(g, 2)
            assert not c1.any()
        # a sidecar bound to another session file is refused (fp32 KV: other bytes)
        other = str(tmp_path / "o.kmss")
        eng.save_session(other, prompt, slot=2, kv_dtype=2, conv_window=False)
        os.rename(path + ".conv.bak", other + ".conv")
        with pytest.raises(DmError):
            eng.load_session(other, slot=2)
