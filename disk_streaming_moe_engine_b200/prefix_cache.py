"""Longest-prefix session cache (reference PrefixCache, src/core/prefix_cache.mojo:102-356).

Same contract as the reference:

* lookup(domain_key, tokens): among valid entries of the same domain whose token list P is
  an exact prefix of the request (0 < |P| <= |tokens|), the longest one wins (the first on
  equal length); a hit advances the access clock and stamps the entry (prefix_cache.mojo:
  127-190).  The domain key (SHA-256 of "model_id:tokenizer_pin:template_rev", :43) only
  partitions; token equality is the only evidence of reuse.
* insert(domain_key, tokens, state, finish_reason): only a clean completion ("stop" or
  "length") inserts; empty token lists are refused; an entry with the same domain and tokens
  is refreshed in place; a full cache replaces the least recently used entry (smallest
  stamp, first on ties); entry ids are "entry_<clock>" (:192-285).
* save_to_dir / load_from_dir: every valid entry as a KMSS v1 file "<entry_id>.kmss" with the
  domain key's 32 bytes as its manifest hash, and "manifest.txt" lines
  "<entry_id> <stamp> <domain_key> <file>"; loading clears the cache, skips malformed lines
  and unreadable files and restores the clock to the largest stamp (:287-356).

What differs is where an entry's state lives.  The reference copies the KV cache and GDN
state objects into host memory; here an entry owns one sequence slot of the engine
(`EngineSlotStore`), and insert / restore are device copies of the whole sequence state
(dm_seq_copy: K/V through the page tables, GDN states and conv windows) — nothing crosses
PCIe.  Files also carry the GDN conv window in a ".conv" sidecar (dm_kmss_save_conv), so a
restored entry decodes like the sequence it was taken from.
"""
from __future__ import annotations

import copy
import dataclasses
import hashlib
import os


def compute_domain_key(model_id: str, tokenizer_pin: str, template_subset_rev: str) -> str:
    """SHA-256 of "model_id:tokenizer_pin:template_subset_rev" as 64 lowercase hex digits."""
    return hashlib.sha256(f"{model_id}:{tokenizer_pin}:{template_subset_rev}".encode()).hexdigest()


def domain_key_to_bytes(domain_key: str) -> bytes:
    """The hex key as 32 bytes (missing digits as zero bytes, as the reference pads)."""
    out = bytearray(32)
    for i in range(32):
        pair = domain_key[2 * i:2 * i + 2]
        if len(pair) == 2:
            try:
                out[i] = int(pair, 16)
            except ValueError:
                out[i] = 0
    return bytes(out)


@dataclasses.dataclass
class PrefixCacheEntry:
    entry_id: str
    domain_key: str
    tokens: list
    last_accessed_step: int
    is_valid: bool = True
    next_token: int | None = None  # the argmax after the entry's last token, when known


@dataclasses.dataclass
class PrefixLookupResult:
    hit: bool
    prefix_len: int
    entry_index: int
    delta_tokens_len: int
    domain_key: str


class HostStore:
    """Entry states held as host objects (deep copies), like the reference's entries."""

    def __init__(self, capacity: int):
        self.states = [None] * capacity

    def snapshot(self, i: int, state):
        self.states[i] = copy.deepcopy(state)

    def restore(self, i: int, dst=None):
        return copy.deepcopy(self.states[i])

    def save(self, i: int, path: str, tokens, manifest_hash: bytes):
        raise NotImplementedError("host store entries are not persisted")

    def load(self, i: int, path: str):
        raise NotImplementedError("host store entries are not persisted")


class EngineSlotStore:
    """Entry i lives in sequence slot slots[i] of `engine` (slots reserved for the cache)."""

    def __init__(self, engine, slots):
        self.engine = engine
        self.slots = list(slots)

    def snapshot(self, i: int, src_slot: int):
        self.engine.seq_copy(src_slot, self.slots[i])

    def restore(self, i: int, dst_slot: int):
        self.engine.seq_copy(self.slots[i], dst_slot)
        return dst_slot

    def save(self, i: int, path: str, tokens, manifest_hash: bytes):
        self.engine.save_session(path, tokens, slot=self.slots[i], manifest_hash=manifest_hash)

    def load(self, i: int, path: str):
        return [int(t) for t in self.engine.load_session(path, slot=self.slots[i])]


class PrefixCache:
    """Bounded LRU cache of session states keyed by exact token prefixes."""

    def __init__(self, capacity: int = 8, store=None):
        if capacity <= 0:
            raise ValueError("capacity must be positive")
        self.capacity = capacity
        self.store = store if store is not None else HostStore(capacity)
        if isinstance(self.store, EngineSlotStore) and len(self.store.slots) < capacity:
            raise ValueError("the engine store needs one slot per entry")
        self.entries: list[PrefixCacheEntry] = []
        self.access_clock = 0

    def size(self) -> int:
        return sum(1 for e in self.entries if e.is_valid)

    def clear(self):
        self.entries.clear()
        self.access_clock = 0

    def lookup(self, domain_key: str, req_tokens) -> PrefixLookupResult:
        req = [int(t) for t in req_tokens]
        if not req:
            return PrefixLookupResult(False, 0, -1, 0, domain_key)
        best, best_len = -1, 0
        for i, e in enumerate(self.entries):
            if not e.is_valid or e.domain_key != domain_key:
                continue
            n = len(e.tokens)
            if n == 0 or n > len(req):
                continue
            if e.tokens == req[:n] and n > best_len:
                best, best_len = i, n
        if best >= 0:
            self.access_clock += 1
            self.entries[best].last_accessed_step = self.access_clock
            return PrefixLookupResult(True, best_len, best, len(req) - best_len, domain_key)
        return PrefixLookupResult(False, 0, -1, len(req), domain_key)

    def insert(self, domain_key: str, canonical_tokens, state, finish_reason: str, next_token: int | None = None) -> bool:
        """`state`: the source slot (engine store) or state object (host store) after exactly
        `canonical_tokens`."""
        if finish_reason not in ("stop", "length"):
            return False
        toks = [int(t) for t in canonical_tokens]
        if not toks:
            return False
        self.access_clock += 1
        for i, e in enumerate(self.entries):
            if e.is_valid and e.domain_key == domain_key and e.tokens == toks:
                self.store.snapshot(i, state)
                e.last_accessed_step = self.access_clock
                e.next_token = next_token
                return True
        entry = PrefixCacheEntry(f"entry_{self.access_clock}", domain_key, toks, self.access_clock, True, next_token)
        if len(self.entries) >= self.capacity:
            lru = 0
            for i in range(1, len(self.entries)):
                if self.entries[i].last_accessed_step < self.entries[lru].last_accessed_step:
                    lru = i
            self.store.snapshot(lru, state)
            self.entries[lru] = entry
            return True
        self.store.snapshot(len(self.entries), state)
        self.entries.append(entry)
        return True

    def restore(self, result: PrefixLookupResult, dst):
        """The hit entry's state into `dst` (engine store: a slot; host store: returned)."""
        if not result.hit:
            raise ValueError("restore of a miss")
        return self.store.restore(result.entry_index, dst)

    def save_to_dir(self, cache_dir: str):
        os.makedirs(cache_dir, exist_ok=True)
        lines = []
        for i, e in enumerate(self.entries):
            if not e.is_valid:
                continue
            name = f"{e.entry_id}.kmss"
            self.store.save(i, os.path.join(cache_dir, name), e.tokens, domain_key_to_bytes(e.domain_key))
            lines.append(f"{e.entry_id} {e.last_accessed_step} {e.domain_key} {name}\n")
        with open(os.path.join(cache_dir, "manifest.txt"), "w") as f:
            f.write("".join(lines))

    def load_from_dir(self, cache_dir: str):
        path = os.path.join(cache_dir, "manifest.txt")
        try:
            text = open(path).read()
        except OSError:
            return
        self.entries.clear()
        for line in text.split("\n"):
            line = line.strip()
            if not line:
                continue
            parts = line.split(" ")
            if len(parts) < 4 or len(self.entries) >= self.capacity:
                continue
            try:
                step = int(parts[1])
            except ValueError:
                step = 0
            try:
                toks = self.store.load(len(self.entries), os.path.join(cache_dir, parts[3]))
            except Exception:  # a damaged or unreadable entry is skipped, as the reference does
                continue
            self.entries.append(PrefixCacheEntry(parts[0], parts[2], toks, step, True))
            self.access_clock = max(self.access_clock, step)


def prefill_with_cache(engine, cache: PrefixCache, domain_key: str, tokens, slot: int, want_logits: bool = False):
    """A prompt through the cache: longest cached prefix restored into `slot` on a hit (a
    device copy), then only the remaining tokens prefilled (the delta prefill of the
    reference's session path, cmd_decode.mojo:1258-1296).  -> (logits or None, next token,
    lookup result).  A request equal to a cached entry needs no prefill: its stored next
    token is returned (logits None)."""
    import numpy as np
    toks = np.ascontiguousarray(tokens, np.int32)
    res = cache.lookup(domain_key, toks)
    if res.hit and res.delta_tokens_len == 0 and cache.entries[res.entry_index].next_token is not None:
        cache.restore(res, slot)
        return None, cache.entries[res.entry_index].next_token, res
    if res.hit and res.delta_tokens_len > 0:
        cache.restore(res, slot)
        delta = toks[res.prefix_len:]
    else:
        engine.seq_reset(slot)
        delta = toks
        res = dataclasses.replace(res, hit=False, prefix_len=0, entry_index=-1, delta_tokens_len=len(toks))
    logits, nxt = engine.prefill(delta, slot=slot, want_logits=want_logits)
    return logits, nxt, res
