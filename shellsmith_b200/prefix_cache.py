"""Byte-bounded LRU of prompt-prefix cache snapshots.

Mirrors studio_compute/cache.py:6-113 (`PrefixCache`): the same key
(identity, policy, precision, tuple(tokens)), longest-prefix match, LRU order
(a hit moves the entry to the back), byte accounting including the logits,
capacity callback, trim, and counters (hits, misses, hit_tokens, evictions,
stored, skipped). Golden traces of the reference class pin the bookkeeping
bit-exactly.

What a snapshot *is* differs: the reference deep-copies MLX arrays; the paged
engine stores page lists with reference counts, so a snapshot shares its
pages with the request that produced it and a fork copies only the partial
last page (copy-on-write). The byte accounting still charges the snapshot's
full size, as the reference does, so eviction and admission decisions match.
The engine supplies the three storage hooks:
  size(cache)   bytes a snapshot of `cache` holds
  copy(cache)   snapshot to store (or the detached copy returned by get)
  fork(cache)   private writable view for a request (get(..., fork=True))
"""

from __future__ import annotations

from collections import OrderedDict
from typing import Any, Callable


class PrefixCache:
    def __init__(self, limit_bytes: int, *, capacity: Callable | None = None,
                 size: Callable | None = None, copy: Callable | None = None,
                 fork: Callable | None = None, logits_nbytes: Callable | None = None):
        self.limit = limit_bytes
        self.capacity = capacity
        self.size = size or (lambda cache: sum(getattr(x, "nbytes", 0) for x in cache))
        self._copy = copy or (lambda cache: cache)
        self._fork = fork or self._copy
        self._logits_nbytes = logits_nbytes or (lambda logits: getattr(logits, "nbytes", 0))
        self.on_evict: Callable | None = None
        self.entries: OrderedDict = OrderedDict()
        self.bytes = 0
        self.hits = self.misses = self.hit_tokens = 0
        self.evictions = self.stored = self.skipped = 0

    def _match(self, identity, policy, precision, tokens):
        best = None
        for key in self.entries:
            prefix = key[3]
            if (key[:3] == (identity, policy, precision) and len(prefix) <= len(tokens)
                    and tuple(tokens[:len(prefix)]) == prefix
                    and (best is None or len(prefix) > len(best[3]))):
                best = key
        return best

    def contains(self, identity, policy, precision, tokens) -> bool:
        return self._match(identity, policy, precision, tokens) is not None

    def get(self, identity, policy, precision, tokens, *, fork: bool = False):
        """(snapshot copy or fork, logits, matched length) of the longest prefix, or None."""
        best = self._match(identity, policy, precision, tokens)
        if best is None:
            self.misses += 1
            return None
        self.hits += 1
        self.hit_tokens += len(best[3])
        cache, logits, _ = self.entries[best]
        self.entries.move_to_end(best)
        return (self._fork(cache) if fork else self._copy(cache)), logits, len(best[3])

    def _drop_oldest(self) -> None:
        _, (cache, _, removed) = self.entries.popitem(last=False)
        self.bytes -= removed
        self.evictions += 1
        if self.on_evict is not None:
            self.on_evict(cache)

    def put(self, identity, policy, precision, tokens, cache, logits) -> None:
        size = self.size(cache) + self._logits_nbytes(logits)
        capacity = self.limit if self.capacity is None else self.capacity(size)
        capacity = max(0, min(self.limit, capacity))
        if size > capacity:
            self.skipped += 1
            return
        key = (identity, policy, precision, tuple(tokens))
        old = self.entries.pop(key, None)
        if old:
            self.bytes -= old[2]
            if self.on_evict is not None:
                self.on_evict(old[0])
        while self.bytes + size > capacity and self.entries:
            self._drop_oldest()
        self.entries[key] = (self._copy(cache), logits, size)
        self.bytes += size
        self.stored += 1

    def trim(self, limit_bytes: int) -> None:
        target = max(0, min(self.limit, limit_bytes))
        while self.bytes > target and self.entries:
            self._drop_oldest()

    def metrics(self) -> dict:
        return {"bytes": self.bytes, "limit_bytes": self.limit, "entries": len(self.entries),
                "hits": self.hits, "misses": self.misses, "hit_tokens": self.hit_tokens,
                "evictions": self.evictions, "stored": self.stored, "skipped": self.skipped}

    def clear(self) -> None:
        if self.on_evict is not None:
            for cache, _, _ in self.entries.values():
                self.on_evict(cache)
        self.entries.clear()
        self.bytes = 0
