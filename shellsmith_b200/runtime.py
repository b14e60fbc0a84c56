"""Request lifecycle over the paged cache, with the reference's admission rules.

Mirrors studio_compute/inference.py:14-118 (`create_request`) and 238-245
(`release_request`) over the same engine attributes the reference reads
(`resident.estimate_inference`, `prefixes`, `policies`, `idle_factors`,
`reserved`, `persistent_bytes()`, `admission_budget_bytes()`, `admit()`,
`_borrow_policy()`, `prefix_identity`, `lm.make_cache()`, `mx`), so the same
engine object can sit behind either. The rules, in order:

  1. the peak is the estimate for prompt + maximum new tokens (maximum = the
     forced target length, else max_tokens), plus -- when the prefix cache is
     in use (default on) -- min(prefix limit, estimate for the prompt alone);
  2. a policy that is not resident is charged every idle factor's bytes;
  3. while other reservations exist, a request that would fit the budget only
     once they are released defers (returns None) before admission;
  4. admit(peak + policy bytes); a MemoryError defers when reservations exist
     and the request could fit after they end, else propagates;
  5. reserve ("continuous_inference", id) -> peak, enter the policy lease
     (MemoryError: drop the reservation, defer if others remain, else raise);
  6. take a prefix-cache fork of the longest cached prefix, else a fresh cache
     (8-bit precision quantizes the items that can be);
  7. the RNG is the durable key when given, else a key from the seed; offset
     and cached_tokens are the matched prefix length, and a full-prompt match
     restores the cached logits;
  8. any exception after the reservation exits the lease if it was entered,
     drops the reservation and propagates.

`release_request` clears the cache, drops logits/RNG/factors, exits the lease
and always drops the reservation. Golden traces of the reference functions
run on fake engines pin every outcome, call order and final reservation
table bit-exactly.

The paged pieces: `PagedSequence` is the per-request cache handle (a state
slot in `HybridCacheEngine`; clear() releases it) and `paged_prefix_cache`
wires `PrefixCache` to refcounted page snapshots with copy-on-write forks.
"""

from __future__ import annotations

import math
import time
from typing import Any

import numpy as np

from .prefix_cache import PrefixCache
from .scheduler import DecodeRequest

RESERVATION = "continuous_inference"


def _maximum(body: dict) -> int:
    return len(body.get("target_token_ids", [])) or body["max_tokens"]


def request_peak(engine: Any, body: dict) -> int:
    """Bytes reserved for a request for its whole life (inference.py:21-33)."""
    precision = body.get("cache_precision", "bf16")
    prompt = len(body["prompt_token_ids"])
    estimate = engine.resident.estimate_inference
    peak = estimate(prompt + _maximum(body), cache_precision=precision)
    if body.get("use_prefix_cache", True):
        peak += min(engine.prefixes.limit, estimate(prompt, cache_precision=precision))
    return peak


def _policy_bytes(engine: Any, body: dict) -> int:
    if body["policy"] in engine.policies:
        return 0
    return sum(value.nbytes for value in engine.idle_factors.values())


def _fresh_cache(engine: Any, precision: str):
    cache = engine.lm.make_cache()
    if precision == "8bit" and isinstance(cache, list):  # a paged cache's precision is its pool's
        cache = [item.to_quantized(bits=8, group_size=64) if hasattr(item, "to_quantized")
                 else item for item in cache]
    return cache


def create_request(engine: Any, request_id: str, body: dict) -> DecodeRequest | None:
    """A request holding its reservation, lease, cache and RNG, or None to defer."""
    started = time.monotonic()
    peak = request_peak(engine, body)
    policy_bytes = _policy_bytes(engine, body)
    if engine.reserved:
        noncache = engine.persistent_bytes() - engine.prefixes.bytes
        needed = noncache + peak + policy_bytes
        budget = engine.admission_budget_bytes()
        # Fits once the other reservations end; evicting prefixes cannot help now.
        if needed <= budget < needed + sum(engine.reserved.values()):
            return None
    try:
        engine.admit(peak + policy_bytes)
    except MemoryError:
        noncache = engine.persistent_bytes() - engine.prefixes.bytes
        if engine.reserved and noncache + peak <= engine.admission_budget_bytes():
            return None
        raise

    key = (RESERVATION, request_id)
    engine.reserved[key] = peak
    lease = engine._borrow_policy(body["policy"])
    entered = False
    try:
        try:
            factors = lease.__enter__()
        except MemoryError:
            engine.reserved.pop(key, None)
            if engine.reserved:
                return None
            raise
        entered = True
        precision = body.get("cache_precision", "bf16")
        hit = None
        if body.get("use_prefix_cache", True):
            hit = engine.prefixes.get(engine.prefix_identity, body["policy"], precision,
                                      body["prompt_token_ids"], fork=True)
        if hit is None:
            cache, logits, offset = _fresh_cache(engine, precision), None, 0
        else:
            cache, logits, offset = hit
        mx = engine.mx
        rng = (mx.array(body["rng_key"], mx.uint32) if "rng_key" in body
               else mx.random.key(body["seed"]))
        request = DecodeRequest(request_id, body, cache, factors, lease, rng, started,
                                offset=offset, cached_tokens=offset)
        if offset == len(body["prompt_token_ids"]):
            request.logits = logits
            request.decode_started = time.monotonic()
            request.prefill_seconds = request.decode_started - started
        return request
    except BaseException:
        if entered:
            lease.__exit__(None, None, None)
        engine.reserved.pop(key, None)
        raise


def release_request(engine: Any, request: DecodeRequest) -> None:
    """Free a request's cache, lease and reservation (success, failure or cancel)."""
    try:
        request.cache.clear()
        request.logits = request.rng = request.factors = None
        request.lease.__exit__(None, None, None)
    finally:
        engine.reserved.pop((RESERVATION, request.request_id), None)


def prefill_request(engine: Any, request: DecodeRequest) -> None:
    """Advance at most engine.prefill_tokens prompt tokens (inference.py:124-163).

    The request's cache is a PagedSequence: a fresh one takes its slot (and the
    pages of the whole prompt) on its first chunk; a prefix-cache fork continues
    from its cached offset. The last chunk sets the logits and, unless the body
    opts out, stores the prompt's snapshot in the prefix cache.
    """
    body = request.body
    prompt = body["prompt_token_ids"]
    start = request.offset
    stop = min(len(prompt), start + engine.prefill_tokens)
    seq = request.cache
    if seq.slot is None:
        seq.slot = seq.engine.admit(request.request_id, len(prompt))
    logits = engine.resident.prefill(seq, prompt[start:stop], start)
    request.offset = stop
    if stop < len(prompt):
        return
    request.logits = logits
    if body.get("use_prefix_cache", True):
        engine.prefixes.put(engine.prefix_identity, body["policy"],
                            body.get("cache_precision", "bf16"), prompt, request.cache,
                            request.logits)
    request.prefill_seconds = time.monotonic() - request.started
    request.decode_started = time.monotonic()


def advance_requests(engine: Any, requests: list) -> None:
    """One decode token for every listed request (inference.py:166-173)."""
    engine.resident.decode_rows(engine, requests)
    for request in requests:
        request.batch_size = max(request.batch_size, len(requests))


def sample_requests(engine: Any, requests: list) -> None:
    """One token per request from its logits (inference.py:176-218): a forced target
    when the body has one, else a categorical draw from a generator seeded with the
    request's RNG key (the reference splits an MLX key; the draws differ, the
    bookkeeping does not)."""
    import torch

    for request in requests:
        lp = torch.log_softmax(request.logits.float(), dim=-1)[0]
        forced = request.body.get("target_token_ids")
        if forced:
            token = int(forced[len(request.tokens)])
        else:
            key = [int(x) for x in np.asarray(request.rng).ravel()]
            gen = torch.Generator(device="cpu").manual_seed(
                (key[0] << 32 | key[-1]) + len(request.tokens))
            token = int(torch.multinomial(lp.exp().cpu(), 1, generator=gen))
        finish_sample(request, token, float(lp[token]))


def finish_sample(request: DecodeRequest, token: int, logprob: float) -> None:
    """Record one sampled token and set the finish reason (inference.py:202-218)."""
    if not math.isfinite(logprob):
        raise FloatingPointError("Nonfinite behavior logprob.")
    request.tokens.append(token)
    request.logprobs.append(logprob)
    body = request.body
    forced = body.get("target_token_ids")
    if not forced and token in body.get("stop_token_ids", []):
        request.reason = "stop"
    elif len(request.tokens) == (len(forced) if forced else body["max_tokens"]):
        request.reason = "length"
    request.needs_decode = request.reason is None


# ---------------------------------------------------------------- paged cache handles
class PagedSequence:
    """A request's cache in the paged engine: one state slot (batch row, block-table
    row, GDN state row). clear() releases the slot; a second clear() is a no-op."""

    def __init__(self, engine, slot: int):
        self.engine, self.slot = engine, slot

    @property
    def tokens(self) -> int:
        return 0 if self.slot is None else int(self.engine.blocks.lengths[self.slot])

    def clear(self) -> None:
        if self.slot is not None:
            self.engine.release(self.slot)
            self.slot = None


def paged_prefix_cache(engine, limit_bytes: int, capacity=None) -> PrefixCache:
    """A PrefixCache whose entries are refcounted page snapshots of `engine`.

    put(cache=PagedSequence) stores a snapshot (full pages shared, partial last
    page and GDN state copied); get(fork=True) opens a new PagedSequence over the
    shared pages with a private copy of the partial page; get(fork=False) hands
    out another snapshot that the caller drops with engine.drop_snapshot.
    Eviction drops the snapshot's page references.
    """
    from .engine import PagedSnapshot

    def copy(cache):
        if isinstance(cache, PagedSnapshot):
            return engine.copy_snapshot(cache)
        return engine.snapshot(cache.slot)

    def fork(snap):
        return PagedSequence(engine, engine.fork(snap))

    prefixes = PrefixCache(limit_bytes, capacity=capacity, size=lambda c: (
        c.nbytes if isinstance(c, PagedSnapshot) else engine.cache_bytes(c.tokens)),
        copy=copy, fork=fork)
    prefixes.on_evict = engine.drop_snapshot
    return prefixes
