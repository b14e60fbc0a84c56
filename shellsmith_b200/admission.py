"""Byte admission for rollout requests, with the reference's estimates and rules.

Mirrors the memory side of the reference runtime over the same engine
attributes (`resident.budget`, `resident.mx.get_active_memory()`,
`persistent_bytes()`, `reserved`, `prefixes`, `policies`, `policy_users`,
`idle_factors`, `execution_profile`, `capabilities`):

  estimate_inference      model.py:271-287   per-request cache bound: K+V bf16 of
                                             every attention layer per token, fp32
                                             GDN state per GDN layer, x batch, +2 GiB
  resident_admit          model.py:289-300   needed = max(active + add,
                                             (persistent or active) + reserved + add)
  admission_budget_bytes  engine.py:509-518
  evict_policy            engine.py:424-434  first policy without users
  engine_admit            engine.py:520-539  bf16-fast check, then resident_admit,
                                             evicting idle policies on MemoryError
  cache_capacity          runtime.py:71-86   bytes the prefix snapshots may hold
  runtime_admit           runtime.py:88-92   trim snapshots to that capacity, admit
  inference_batch_capacity runtime.py:119-133

Golden traces of the reference methods on seeded fake engines pin every
result, error text, trim target and policy eviction bit-exactly.

`paged_cache_bytes` is the paged engine's exact footprint of a request (whole
pages plus its GDN state rows); the reference's estimate stays the admission
bound so that decisions match the reference's.
"""

from __future__ import annotations

from typing import Any

HEADROOM = 2 << 30


def estimate_inference(cfg, length: int, batch: int = 1, *, cache_precision: str = "bf16") -> int:
    """The reference's conservative bound: the 8-bit cache is charged as bf16 too."""
    if cache_precision not in ("bf16", "8bit"):
        raise ValueError("Unsupported inference cache precision.")
    cache = length * cfg.kv_heads * cfg.head_dim * 4 * len(cfg.attention_layers)
    recurrent = cfg.gdn_value_heads * cfg.value_dim * cfg.key_dim * 4 * len(cfg.gdn_layers)
    return batch * (cache + recurrent) + HEADROOM


def paged_cache_bytes(cfg, length: int, batch: int = 1) -> int:
    """Bytes the paged pools hold for `batch` sequences of `length` tokens."""
    pages = -(-int(length) // cfg.page_size)
    page = cfg.kv_heads * 2 * cfg.page_size * cfg.head_dim * 2
    state = cfg.gdn_value_heads * cfg.value_dim * cfg.key_dim * 4 * len(cfg.gdn_layers)
    return batch * (pages * page * len(cfg.attention_layers) + state)


def resident_admit(resident: Any, additional: int, reserved: int = 0, persistent=None) -> None:
    active = resident.mx.get_active_memory()
    base = active if persistent is None else persistent
    needed = max(active + additional, base + reserved + additional)
    if needed > resident.budget:
        raise MemoryError(f"Admission needs {needed} bytes; budget is {resident.budget}.")


def admission_budget_bytes(engine: Any) -> int:
    budget = engine.resident.budget
    if engine.execution_profile == "legacy":
        return budget
    recommended = engine.capabilities.get("recommended_working_set_bytes")
    return min(budget, int(recommended or budget))


def evict_policy(engine: Any) -> bool:
    """Drop the least recently used policy nobody is using; False when none can go."""
    for name in engine.policies:
        if engine.policy_users.get(name, 0):
            continue
        policy = engine.policies.pop(name)
        if engine.resident.selected is policy["factors"]:
            engine.resident.select(engine.idle_factors)
        return True
    return False


def engine_admit(engine: Any, additional: int) -> None:
    while True:
        try:
            persistent = engine.persistent_bytes()
            reserved = sum(engine.reserved.values())
            if engine.execution_profile == "bf16-fast":
                needed = max(engine.mx.get_active_memory() + additional,
                             persistent + reserved + additional)
                budget = engine.admission_budget_bytes()
                if needed > budget:
                    raise MemoryError(f"Admission needs {needed} bytes; budget is {budget}.")
            engine.resident.admit(additional, reserved, persistent=persistent)
            return
        except MemoryError:
            if not engine._evict_policy():
                raise


def cache_capacity(engine: Any, snapshot_bytes: int = 0, *, additional: int = 0) -> int:
    retained = engine.prefixes.bytes
    noncache = engine.persistent_bytes() - retained
    budget = engine.admission_budget_bytes()
    return max(0, min(engine.prefixes.limit,
                      budget - noncache - sum(engine.reserved.values()) - additional,
                      retained + budget - engine.mx.get_active_memory() - snapshot_bytes
                      - additional))


def runtime_admit(engine: Any, additional: int) -> None:
    """Evict detached prefix snapshots down to what fits, then admit."""
    engine.prefixes.trim(cache_capacity(engine, additional=additional))
    engine_admit(engine, additional)


def inference_batch_capacity(engine: Any, body: dict, requested: int) -> int:
    """Largest batch of copies of `body` whose peak fits the budget (at least 1)."""
    noncache = engine.persistent_bytes() - engine.prefixes.bytes
    active = engine.mx.get_active_memory() - engine.prefixes.bytes
    reserved = sum(engine.reserved.values())
    length = len(body["prompt_token_ids"]) + body["max_tokens"]
    budget = engine.admission_budget_bytes()
    top = min(getattr(engine, "inference_concurrency", requested), requested)
    for count in range(top, 1, -1):
        peak = engine.resident.estimate_inference(
            length, count, cache_precision=body.get("cache_precision", "bf16"))
        if max(active + peak, noncache + reserved + peak) <= budget:
            return count
    return 1


class ResidentBudget:
    """The resident model's side of admission for a hybrid GDN/attention layout:
    `estimate_inference` and `admit` against `budget`, with `mx.get_active_memory()`
    the live device bytes (the reference's names)."""

    def __init__(self, cfg, budget: int, mx: Any):
        self.cfg, self.budget, self.mx = cfg, budget, mx

    def estimate_inference(self, length, batch=1, *, cache_precision="bf16"):
        return estimate_inference(self.cfg, length, batch, cache_precision=cache_precision)

    def admit(self, additional, reserved=0, persistent=None):
        resident_admit(self, additional, reserved, persistent)


class AdmissionMixin:
    """Engine methods with the reference's names; the engine supplies `resident`,
    `mx`, `reserved`, `prefixes`, `policies`, `policy_users`, `idle_factors`,
    `execution_profile`, `capabilities` and `persistent_bytes()`."""

    _evict_policy = evict_policy
    admission_budget_bytes = admission_budget_bytes
    _cache_capacity = cache_capacity
    admit = runtime_admit
    inference_batch_capacity = inference_batch_capacity
