"""Continuous batching scheduler with the reference's admission and retirement rules.

Mirrors studio_compute/mlx_racing.py:13-153 (`DecodeRequest`,
`ContinuousBatcher`): same constructor, callbacks, step record and error
isolation, so an engine written for the reference can drive this one and the
paged engine below can be driven by either. The rules, per step:

  1. admit from the FIFO queue while fewer than `concurrency` are active;
     create() returning None defers (stops admission this step), raising
     fails that request and admission continues (mlx_racing.py:83-94);
  2. prefill exactly one request whose logits are still None, chosen
     round-robin by a cursor over those requests (96-105); a prefill error
     retires that request only;
  3. group the requests with logits by body["policy"] in insertion order;
     per group advance the rows that need a decode, then sample the whole
     group; an error retires the whole group (107-122);
  4. retire every sampled request that set a finish reason (128-129).

Bit-exact equality of the step records and callback order with the
reference batcher is checked against golden traces of the reference itself.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from typing import Any, Callable


@dataclass
class DecodeRequest:
    """One request's resources and progress (fields of mlx_racing.py:13-37)."""

    request_id: str
    body: dict
    cache: Any
    factors: Any
    lease: Any
    rng: Any
    started: float
    offset: int = 0
    cached_tokens: int = 0
    logits: Any = None
    needs_decode: bool = False
    batch_size: int = 1
    prefill_seconds: float = 0.0
    decode_started: float = 0.0
    tokens: list = field(default_factory=list)
    logprobs: list = field(default_factory=list)
    reason: str | None = None


class ContinuousBatcher:
    """Refills free slots at every token boundary; one prefill chunk per step."""

    def __init__(self, concurrency: int, *, create: Callable, prefill: Callable,
                 advance: Callable, sample: Callable, finish: Callable, fail: Callable,
                 release: Callable) -> None:
        if type(concurrency) is not int or concurrency < 1:
            raise ValueError("Inference concurrency must be a positive integer.")
        self.concurrency = concurrency
        self.create = create
        self.prefill = prefill
        self.advance = advance
        self.sample = sample
        self.finish = finish
        self.fail = fail
        self.release = release
        self.pending: deque = deque()
        self.active: dict = {}
        self.prefill_cursor = 0

    def enqueue(self, request_id: str, body: dict) -> None:
        self.pending.append((request_id, body))

    def cancel(self, request_id: str) -> None:
        self.pending = deque(item for item in self.pending if item[0] != request_id)
        request = self.active.pop(request_id, None)
        if request is not None:
            self.release(request)

    # ------------------------------------------------------------------ step
    def _admit(self) -> None:
        while self.pending and len(self.active) < self.concurrency:
            request_id, body = self.pending[0]
            try:
                request = self.create(request_id, body)
            except Exception as error:  # noqa: BLE001 -- one request fails alone
                self.pending.popleft()
                self.fail(request_id, error)
                continue
            if request is None:
                return  # temporary pressure: keep the queue order, try next step
            self.pending.popleft()
            self.active[request_id] = request

    def _prefill_one(self):
        waiting = [r for r in self.active.values() if r.logits is None]
        if not waiting:
            return None
        request = waiting[self.prefill_cursor % len(waiting)]
        self.prefill_cursor += 1
        try:
            self.prefill(request)
        except Exception as error:  # noqa: BLE001 -- one request fails alone
            self._retire(request, error=error)
            return None
        return (request.request_id, request.offset)

    def step(self) -> dict:
        """Admit, prefill one chunk, decode every ready group, retire finishers."""
        self._admit()
        prefilled = self._prefill_one()
        groups: dict = {}
        for request in self.active.values():
            if request.logits is not None:
                groups.setdefault(request.body["policy"], []).append(request)
        ids, counts, ended, sizes, decode_sizes = [], [], [], [], []
        for rows in groups.values():
            try:
                advancing = [r for r in rows if r.needs_decode]
                if advancing:
                    self.advance(advancing)
                    decode_sizes.append(len(advancing))
                self.sample(rows)
            except Exception as error:  # noqa: BLE001 -- the group's rows fail together
                for request in rows:
                    self._retire(request, error=error)
                continue
            sizes.append(sum(not r.body.get("target_token_ids") for r in rows))
            for request in rows:
                ids.append(request.request_id)
                counts.append(len(request.tokens))
                ended.append(request.reason is not None)
                if request.reason is not None:
                    self._retire(request)
        return {
            "phase": "continuous_decode",
            "request_ids": ids,
            "generated_tokens": counts,
            "finished_requests": ended,
            "batch_sizes": sizes,
            "decode_batch_sizes": decode_sizes,
            "prefill": prefilled,
        }

    def close(self) -> None:
        for request in list(self.active.values()):
            self.cancel(request.request_id)
        self.pending.clear()

    def _retire(self, request, *, error=None) -> None:
        self.active.pop(request.request_id)
        try:
            if error is None:
                self.finish(request)
            else:
                self.fail(request.request_id, error)
        finally:
            self.release(request)
