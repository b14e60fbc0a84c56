"""The scheduler and prefix cache reproduce the reference's own traces bit-exactly.

Fixtures come from running the reference ContinuousBatcher / PrefixCache
(tests/golden/make_golden.py); here the same scenarios drive this build's
classes and every step record, callback event and counter must be equal.
"""

import json
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest

from shellsmith_b200.prefix_cache import PrefixCache
from shellsmith_b200.scheduler import ContinuousBatcher

GOLDEN = Path(__file__).resolve().parent / "golden"
SCHED = json.loads((GOLDEN / "scheduler_traces.json").read_text())
PREFIX = json.loads((GOLDEN / "prefix_cache_traces.json").read_text())


def harness(concurrency, memory_slots=None, churn_rng=None):
    events, released, completed, failed, live = [], [], {}, {}, set()

    def create(request_id, body):
        if body.get("invalid"):
            raise ValueError("invalid request")
        if memory_slots is not None and len(live) >= memory_slots:
            events.append(("defer", request_id))
            return None
        live.add(request_id)
        events.append(("admit", request_id))
        return SimpleNamespace(request_id=request_id, body=body, tokens=[], offset=0,
                               logits=None, needs_decode=False, reason=None)

    def prefill(request):
        step = request.body.get("chunk", 2)
        request.offset += min(step, request.body["prompt_length"] - request.offset)
        events.append(("prefill", request.request_id, request.offset))
        if request.offset == request.body["prompt_length"]:
            request.logits = True

    def advance(requests):
        events.append(("advance", [r.request_id for r in requests]))
        for r in requests:
            r.needs_decode = False

    def sample(requests):
        events.append(("sample", [r.request_id for r in requests]))
        for r in requests:
            if r.body.get("fail"):
                raise RuntimeError("kernel failed")
            r.tokens.append(len(r.tokens))
            done = len(r.tokens) == r.body["maximum"]
            if churn_rng is not None and not done:
                done = churn_rng.random() < r.body.get("finish_p", 0.0)
            r.reason = "length" if done else None
            r.needs_decode = r.reason is None

    def release(request):
        live.discard(request.request_id)
        released.append(request.request_id)
        events.append(("release", request.request_id))

    batcher = ContinuousBatcher(
        concurrency, create=create, prefill=prefill, advance=advance, sample=sample,
        finish=lambda r: (completed.__setitem__(r.request_id, list(r.tokens)),
                          events.append(("finish", r.request_id))),
        fail=lambda name, error: (failed.__setitem__(name, str(error)),
                                  events.append(("fail", name, str(error)))),
        release=release)
    return batcher, events, released, completed, failed


def run(scenario):
    churn = np.random.default_rng(scenario["seed"]) if scenario.get("churn") else None
    batcher, events, released, completed, failed = harness(
        scenario["concurrency"], scenario.get("memory_slots"), churn)
    records = []
    for op in scenario["script"]:
        if op[0] == "enqueue":
            batcher.enqueue(op[1], op[2])
        elif op[0] == "cancel":
            batcher.cancel(op[1])
        elif op[0] == "step":
            records.extend(batcher.step() for _ in range(op[1]))
        elif op[0] == "drain":
            while batcher.pending or batcher.active:
                records.append(batcher.step())
                assert len(records) < 5000
        elif op[0] == "close":
            batcher.close()
    return {"records": records, "events": [list(e) for e in events], "released": released,
            "completed": completed, "failed": failed, "active": sorted(batcher.active),
            "pending": [p[0] for p in batcher.pending]}


@pytest.mark.parametrize("name", sorted(SCHED))
def test_scheduler_matches_reference_trace(name):
    want = SCHED[name]["trace"]
    got = json.loads(json.dumps(run(SCHED[name]["scenario"])))
    assert got["events"] == want["events"]
    assert got["records"] == want["records"]
    for key in ("released", "completed", "failed", "active", "pending"):
        assert got[key] == want[key], key


def test_rejects_nonpositive_concurrency():
    for bad in (0, -1, 2.0):
        with pytest.raises(ValueError):
            ContinuousBatcher(bad, create=None, prefill=None, advance=None, sample=None,
                              finish=None, fail=None, release=None)


class _Arr:
    def __init__(self, n):
        self.nbytes = n


@pytest.mark.parametrize("name", sorted(PREFIX))
def test_prefix_cache_matches_reference_trace(name):
    case = PREFIX[name]
    spare = {"v": 120}
    capacity = (lambda size: spare["v"] - size) if case["capacity"] == "spare" else None
    cache = PrefixCache(case["limit"], capacity=capacity,
                        size=lambda c: sum(x.nbytes for item in c for x in item.state))
    for op, want in zip(case["ops"], case["outcomes"]):
        if op[0] == "put":
            _, ident, pol, prec, tokens, size, logits = op
            cache.put(ident, pol, prec, tokens, [SimpleNamespace(state=[_Arr(size)])],
                      _Arr(logits))
            result = None
        elif op[0] in ("get", "get_fork"):
            hit = cache.get(*op[1:5], fork=op[0] == "get_fork")
            result = None if hit is None else hit[2]
        elif op[0] == "contains":
            result = cache.contains(*op[1:5])
        else:
            cache.trim(op[1])
            result = None
        assert result == want["result"]
        assert cache.metrics() == want["metrics"]
        assert [[k[0], k[1], k[2], list(k[3])] for k in cache.entries] == want["keys"]
