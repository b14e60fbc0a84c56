"""The reference's scheduler drives the paged engine end to end on the GPU.

runtime.create_request / prefill_request / advance_requests / sample_requests /
release_request run under scheduler.ContinuousBatcher, with PagedResident
doing each step's cache work (GDN glue + recurrence, paged K/V and attention)
for a small seeded hybrid model. Bars: a request interleaved with others
(chunked prefill, shared decode launches, slot reuse) gives the logprobs it
gives alone within 0.02 (batch shape changes bf16 GEMM and split-K rounding
only); a prefix-cache hit continues from the cached offset to the logprobs of
a full prefill within the same bar; every page and reservation is returned.
"""

import numpy as np
import pytest
import torch

from shellsmith_b200.engine import HybridConfig
from shellsmith_b200.resident import PagedRuntimeEngine, ToyHybridModel

pytestmark = pytest.mark.gpu

TOL = 0.02  # measured worst 0.005 (most requests bit-identical)


def _cfg():
    return HybridConfig(layers=4, gdn_key_heads=2, gdn_value_heads=4, q_heads=4, kv_heads=2,
                        head_dim=128, max_seqs=6, num_pages=128, max_context=512,
                        snapshot_rows=4, gdn_taps=True)


def _bodies(rng, n, use_prefix_cache=False):
    out = []
    for i in range(n):
        plen = int(rng.integers(3, 70))
        targets = [int(t) for t in rng.integers(0, 97, size=int(rng.integers(3, 8)))]
        out.append((f"r{i}", {"policy": "p", "prompt_token_ids": [int(t) for t in
                                                                   rng.integers(0, 97, plen)],
                              "max_tokens": len(targets), "target_token_ids": targets,
                              "use_prefix_cache": use_prefix_cache, "seed": i}))
    return out


def _run(bodies, concurrency, prefill_tokens=16, model=None, runtime=None):
    cfg = _cfg()
    rt = runtime or PagedRuntimeEngine(cfg, model or ToyHybridModel(cfg, seed=3),
                                       prefill_tokens=prefill_tokens, concurrency=concurrency)
    done, failed = {}, {}
    batcher = rt.inference_scheduler(
        finish=lambda r: done.__setitem__(r.request_id, (list(r.tokens), list(r.logprobs),
                                                         r.cached_tokens, r.reason)),
        fail=lambda name, error: failed.__setitem__(name, repr(error)))
    for request_id, body in bodies:
        batcher.enqueue(request_id, body)
    steps = 0
    while batcher.pending or batcher.active:
        batcher.step()
        steps += 1
        assert steps < 500
    torch.cuda.synchronize()
    assert not failed, failed
    return rt, done


def test_interleaved_requests_match_each_request_alone(cuda):
    bodies = _bodies(np.random.default_rng(0), 6)
    rt, together = _run(bodies, concurrency=3)
    model = rt.model
    for request_id, body in bodies:
        _, alone = _run([(request_id, body)], concurrency=1, model=model)
        tokens, lps, _, reason = together[request_id]
        assert tokens == body["target_token_ids"] and reason == "length"
        assert alone[request_id][0] == tokens
        np.testing.assert_allclose(lps, alone[request_id][1], atol=TOL)
    # Everything returned: no reservation, no live slot, every page free.
    assert rt.reserved == {} and not rt.cache.blocks.active.any()
    assert rt.cache.blocks.free_pages == rt.cache.cfg.num_pages


def test_prefix_cache_hit_continues_from_the_cached_prompt(cuda):
    rng = np.random.default_rng(1)
    base = [int(t) for t in rng.integers(0, 97, 40)]
    first = ("a", {"policy": "p", "prompt_token_ids": base, "max_tokens": 3,
                   "target_token_ids": [5, 6, 7], "seed": 1})
    longer = base + [int(t) for t in rng.integers(0, 97, 21)]
    second = {"policy": "p", "prompt_token_ids": longer, "max_tokens": 4,
              "target_token_ids": [9, 8, 7, 6], "seed": 2}
    cfg = _cfg()
    model = ToyHybridModel(cfg, seed=3)
    rt = PagedRuntimeEngine(cfg, model, prefill_tokens=16, concurrency=2)
    _run([first], concurrency=2, runtime=rt)
    _, hit = _run([("b", dict(second))], concurrency=2, runtime=rt)
    assert rt.prefixes.metrics()["hits"] >= 1
    assert hit["b"][2] == len(base)                     # cached_tokens: the stored prompt
    _, cold = _run([("b", dict(second, use_prefix_cache=False))], concurrency=1, model=model)
    assert cold["b"][2] == 0
    np.testing.assert_allclose(hit["b"][1], cold["b"][1], atol=TOL)
    # Snapshots hold pages until the prefix cache lets them go.
    held = rt.cache.cfg.num_pages - rt.cache.blocks.free_pages
    assert held > 0 and rt.reserved == {}
    rt.prefixes.clear()
    assert rt.cache.blocks.free_pages == rt.cache.cfg.num_pages
