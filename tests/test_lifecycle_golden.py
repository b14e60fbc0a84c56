"""Request lifecycle and page sharing on the host, no GPU.

The lifecycle fixtures come from running the reference `create_request` /
`release_request` on seeded fake engines (tests/golden/make_golden.py); the
same scenarios drive this build's functions and every outcome (request
fields, deferral or exception text), engine call log and final reservation
table must be equal. The block-manager tests pin the reference counting that
prefix snapshots and forks rely on.
"""

import json
import sys
from pathlib import Path

import numpy as np
import pytest

from shellsmith_b200.block_manager import BlockManager, OutOfPages
from shellsmith_b200.runtime import create_request, finish_sample, release_request
from shellsmith_b200.scheduler import DecodeRequest

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
import make_golden  # noqa: E402  (the fake engine the fixtures were recorded on)

TRACES = json.loads((GOLDEN / "lifecycle_traces.json").read_text())


def _normal(x):
    return json.loads(json.dumps(x, default=list))


def test_lifecycle_fixture_covers_every_outcome():
    kinds = {t["trace"]["outcome"].split(":")[0] for t in TRACES}
    assert {"request", "defer", "MemoryError", "ValueError"} <= kinds


@pytest.mark.parametrize("case", range(len(TRACES)))
def test_lifecycle_matches_reference(case):
    item = TRACES[case]
    got = make_golden.run_lifecycle(create_request, release_request, item["scenario"])
    assert _normal(got) == item["trace"]


def _request(body):
    return DecodeRequest("r", body, [], None, None, None, 0.0)


def test_finish_reasons():
    r = _request({"max_tokens": 3, "stop_token_ids": [9]})
    finish_sample(r, 1, -0.5)
    assert r.reason is None and r.needs_decode
    finish_sample(r, 9, -0.1)
    assert r.reason == "stop" and not r.needs_decode
    r = _request({"max_tokens": 2})
    finish_sample(r, 1, -0.5)
    finish_sample(r, 2, -0.5)
    assert r.reason == "length"
    # Forced targets ignore stop tokens and finish at their own length.
    r = _request({"max_tokens": 9, "target_token_ids": [9, 9], "stop_token_ids": [9]})
    finish_sample(r, 9, -0.5)
    assert r.reason is None
    finish_sample(r, 9, -0.5)
    assert r.reason == "length"
    with pytest.raises(FloatingPointError):
        finish_sample(_request({"max_tokens": 2}), 1, float("-inf"))


def test_shared_pages_return_once_last_owner_drops():
    bm = BlockManager(num_pages=12, page_size=4, max_seqs=4, max_pages_per_seq=8, seed=1)
    a = bm.admit("a", 10)                     # 3 pages, the last one partial
    pages = list(bm.pages[a])
    assert list(bm.refcount[pages]) == [1, 1, 1]
    snap = pages[:2] + bm.take_pages(1)      # a snapshot: full pages shared, copy of partial
    bm.share(pages[:2])
    fork = pages[:2] + bm.take_pages(1)
    bm.share(pages[:2])
    f = bm.adopt("f", fork, 10)
    assert list(bm.refcount[pages[:2]]) == [3, 3]
    assert bm.free_pages == 12 - 5
    bm.extend(f, 17)                           # 5 pages
    assert len(bm.pages[f]) == 5 and bm.lengths[f] == 17
    assert list(bm.table[f, :5]) == bm.pages[f]
    bm.release(a)
    assert bm.free_pages == 12 - 6             # a's private partial page came back
    bm.release(f)
    assert bm.free_pages == 12 - 3 and list(bm.refcount[pages[:2]]) == [1, 1]
    bm.drop(snap)
    assert bm.free_pages == 12 and not bm.refcount.any()
    with pytest.raises(RuntimeError):
        bm.drop([pages[0]])


def test_adopt_extend_and_take_check_sizes_first():
    bm = BlockManager(num_pages=4, page_size=4, max_seqs=2, max_pages_per_seq=3, seed=None)
    s = bm.admit("x", 4)
    with pytest.raises(ValueError):
        bm.adopt("y", bm.pages[s], 9)          # 1 page cannot hold 9 tokens
    with pytest.raises(OutOfPages):
        bm.extend(s, 13)                       # 4 pages > max_pages_per_seq
    with pytest.raises(ValueError):
        bm.extend(s, 2)
    assert bm.free_pages == 3 and bm.lengths[s] == 4
    with pytest.raises(OutOfPages):
        bm.take_pages(4)
    assert bm.free_pages == 3
    np.testing.assert_array_equal(bm.refcount, [1, 0, 0, 0])


def test_slots_lowest_first_and_highest_active():
    """A new sequence takes the lowest free slot, so the engine's decode step can launch
    over rows [0, highest_active()) only; page growth takes pages in row order."""
    bm = BlockManager(num_pages=64, page_size=4, max_seqs=8, max_pages_per_seq=8, seed=2)
    assert bm.highest_active() == 0
    slots = [bm.admit(i, 4) for i in range(5)]
    assert slots == [0, 1, 2, 3, 4] and bm.highest_active() == 5
    bm.release(1)
    bm.release(3)
    assert bm.highest_active() == 5
    assert bm.admit("new", 4) == 1             # the lowest hole, not the last released
    bm.release(4)
    assert bm.highest_active() == 3            # slots 0, 1, 2 remain
    # Every listed row sits at a page boundary (4 tokens): each takes one page, in row
    # order, from the free list's end.
    rows = np.array([0, 1, 2, 3], np.int64)
    rows = rows[bm.active[rows]]
    expect = [bm._free_pages[-1 - i] for i in range(len(rows))]
    out = bm.append_token(rows)
    assert [bm.pages[int(r)][-1] for r in rows] == expect
    np.testing.assert_array_equal(out, np.array(expect, np.int64) * 4)
    np.testing.assert_array_equal(bm.lengths[rows], 5)
