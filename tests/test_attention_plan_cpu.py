"""The attention layer's launch choice (no GPU): paged.append_and_attend folds the append
into the split-K launch exactly when the plan gives every sequence one split, and runs the
append, the split-K kernel and the merge otherwise; the launch counter follows."""

import torch

from shellsmith_b200 import paged


def _record(monkeypatch):
    calls = []
    monkeypatch.setattr(paged, "require_cuda", lambda *a, **k: None)
    monkeypatch.setattr(paged, "ptr", lambda t: 0)
    monkeypatch.setattr(paged, "stream_of", lambda t: 0)
    monkeypatch.setattr(paged, "sm_count", lambda device: 148)
    monkeypatch.setattr(paged._capi, "call", lambda name, *args: calls.append((name, args)))
    return calls


def _operands(B, pages, width):
    q = torch.zeros((B, 16, 256), dtype=torch.bfloat16)
    kn = torch.zeros((B, 2, 256), dtype=torch.bfloat16)
    pool = torch.zeros((pages, 2, 2, 16, 256), dtype=torch.bfloat16)
    table = torch.zeros((B, width), dtype=torch.int32)
    ctx = torch.zeros((B,), dtype=torch.int32)
    slots = torch.zeros((B,), dtype=torch.int64)
    return q, kn, pool, table, ctx, slots


def test_one_split_per_sequence_takes_the_fused_launch(monkeypatch):
    calls = _record(monkeypatch)
    q, kn, pool, table, ctx, slots = _operands(256, 4096, 1025)
    before = paged.attention_launches
    # Config 3's batch: 256 sequences, ~115k pages; the plan picks 1,024-page splits.
    paged.append_and_attend(q, kn, kn, slots, pool, table, ctx, 0.0625,
                            max_pages_in_batch=1000, total_pages=115_000)
    assert [c[0] for c in calls] == ["sc_paged_decode_attention_fused"]
    assert calls[0][1][16] == 1                      # num_splits
    assert paged.attention_launches - before == 1


def test_several_splits_take_append_split_and_merge(monkeypatch):
    calls = _record(monkeypatch)
    q, kn, pool, table, ctx, slots = _operands(8, 4096, 2100)
    before = paged.attention_launches
    # A config-2 share at 8 GPUs: 8 long sequences, splits of 128 pages.
    paged.append_and_attend(q, kn, kn, slots, pool, table, ctx, 0.0625,
                            max_pages_in_batch=2048, total_pages=8_000)
    assert [c[0] for c in calls] == ["sc_kv_append", "sc_paged_decode_attention"]
    assert calls[1][1][13] > 1                       # num_splits: the merge follows
    assert paged.attention_launches - before == 3


def test_eight_bit_pools_keep_their_own_kernels(monkeypatch):
    calls = _record(monkeypatch)
    q, kn, _, table, ctx, slots = _operands(4, 64, 8)
    pool8 = torch.zeros((64, 2, 34 * 256), dtype=torch.uint8)
    paged.append_and_attend(q, kn, kn, slots, pool8, table, ctx, 0.0625, pages_per_split=8)
    assert [c[0] for c in calls] == ["sc_kv_append_q8", "sc_paged_decode_attention_q8"]
