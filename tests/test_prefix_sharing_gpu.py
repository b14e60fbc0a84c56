"""Paged prefix sharing on the GPU: snapshots share full pages, forks copy the
partial last page and the GDN state rows, and a forked prompt continues to the
same cache as a prompt prefilled in one go.

Bars: K/V of shared and copied pages bit-exact; decode attention of a fork vs
the one-go sequence bit-exact (same K/V, same split plan); GDN state after a
fork + continuation within 1e-4 of the one-go state (chunk boundaries differ,
fp32 accumulation order changes); page reference counts exact, and every page
returns to the free list when the last owner lets go.
"""

import numpy as np
import pytest
import torch

from shellsmith_b200 import paged
from shellsmith_b200.engine import HybridCacheEngine, HybridConfig
from shellsmith_b200.runtime import PagedSequence, paged_prefix_cache
from shellsmith_b200.workloads import gdn_sequence_inputs, to_device

pytestmark = pytest.mark.gpu

PROMPT, CUT = 50, 37          # the snapshot covers 37 tokens: 2 full pages + 5 tokens


def _cfg():
    return HybridConfig(layers=8, gdn_key_heads=2, gdn_value_heads=4, q_heads=8, kv_heads=2,
                        head_dim=128, max_seqs=8, num_pages=64, max_context=512,
                        snapshot_rows=4)


def _inputs(cfg, cuda, seed=5):
    """Per-layer inputs for PROMPT tokens: GDN (q, k, v, decay, beta), attention (k, v)."""
    rng = np.random.default_rng(seed)
    gdn, kv = {}, {}
    for layer in range(cfg.layers):
        if cfg.is_attention(layer):
            k = torch.randn((PROMPT, cfg.kv_heads, cfg.head_dim), device=cuda).to(torch.bfloat16)
            v = torch.randn((PROMPT, cfg.kv_heads, cfg.head_dim), device=cuda).to(torch.bfloat16)
            kv[layer] = (k, v)
        else:
            q, k, v, g, b = gdn_sequence_inputs(rng, 1, PROMPT, cfg.gdn_key_heads,
                                                cfg.gdn_value_heads, cfg.key_dim, cfg.value_dim)
            qd, kd, vd = to_device(q[0], k[0], v[0], device=cuda)
            gd, bd = to_device(g[0], b[0], dtype=torch.float32, device=cuda)
            gdn[layer] = (qd, kd, vd, gd, bd)
    return gdn, kv


def _prefill(eng, new, gdn, kv, start, stop):
    eng.prefill(new, lambda l, n: tuple(t[start:stop] for t in gdn[l]),
                lambda l, n: tuple(t[start:stop] for t in kv[l]))


def _kv_of(eng, slot, layer, tokens):
    slots = torch.from_numpy(eng.blocks.prompt_slots(slot, 0, tokens)).to(eng.device)
    return paged.kv_gather(eng.kv[eng.attn_index[layer]], slots)


def _attention(eng, rows, cuda):
    """Decode attention of the listed rows at their current length (no append)."""
    cfg = eng.cfg
    table = torch.from_numpy(eng.blocks.table[rows]).to(cuda)
    ctx = torch.from_numpy(eng.blocks.lengths[rows].astype(np.int32)).to(cuda)
    gen = torch.Generator(device=cuda).manual_seed(3)
    q = torch.randn((1, cfg.q_heads, cfg.head_dim), generator=gen, device=cuda)
    q = q.to(torch.bfloat16).expand(len(rows), -1, -1).contiguous()
    layer = cfg.attention_layers[-1]
    return paged.paged_decode_attention(q, eng.kv[eng.attn_index[layer]], table, ctx,
                                        eng.scale, pages_per_split=2)


def test_snapshot_fork_continue_matches_one_go_prefill(cuda):
    cfg = _cfg()
    eng = HybridCacheEngine(cfg, device=cuda)
    gdn, kv = _inputs(cfg, cuda)
    free0 = eng.blocks.free_pages

    # Sequence A: the first CUT tokens, then a snapshot.
    a = eng.admit("A", CUT)
    _prefill(eng, [(a, CUT)], gdn, kv, 0, CUT)
    a_pages = list(eng.blocks.pages[a])
    snap = eng.snapshot(a)
    rc = eng.blocks.refcount
    assert list(rc[a_pages[:2]]) == [2, 2] and rc[a_pages[2]] == 1
    assert snap.pages[:2] == a_pages[:2] and snap.pages[2] != a_pages[2]
    assert rc[snap.pages[2]] == 1 and snap.tokens == CUT

    # A keeps writing its own partial page; the snapshot must not see it.
    junk = torch.full((1, cfg.kv_heads, cfg.head_dim), 7.0, device=cuda).to(torch.bfloat16)
    eng.extend(a, CUT + 1)
    for layer in cfg.attention_layers:
        eng.write_prompt_kv(a, layer, junk, junk, start=CUT)
    torch.cuda.synchronize()

    # Fork the snapshot and continue the prompt to PROMPT tokens.
    f = eng.fork(snap, owner="F")
    assert eng.blocks.pages[f][:2] == a_pages[:2]
    assert list(eng.blocks.refcount[a_pages[:2]]) == [3, 3]
    assert eng.blocks.pages[f][2] not in (a_pages[2], snap.pages[2])
    eng.extend(f, PROMPT)
    _prefill(eng, [(f, CUT, PROMPT)], gdn, kv, CUT, PROMPT)

    # Sequence R: the whole prompt in one go.
    r = eng.admit("R", PROMPT)
    _prefill(eng, [(r, PROMPT)], gdn, kv, 0, PROMPT)
    torch.cuda.synchronize()

    for layer in cfg.attention_layers:
        kf, vf = _kv_of(eng, f, layer, PROMPT)
        kr, vr = _kv_of(eng, r, layer, PROMPT)
        assert torch.equal(kf, kr) and torch.equal(vf, vr)
        ks, vs = paged.kv_gather(eng.kv[eng.attn_index[layer]], torch.from_numpy(
            (np.asarray(snap.pages, np.int64)[np.arange(CUT) // cfg.page_size] * cfg.page_size
             + np.arange(CUT) % cfg.page_size)).to(cuda))
        assert torch.equal(ks, kr[:CUT]) and torch.equal(vs, vr[:CUT])
    out = _attention(eng, [f, r], cuda)
    assert torch.equal(out[0], out[1])
    gap = (eng.state[:, f] - eng.state[:, r]).abs().max().item()
    assert gap <= 1e-4, gap
    assert torch.isfinite(eng.state[:, f]).all()

    # Release everything: every page comes back exactly once.
    for slot in (a, f, r):
        eng.release(slot)
    assert eng.blocks.free_pages == free0 - len(snap.pages)
    eng.drop_snapshot(snap)
    assert eng.blocks.free_pages == free0 and not eng.blocks.refcount.any()


def test_prefix_cache_over_paged_snapshots(cuda):
    """PrefixCache with paged storage hooks: put snapshots, fork on get, evict drops."""
    cfg = _cfg()
    eng = HybridCacheEngine(cfg, device=cuda)
    gdn, kv = _inputs(cfg, cuda, seed=9)
    free0 = eng.blocks.free_pages
    one = eng.cache_bytes(CUT)
    prefixes = paged_prefix_cache(eng, limit_bytes=one + one // 2)
    tokens = list(range(PROMPT))

    a = eng.admit("A", CUT)
    _prefill(eng, [(a, CUT)], gdn, kv, 0, CUT)
    prefixes.put("id", "p", "bf16", tokens[:CUT], PagedSequence(eng, a), logits=None)
    assert prefixes.metrics()["stored"] == 1 and prefixes.bytes == one
    seq_a = PagedSequence(eng, a)
    seq_a.clear()
    seq_a.clear()

    hit = prefixes.get("id", "p", "bf16", tokens, fork=True)
    assert hit is not None and hit[2] == CUT
    fork = hit[0]
    assert isinstance(fork, PagedSequence) and fork.tokens == CUT
    eng.extend(fork.slot, PROMPT)
    _prefill(eng, [(fork.slot, CUT, PROMPT)], gdn, kv, CUT, PROMPT)
    r = eng.admit("R", PROMPT)
    _prefill(eng, [(r, PROMPT)], gdn, kv, 0, PROMPT)
    torch.cuda.synchronize()
    for layer in cfg.attention_layers:
        assert all(torch.equal(x, y) for x, y in zip(_kv_of(eng, fork.slot, layer, PROMPT),
                                                     _kv_of(eng, r, layer, PROMPT)))

    # A second, longer prefix pushes the first out (limit holds one and a half).
    prefixes.put("id", "p", "bf16", tokens, PagedSequence(eng, r), logits=None)
    assert prefixes.metrics()["evictions"] == 1 and len(prefixes.entries) == 1
    fork.clear()
    eng.release(r)
    prefixes.clear()
    assert eng.blocks.free_pages == free0 and not eng.blocks.refcount.any()
