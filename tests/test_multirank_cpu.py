"""Multi-rank host logic on CPU with gloo (world size 2): the KV-page partition of a
long sequence, the packed-partial all-gather and the (out, lse) combine, checked
against single-pass attention from the CPU oracle."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import attention as oatt
from shellsmith_b200.longctx import PageRanges

P = 16


def test_page_ranges_cover_every_page_once():
    for total, world in [(0, 1), (1, 4), (7, 2), (8192, 8), (8193, 8), (100, 3)]:
        pr = PageRanges(total, world)
        seen = []
        for r in range(world):
            a, b = pr.range_of(r)
            assert 0 <= a <= b <= total
            seen.extend(range(a, b))
            for p in range(a, b):
                assert pr.owner(p) == r
        assert seen == list(range(total))
        sizes = [pr.range_of(r)[1] - pr.range_of(r)[0] for r in range(world)]
        assert max(sizes) - min(sizes) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, tokens, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(0)  # every rank builds the same sequence
        hq, hkv, d = 4, 2, 32
        q = rng.standard_normal((hq, d))
        k = rng.standard_normal((tokens, hkv, d))
        v = rng.standard_normal((tokens, hkv, d))
        pr = PageRanges(-(-tokens // P), world)
        a, b = pr.range_of(rank)
        lo, hi = a * P, min(b * P, tokens)
        o, lse = oatt.decode_attention(q, k[lo:hi], v[lo:hi], 0.2)
        packed = torch.from_numpy(np.concatenate([o, lse[:, None]], axis=1).astype(np.float64))
        parts = [torch.empty_like(packed) for _ in range(world)]
        dist.all_gather(parts, packed)
        gathered = torch.stack(parts).numpy()
        out, out_lse = oatt.combine(gathered[:, :, :d].transpose(1, 0, 2),
                                    gathered[:, :, d].T)
        want, want_lse = oatt.decode_attention(q, k, v, 0.2)
        results[rank] = (float(np.abs(out - want).max()), float(np.abs(out_lse - want_lse).max()))
        # The bench's max-over-ranks / sum-over-ranks reductions.
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        s = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(s, op=dist.ReduceOp.SUM)
        assert t.item() == world and s.item() == world * (world + 1) / 2
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens", [1, 40, 1000])
def test_kv_sharded_attention_two_gloo_ranks(tokens):
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        results = manager.dict()
        procs = [ctx.Process(target=_worker, args=(r, world, _free_port_for(tokens),
                                                   tokens, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        for r in range(world):
            err, lse_err = results[r]
            assert err < 1e-12 and lse_err < 1e-12


_PORTS = {}


def _free_port_for(key):
    if key not in _PORTS:
        _PORTS[key] = _free_port()
    return _PORTS[key]
