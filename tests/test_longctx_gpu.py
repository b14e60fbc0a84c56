"""KV-page-sharded decode of one long sequence (the config-4 path) on the GPU.

Single-GPU: W ranks are emulated as W ShardedSequence objects on one device
(each with its own pool); their packed partials are stacked as the all-gather
would and merged with sc_attention_combine_packed. Two GPUs (when present):
two processes, NCCL all-gather, and the NVLink peer exchange (put + epoch
flags) over two layers and two tokens, which must give bit-identical outputs
to the NCCL path. All are checked against the CPU oracle on the whole
sequence, rtol 2e-2 / atol 2e-3.
"""

import math
import os
import socket

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from shellsmith_b200 import paged
from shellsmith_b200.longctx import ShardedSequence

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3
HQ, HKV, D = 16, 2, 256


def _sequence(tokens, seed=4):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn((tokens + 1, HKV, D), generator=g).to(torch.bfloat16)
    v = torch.randn((tokens + 1, HKV, D), generator=g).to(torch.bfloat16)
    q = torch.randn((1, HQ, D), generator=g).to(torch.bfloat16)
    return q, k, v


def _fill(shard, k, v, layer=0):
    """Write this rank's share of the prompt (tokens [first*P, first*P + local)) into its pool."""
    lo = shard.first_page * paged.PAGE_SIZE
    n = shard.local_tokens
    if n:
        slots = torch.arange(n, dtype=torch.int64, device="cuda")
        paged.kv_append(k[lo:lo + n].cuda(), v[lo:lo + n].cuda(), shard.kv[layer], slots)


@pytest.mark.parametrize("world,tokens", [(1, 100), (3, 1000), (4, 5000), (8, 2049)])
def test_emulated_ranks_match_single_pass(cuda, world, tokens):
    q, k, v = _sequence(tokens)
    shards = [ShardedSequence(tokens, r, world, attention_layers=1, kv_heads=HKV, head_dim=D,
                              q_heads=HQ) for r in range(world)]
    for s in shards:
        _fill(s, k, v)
    # Decode one token: the tail rank appends k/v[tokens]; every rank attends.
    packed = []
    for s in shards:
        s.begin_token()
        pool = s.kv[0]
        paged.kv_append(k[tokens:tokens + 1].cuda(), v[tokens:tokens + 1].cuda(), pool, s.slot)
        pages = max(1, math.ceil(s.local_tokens / paged.PAGE_SIZE))
        packed.append(paged.paged_decode_attention_packed(q.cuda(), pool, s.table, s.ctx,
                                                          1 / 16, max_pages_in_batch=pages,
                                                          total_pages=pages).clone())
    out, lse = paged.attention_combine_packed(torch.stack(packed))
    want, want_lse = oatt.decode_attention(q[0].float().numpy(), k.float().numpy(),
                                           v.float().numpy(), 1 / 16)
    np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(lse.cpu().numpy(), want_lse, atol=1e-3)


def test_packed_partial_matches_bf16_entry(cuda):
    """The packed fp32 output equals the regular entry's output (before bf16 rounding)."""
    rng = np.random.default_rng(1)
    B, pages = 3, 40
    pool = torch.randn((pages * B, HKV, 2, 16, D), device=cuda).to(torch.bfloat16)
    table = torch.from_numpy(rng.permutation(pages * B).reshape(B, pages).astype(np.int32)).cuda()
    ctx = torch.tensor([1, 300, 640], dtype=torch.int32, device=cuda)
    q = torch.randn((B, HQ, D), device=cuda).to(torch.bfloat16)
    for pps in (4, 64):
        lse = torch.empty(B * HQ, dtype=torch.float32, device=cuda)
        out = paged.paged_decode_attention(q, pool, table, ctx, 0.07, pages_per_split=pps,
                                           lse_out=lse)
        packed = paged.paged_decode_attention_packed(q, pool, table, ctx, 0.07,
                                                     pages_per_split=pps)
        np.testing.assert_allclose(packed[:, :D].cpu().numpy(),
                                   out.view(B * HQ, D).float().cpu().numpy(), rtol=1e-2,
                                   atol=1e-2)
        np.testing.assert_allclose(packed[:, D].cpu().numpy(), lse.cpu().numpy(), rtol=1e-6,
                                   atol=1e-6)


def _nccl_worker(rank, world, port, tokens, result):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    try:
        q, k, v = _sequence(tokens)
        s = ShardedSequence(tokens, rank, world, attention_layers=1, kv_heads=HKV, head_dim=D,
                            q_heads=HQ, device=f"cuda:{rank}")
        lo = s.first_page * paged.PAGE_SIZE
        if s.local_tokens:
            slots = torch.arange(s.local_tokens, dtype=torch.int64, device=f"cuda:{rank}")
            paged.kv_append(k[lo:lo + s.local_tokens].cuda(), v[lo:lo + s.local_tokens].cuda(),
                            s.kv[0], slots)
        s.begin_token()
        out = s.attention(0, q.cuda(), k[tokens:tokens + 1].cuda(), v[tokens:tokens + 1].cuda(),
                          1 / 16)
        torch.cuda.synchronize()
        result[rank] = out.float().cpu().numpy()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpus_nccl_all_gather():
    import torch.multiprocessing as mp

    tokens = 10000
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        result = manager.dict()
        procs = [ctx.Process(target=_nccl_worker, args=(r, 2, port, tokens, result))
                 for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            assert p.exitcode == 0
        q, k, v = _sequence(tokens)
        want, _ = oatt.decode_attention(q[0].float().numpy(), k.float().numpy(),
                                        v.float().numpy(), 1 / 16)
        for r in range(2):
            np.testing.assert_allclose(result[r], want, rtol=RTOL, atol=ATOL)


def _p2p_worker(rank, world, port, tokens, result):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            device_id=torch.device("cuda", rank))
    dev = f"cuda:{rank}"
    try:
        q, k, v = _sequence(tokens + 1)
        shards = {}
        for mode in ("nccl", "p2p", "fused"):
            s = ShardedSequence(tokens, rank, world, attention_layers=2, kv_heads=HKV,
                                head_dim=D, q_heads=HQ, device=dev)
            lo = s.first_page * paged.PAGE_SIZE
            if s.local_tokens:
                slots = torch.arange(s.local_tokens, dtype=torch.int64, device=dev)
                for layer in range(2):
                    paged.kv_append(k[lo:lo + s.local_tokens].to(dev),
                                    v[lo:lo + s.local_tokens].to(dev), s.kv[layer], slots)
            if mode != "nccl":
                s.enable_peer_exchange(fused=mode == "fused")
            shards[mode] = s
        outs = {"nccl": [], "p2p": [], "fused": []}
        for step in range(2):
            t = tokens + step
            for mode, s in shards.items():
                s.begin_token()
                for layer in range(2):
                    out = s.attention(layer, q.to(dev), k[t:t + 1].to(dev), v[t:t + 1].to(dev),
                                      1 / 16)
                    outs[mode].append(out.float().cpu().numpy())
        torch.cuda.synchronize()
        from shellsmith_b200 import _capi

        _capi.check_device()
        result[rank] = outs
        dist.barrier()
        shards["p2p"].close()
        shards["fused"].close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_gpus_peer_exchange_matches_nccl():
    import torch.multiprocessing as mp

    tokens = 10000
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        port = sock.getsockname()[1]
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        result = manager.dict()
        procs = [ctx.Process(target=_p2p_worker, args=(r, 2, port, tokens, result))
                 for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(300)
            assert p.exitcode == 0
        q, k, v = _sequence(tokens + 1)
        for r in range(2):
            outs = result[r]
            for mode in ("p2p", "fused"):
                for i, (a, b) in enumerate(zip(outs["nccl"], outs[mode])):
                    assert np.array_equal(a, b), (r, mode, i)
            for step in range(2):
                n = tokens + 1 + step
                want, _ = oatt.decode_attention(q[0].float().numpy(), k[:n].float().numpy(),
                                                v[:n].float().numpy(), 1 / 16)
                for layer in range(2):
                    np.testing.assert_allclose(outs["p2p"][2 * step + layer], want, rtol=RTOL,
                                               atol=ATOL)


@pytest.mark.parametrize("fused", [False, True])
def test_peer_exchange_single_rank_matches_local_path(cuda, fused):
    """World 1: the put/flag/wait kernels (separate, or folded into the attention merge
    and the final merge) run against this GPU's own buffer."""
    tokens = 3000
    q, k, v = _sequence(tokens + 1)
    shards = []
    for use_peer in (False, True):
        s = ShardedSequence(tokens, 0, 1, attention_layers=2, kv_heads=HKV, head_dim=D,
                            q_heads=HQ)
        for layer in range(2):
            _fill(s, k, v, layer)
        if use_peer:
            s.enable_peer_exchange(fused=fused)
        shards.append(s)

    def gather(dst, src):
        dst[0].copy_(src)

    for step in range(2):
        t = tokens + step
        for s in shards:
            s.begin_token()
        for layer in range(2):
            a = shards[0].attention(layer, q.cuda(), k[t:t + 1].cuda(), v[t:t + 1].cuda(), 1 / 16,
                                    all_gather=gather).clone()
            b = shards[1].attention(layer, q.cuda(), k[t:t + 1].cuda(), v[t:t + 1].cuda(), 1 / 16)
            torch.cuda.synchronize()
            assert torch.equal(a, b)
    from shellsmith_b200 import _capi

    _capi.check_device()
    shards[1].close()


def test_single_rank_direct_path_matches_packed_path(cuda):
    """World 1 without an all-gather: the split merge writes the final rows, equal bit for
    bit to the packed partial merged as one part."""
    tokens = 3000
    q, k, v = _sequence(tokens + 1)
    shards = []
    for _ in range(2):
        s = ShardedSequence(tokens, 0, 1, attention_layers=2, kv_heads=HKV, head_dim=D,
                            q_heads=HQ)
        for layer in range(2):
            _fill(s, k, v, layer)
        shards.append(s)

    def gather(dst, src):
        dst[0].copy_(src)

    for step in range(2):
        t = tokens + step
        for s in shards:
            s.begin_token()
        for layer in range(2):
            a = shards[0].attention(layer, q.cuda(), k[t:t + 1].cuda(), v[t:t + 1].cuda(), 1 / 16,
                                    all_gather=gather).clone()
            b = shards[1].attention(layer, q.cuda(), k[t:t + 1].cuda(), v[t:t + 1].cuda(), 1 / 16)
            torch.cuda.synchronize()
            assert torch.equal(a, b)
    from shellsmith_b200 import _capi

    _capi.check_device()


@pytest.mark.parametrize("world", [1, 2])
def test_config4_full_context(cuda, world):
    """Config 4 at full size: one 131,072-token sequence (then one decode token) with the
    one-wave split, on one GPU or emulated as two ranks on this GPU merged as the
    exchange would; the whole context against the float64 oracle."""
    tokens = 131_072
    q, k, v = _sequence(tokens + 1, seed=40)
    shards = [ShardedSequence(tokens, r, world, attention_layers=1, kv_heads=HKV, head_dim=D,
                              q_heads=HQ, headroom_pages=8) for r in range(world)]
    for s in shards:
        _fill(s, k, v)
        s.begin_token()
    t = tokens
    if world == 1:
        out = shards[0].attention(0, q.cuda(), k[t:t + 1].cuda(), v[t:t + 1].cuda(), 1 / 16)
    else:
        parts = []
        for s in shards:
            def keep(dst, src):
                parts.append(src.clone())
            s.attention(0, q.cuda(), k[t:t + 1].cuda(), v[t:t + 1].cuda(), 1 / 16,
                        all_gather=keep)
        out, _ = paged.attention_combine_packed(torch.stack(parts))
    torch.cuda.synchronize()
    want, _ = oatt.decode_attention(q[0].float().numpy(), k[:t + 1].float().numpy(),
                                    v[:t + 1].float().numpy(), 1 / 16)
    np.testing.assert_allclose(out.float().cpu().numpy().reshape(HQ, D), want, rtol=RTOL,
                               atol=ATOL)
    from shellsmith_b200 import _capi

    _capi.check_device()


def test_exchange_wait_times_out_and_the_context_stays_usable(cuda):
    """A wait on a flag that nothing raises gives up after its poll limit: the kernel
    returns, the device status word carries the time-out (DeviceFault on the host), and a
    later wait whose flag is raised completes normally."""
    from shellsmith_b200 import _capi
    from shellsmith_b200._torch import ptr, stream_of

    _capi.check_device()
    flags = torch.zeros(1, dtype=torch.int32, device=cuda)
    epoch = torch.zeros(1, dtype=torch.int32, device=cuda)
    _capi.call("sc_exchange_wait_limited", ptr(flags), 1, ptr(epoch), 7, 4096, stream_of(flags))
    torch.cuda.synchronize()
    with pytest.raises(_capi.DeviceFault, match="bounded wait"):
        _capi.check_device()
    flags.fill_(7)
    _capi.call("sc_exchange_wait_limited", ptr(flags), 1, ptr(epoch), 7, 4096, stream_of(flags))
    torch.cuda.synchronize()
    _capi.check_device()
