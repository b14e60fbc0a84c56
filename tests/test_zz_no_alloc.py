"""sc_paged_decode_attention_noalloc against sc_paged_decode_attention, through the C ABI.

Some callers of this library cannot allocate device memory when they call
it: a plain C / FFI host without a device allocator of its own, a process
whose device memory belongs to another framework's caching allocator, or a
decode loop that must not synchronise the device (cudaFree does) or run out
of memory mid-step. For them the no-allocation entry point keeps the split-K
partials in a fixed 32 MiB array inside the library instead of caller scratch.

This file is collected last on purpose (its name sorts last), so a run that
stops at the first failure has already run every other test. It passes both
alone in a fresh process and after the other tests.
"""

import math

import numpy as np
import pytest
import torch

from shellsmith_b200 import _build, _capi, paged
from shellsmith_b200._torch import ptr, stream_of

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3
SCRATCH_FLOATS = 8388608  # SC_NOALLOC_SCRATCH_FLOATS in include/shellcache.h


def _case(rng, cuda, lengths, hq=16, hkv=2, D=256, num_pages=600):
    P = paged.PAGE_SIZE
    need = [math.ceil(L / P) for L in lengths]
    width = max(need)
    perm = rng.permutation(num_pages)
    table = np.zeros((len(lengths), width), np.int32)
    cursor = 0
    for b, n in enumerate(need):
        table[b, :n] = perm[cursor:cursor + n]
        cursor += n
    gen = torch.Generator(device=cuda)
    gen.manual_seed(int(rng.integers(1 << 31)))
    pool = torch.randn((num_pages, hkv, 2, P, D), generator=gen, device=cuda).to(torch.bfloat16)
    q = torch.randn((len(lengths), hq, D), generator=gen, device=cuda).to(torch.bfloat16)
    return (pool, q, torch.from_numpy(table).to(cuda),
            torch.tensor(lengths, dtype=torch.int32, device=cuda), width)


def _regular(pool, q, table, ctx, width, pps, nsplit):
    B, hq, D = q.shape
    part_out = torch.empty((B, hq, nsplit, D), dtype=torch.float32, device=q.device)
    part_lse = torch.empty((B, hq, nsplit), dtype=torch.float32, device=q.device)
    out = torch.empty((B, hq, D), dtype=torch.bfloat16, device=q.device)
    lse = torch.empty((B * hq,), dtype=torch.float32, device=q.device)
    _capi.call("sc_paged_decode_attention", ptr(q), ptr(pool), pool.shape[0], ptr(table),
               ptr(ctx), None, B, hq, pool.shape[1], D, pool.shape[3], width, pps, nsplit, 1.0 / 16,
               ptr(part_out), ptr(part_lse), ptr(out), ptr(lse), stream_of(q))
    return out, lse


def _noalloc(pool, q, table, ctx, width, pps, nsplit, with_lse=True):
    B, hq, D = q.shape
    out = torch.empty((B, hq, D), dtype=torch.bfloat16, device=q.device)
    lse = torch.empty((B * hq,), dtype=torch.float32, device=q.device) if with_lse else None
    _capi.call("sc_paged_decode_attention_noalloc", ptr(q), ptr(pool), pool.shape[0], ptr(table),
               ptr(ctx), B, hq, pool.shape[1], D, pool.shape[3], width, pps, nsplit, 1.0 / 16,
               ptr(out), ptr(lse), stream_of(q))
    return out, lse


def test_noalloc_matches_caller_scratch_on_two_calls_in_a_row(cuda):
    _build.build()
    rng = np.random.default_rng(21)
    # The second call runs over the first call's leftover partials, with a
    # different batch, lengths and split count.
    for lengths, pps in (([1, 300, 1000, 2500, 33], 8), ([700, 17, 3000, 64, 5, 1600, 16], 5)):
        pool, q, table, ctx, width = _case(rng, cuda, lengths)
        nsplit = math.ceil(width / pps)
        want, want_lse = _regular(pool, q, table, ctx, width, pps, nsplit)
        got, got_lse = _noalloc(pool, q, table, ctx, width, pps, nsplit)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.float().cpu().numpy(), want.float().cpu().numpy(),
                                   rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(got_lse.cpu().numpy(), want_lse.cpu().numpy(), rtol=1e-5,
                                   atol=1e-5)
    _capi.check_device()


def test_noalloc_single_split_and_no_lse_match_caller_scratch(cuda):
    """One split (the kernel writes the output itself and the built-in array is not
    touched) and a call without lse_out, each against the caller-scratch path."""
    _build.build()
    rng = np.random.default_rng(23)
    lengths = [1, 300, 1000, 2500, 33]
    pool, q, table, ctx, width = _case(rng, cuda, lengths)
    for pps, with_lse in ((width, True), (width + 7, False), (8, False)):
        nsplit = math.ceil(width / pps)
        want, want_lse = _regular(pool, q, table, ctx, width, pps, nsplit)
        got, got_lse = _noalloc(pool, q, table, ctx, width, pps, nsplit, with_lse=with_lse)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.float().cpu().numpy(), want.float().cpu().numpy(),
                                   rtol=RTOL, atol=ATOL)
        if with_lse:
            np.testing.assert_allclose(got_lse.cpu().numpy(), want_lse.cpu().numpy(),
                                       rtol=1e-5, atol=1e-5)
    _capi.check_device()


def test_noalloc_rejects_batches_beyond_its_scratch(cuda):
    _build.build()
    rng = np.random.default_rng(22)
    pool, q, table, ctx, width = _case(rng, cuda, [40, 50])
    B, hq, D = q.shape
    nsplit = SCRATCH_FLOATS // (B * hq * (D + 1)) + 1
    out = torch.empty((B, hq, D), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(_capi.ShellcacheError) as info:
        _capi.call("sc_paged_decode_attention_noalloc", ptr(q), ptr(pool), pool.shape[0],
                   ptr(table), ptr(ctx), B, hq, pool.shape[1], D, pool.shape[3], width, 1, nsplit,
                   1.0 / 16, ptr(out), ptr(None), stream_of(q))
    assert info.value.code == 1 and "exceeds the built-in scratch" in str(info.value)
