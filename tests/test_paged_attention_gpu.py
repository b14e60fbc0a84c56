"""K4 paged KV append and K7 split-K decode attention on the GPU vs the CPU oracle.

Bars: the pool layout and append/gather round trip are bit-exact; attention
outputs are within rtol 2e-2 / atol 2e-3 of float64 `numpy_attention` math
(restated in oracle.attention), lse within 1e-3.
"""

import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from shellsmith_b200 import paged

pytestmark = pytest.mark.gpu

# The kernel feeds the probabilities to the P.V product in bf16 (relative rounding
# 2^-9), so an output's error has a standard deviation near 2^-9 / sqrt(3) * ||p||_2:
# up to ~5e-4 for the short contexts below (||p||_2 ~ 0.5). ATOL is ~6 of those.
RTOL, ATOL = 2e-2, 3e-3


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def test_append_layout_bit_exact_and_gather_roundtrip(cuda):
    rng = np.random.default_rng(3)
    num_pages, hkv, P, D = 11, 2, 16, 256
    pool = torch.zeros((num_pages, hkv, 2, P, D), dtype=torch.bfloat16, device=cuda)
    ntok = 40
    slots = rng.permutation(num_pages * P)[:ntok].astype(np.int64)
    slots[5] = -1
    k = torch.randn((ntok, hkv, D), device=cuda).to(torch.bfloat16)
    v = torch.randn((ntok, hkv, D), device=cuda).to(torch.bfloat16)
    slot_t = torch.from_numpy(slots).to(cuda)
    paged.kv_append(k, v, pool, slot_t)
    # Layout: the oracle's scatter of the same bits must produce the same pool.
    want = np.zeros(pool.numel(), np.uint16)
    oatt.pool_write(want, slots, _bits(k), _bits(v), hkv, P, D)
    assert np.array_equal(_bits(pool).reshape(-1), want)
    kg, vg = paged.kv_gather(pool, slot_t)
    keep = slots >= 0
    assert torch.equal(kg[keep], k[keep]) and torch.equal(vg[keep], v[keep])
    assert torch.count_nonzero(kg[~keep]) == 0
    # Copy-on-write pages.
    src = torch.tensor([1, 4], dtype=torch.int32, device=cuda)
    dst = torch.tensor([9, 0], dtype=torch.int32, device=cuda)
    before = pool.clone()
    paged.kv_copy_pages(pool, src, dst)
    assert torch.equal(pool[9], before[1]) and torch.equal(pool[0], before[4])
    assert torch.equal(pool[2:9], before[2:9])


def _build_case(rng, lengths, hq, hkv, D, num_pages, cuda, pages_per_seq=None):
    """Random pool contents and block tables for the given context lengths."""
    P = paged.PAGE_SIZE
    need = [math.ceil(L / P) for L in lengths]
    width = pages_per_seq or max(1, max(need))
    perm = rng.permutation(num_pages)
    assert sum(need) <= num_pages
    table = np.zeros((len(lengths), width), np.int32)
    cursor = 0
    for b, n in enumerate(need):
        table[b, :n] = perm[cursor:cursor + n]
        cursor += n
    pool = torch.randn((num_pages, hkv, 2, P, D), device=cuda).to(torch.bfloat16)
    q = torch.randn((len(lengths), hq, D), device=cuda).to(torch.bfloat16)
    return pool, q, table


def _oracle(pool_np, q_np, table, lengths, hkv, D, scale):
    outs, lses = [], []
    for b, L in enumerate(lengths):
        k, v = oatt.pool_read_pages(pool_np, table[b], L, hkv, paged.PAGE_SIZE, D)
        o, l = oatt.decode_attention(q_np[b], k, v, scale)
        outs.append(o)
        lses.append(l)
    return np.stack(outs), np.stack(lses)


@pytest.mark.parametrize("hq,hkv,D", [(16, 2, 256), (24, 4, 256), (24, 2, 256), (8, 8, 128),
                                      (4, 1, 64)])
@pytest.mark.parametrize("pages_per_split", [1, 3, 64])
def test_decode_attention_matches_oracle(cuda, hq, hkv, D, pages_per_split):
    rng = np.random.default_rng(hq * 100 + hkv * 10 + D + pages_per_split)
    lengths = [1, 15, 16, 17, 33, 200, 517, 64]
    pool, q, table = _build_case(rng, lengths, hq, hkv, D, 160, cuda, pages_per_seq=40)
    scale = 1.0 / math.sqrt(D)
    ctx = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    lse = torch.empty(len(lengths) * hq, dtype=torch.float32, device=cuda)
    out = paged.paged_decode_attention(q, pool, torch.from_numpy(table).to(cuda), ctx, scale,
                                       pages_per_split=pages_per_split, lse_out=lse)
    want, want_lse = _oracle(pool.float().cpu().numpy(), q.float().cpu().numpy(), table, lengths,
                             hkv, D, scale)
    np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(lse.cpu().numpy().reshape(want_lse.shape), want_lse, atol=1e-3)


def test_known_answer_uniform_scores(cuda):
    """q = 0 makes every score equal: the output is the mean of the values.
    (The reference oracle's known answer: v = [1, 3, 8] seen by the last query -> 4.)"""
    P, D = paged.PAGE_SIZE, 64
    pool = torch.zeros((4, 1, 2, P, D), dtype=torch.bfloat16, device=cuda)
    k = torch.zeros((3, 1, D), dtype=torch.bfloat16, device=cuda)
    v = torch.zeros((3, 1, D), dtype=torch.bfloat16, device=cuda)
    v[:, 0, :] = torch.tensor([1.0, 3.0, 8.0], device=cuda)[:, None]
    paged.kv_append(k, v, pool, torch.tensor([32, 33, 34], dtype=torch.int64, device=cuda))
    q = torch.zeros((1, 2, D), dtype=torch.bfloat16, device=cuda)
    out = paged.paged_decode_attention(q, pool, torch.tensor([[2]], dtype=torch.int32,
                                                             device=cuda),
                                       torch.tensor([3], dtype=torch.int32, device=cuda), 1.0)
    assert torch.all(out.float() == 4.0)
    # The first two keys alone (the reference's first query row) average to 2.
    out = paged.paged_decode_attention(q, pool, torch.tensor([[2]], dtype=torch.int32,
                                                             device=cuda),
                                       torch.tensor([2], dtype=torch.int32, device=cuda), 1.0)
    assert torch.all(out.float() == 2.0)


def test_empty_sequence_gives_zero(cuda):
    pool = torch.randn((4, 2, 2, 16, 128), device=cuda).to(torch.bfloat16)
    q = torch.randn((2, 4, 128), device=cuda).to(torch.bfloat16)
    table = torch.tensor([[0, 1], [2, 3]], dtype=torch.int32, device=cuda)
    ctx = torch.tensor([0, 20], dtype=torch.int32, device=cuda)
    for pps in (1, 8):
        out = paged.paged_decode_attention(q, pool, table, ctx, 0.1, pages_per_split=pps)
        assert torch.count_nonzero(out[0]) == 0 and torch.isfinite(out[1].float()).all()


@pytest.mark.parametrize("parts", [5, 40, 1500])
def test_combine_matches_oracle(cuda, parts):
    """Few parts (per-row kernel), many parts (tiled kernel), > 1024 parts (windows)."""
    rng = np.random.default_rng(11 + parts)
    rows, D = 7, 256
    po = rng.standard_normal((rows, parts, D)).astype(np.float32)
    pl = (rng.standard_normal((rows, parts)) * 3).astype(np.float32)
    pl[2, 1] = -np.inf
    pl[4, :] = -np.inf
    out, lse = paged.attention_combine(torch.from_numpy(po).to(cuda),
                                       torch.from_numpy(pl).to(cuda))
    want, want_lse = oatt.combine(po, pl)
    np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)
    got_lse = lse.cpu().numpy()
    assert np.isneginf(got_lse[4]) and np.isneginf(want_lse[4])
    fin = np.isfinite(want_lse)
    np.testing.assert_allclose(got_lse[fin], want_lse[fin], rtol=1e-5, atol=1e-5)


def test_split_combine_algebra_matches_single_pass(cuda):
    """Splitting a long sequence into parts and combining equals one pass."""
    rng = np.random.default_rng(12)
    pool, q, table = _build_case(rng, [3000], 16, 2, 256, 200, cuda)
    ctx = torch.tensor([3000], dtype=torch.int32, device=cuda)
    bt = torch.from_numpy(table).to(cuda)
    one = paged.paged_decode_attention(q, pool, bt, ctx, 0.0625, pages_per_split=4096)
    many = paged.paged_decode_attention(q, pool, bt, ctx, 0.0625, pages_per_split=5)
    np.testing.assert_allclose(one.float().cpu().numpy(), many.float().cpu().numpy(),
                               rtol=RTOL, atol=ATOL)


def test_bad_page_index_sets_device_status(cuda):
    """An out-of-range page in a block table is reported, not dereferenced."""
    from shellsmith_b200 import _capi

    _capi.device_status()
    pool = torch.randn((4, 1, 2, 16, 64), device=cuda).to(torch.bfloat16)
    q = torch.randn((1, 2, 64), device=cuda).to(torch.bfloat16)
    table = torch.tensor([[0, 99]], dtype=torch.int32, device=cuda)
    paged.paged_decode_attention(q, pool, table, torch.tensor([20], dtype=torch.int32,
                                                              device=cuda), 0.1)
    with pytest.raises(_capi.DeviceFault):
        _capi.check_device()
    assert _capi.device_status() == 0


def test_context_beyond_its_table_row_or_its_splits_is_flagged(cuda):
    """A ctx_len whose pages exceed the block-table row, or the pages the launch's
    splits cover, or a negative ctx_len, sets the device status word; the kernel
    attends the clamped context (never past the row, never dropping pages silently)
    and the other sequences of the launch stay exact."""
    from shellsmith_b200 import _capi
    from shellsmith_b200._torch import ptr, stream_of

    rng = np.random.default_rng(31)
    hq, hkv, D, P = 16, 2, 256, paged.PAGE_SIZE
    lengths = [64, 40]                       # 4 and 3 pages: the rows hold 4
    pool, q, table = _build_case(rng, lengths, hq, hkv, D, 12, cuda, pages_per_seq=4)
    bt = torch.from_numpy(table).to(cuda)
    want, _ = _oracle(pool.float().cpu().numpy(), q.float().cpu().numpy(), table, lengths, hkv,
                      D, 1 / 16)

    def run(ctx_values, pps, nsplit):
        ctx = torch.tensor(ctx_values, dtype=torch.int32, device=cuda)
        part_out = torch.empty((2, hq, nsplit, D), dtype=torch.float32, device=cuda)
        part_lse = torch.empty((2, hq, nsplit), dtype=torch.float32, device=cuda)
        out = torch.empty((2, hq, D), dtype=torch.bfloat16, device=cuda)
        _capi.call("sc_paged_decode_attention", ptr(q), ptr(pool), pool.shape[0], ptr(bt),
                   ptr(ctx), None, 2, hq, hkv, D, P, 4, pps, nsplit, 1 / 16, ptr(part_out),
                   ptr(part_lse), ptr(out), None, stream_of(q))
        torch.cuda.synchronize()
        return out.float().cpu().numpy()

    _capi.device_status()
    assert np.allclose(run([64, 40], 2, 2), want, rtol=RTOL, atol=ATOL)
    _capi.check_device()
    # 100 tokens need 7 pages; the row holds 4: only the row's 64 tokens are read.
    got = run([100, 40], 2, 2)
    with pytest.raises(_capi.DeviceFault, match="outside the pool"):
        _capi.check_device()
    np.testing.assert_allclose(got, want, rtol=RTOL, atol=ATOL)
    # 64 tokens, but one split of 2 pages covers only 32 of them.
    got = run([64, 40], 2, 1)
    with pytest.raises(_capi.DeviceFault):
        _capi.check_device()
    want32, _ = _oracle(pool.float().cpu().numpy(), q.float().cpu().numpy(), table, [32, 32],
                        hkv, D, 1 / 16)
    np.testing.assert_allclose(got, want32, rtol=RTOL, atol=ATOL)
    # A negative length attends nothing (zero output); the other row is unaffected.
    got = run([-5, 40], 2, 2)
    with pytest.raises(_capi.DeviceFault):
        _capi.check_device()
    assert not np.any(got[0])
    np.testing.assert_allclose(got[1], want[1], rtol=RTOL, atol=ATOL)
    assert _capi.device_status() == 0


def test_launch_order_changes_nothing_but_the_schedule(cuda):
    """Any permutation as seq_order gives bit-identical outputs; an entry outside
    0..B-1 is reported through the device status word."""
    from shellsmith_b200 import _capi

    rng = np.random.default_rng(21)
    lengths = [3000, 17, 512, 1, 0, 700, 64, 1300]
    pool, q, table = _build_case(rng, lengths, 16, 2, 256, 400, cuda)
    bt = torch.from_numpy(table).to(cuda)
    ctx = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    base = paged.paged_decode_attention(q, pool, bt, ctx, 0.0625, pages_per_split=8)
    for order in (np.argsort(-np.array(lengths), kind="stable"), rng.permutation(len(lengths))):
        got = paged.paged_decode_attention(q, pool, bt, ctx, 0.0625, pages_per_split=8,
                                           seq_order=torch.from_numpy(order.astype(np.int32))
                                           .to(cuda))
        assert torch.equal(got, base)
    _capi.device_status()
    bad = torch.tensor([0, 1, 2, 3, 4, 5, 6, 99], dtype=torch.int32, device=cuda)
    paged.paged_decode_attention(q, pool, bt, ctx, 0.0625, pages_per_split=8, seq_order=bad)
    with pytest.raises(_capi.DeviceFault):
        _capi.check_device()


@pytest.mark.parametrize("B", [64, 8])
def test_config2_scale_sample_matches_oracle(cuda, B):
    """Config 2's shapes at full size: 64 sequences with contexts U[1k, 32k] whose pages
    come from a random permutation of a 150k-page pool (4.9 GB), and the 8 sequences one
    GPU holds when config 2 is sharded over 8 (there the split floor picks 128-page
    splits). One append + attention step with the default split plan and longest-first
    launch order: every appended token reads back bit for bit, and three sequences
    (shortest, longest, one more) match the oracle."""
    rng = np.random.default_rng(20)
    hq, hkv, D, P, NP = 16, 2, 256, paged.PAGE_SIZE, 150_000
    lengths = rng.integers(1024, 32 * 1024 + 1, size=B)
    need = -(-(lengths + 1) // P)
    perm = rng.permutation(NP).astype(np.int32)
    table = np.zeros((B, int(need.max())), np.int32)
    cursor = 0
    for b in range(B):
        table[b, :need[b]] = perm[cursor:cursor + need[b]]
        cursor += need[b]
    pool = torch.empty((NP, hkv, 2, P, D), dtype=torch.bfloat16, device=cuda)
    flat = pool.view(-1)
    for start in range(0, flat.numel(), 1 << 26):
        part = flat[start:start + (1 << 26)]
        part.copy_(torch.randn(part.shape, device=cuda))
    slots = torch.from_numpy(table[np.arange(B), lengths // P].astype(np.int64) * P
                             + lengths % P).to(cuda)
    ctx = lengths + 1
    q = torch.randn((B, hq, D), device=cuda).to(torch.bfloat16)
    kn = torch.randn((B, hkv, D), device=cuda).to(torch.bfloat16)
    vn = torch.randn((B, hkv, D), device=cuda).to(torch.bfloat16)
    order = torch.from_numpy(np.argsort(-ctx, kind="stable").astype(np.int32)).to(cuda)
    scale = 1.0 / math.sqrt(D)
    if B == 8:
        pps, _ = paged.split_plan(int(need.max()), None, int(need.sum()) * hkv,
                                  paged.sm_count(cuda), waves=3, cap=1024, rows=B * hkv,
                                  min_pages=128)
        assert pps == 128
    paged.kv_append(kn, vn, pool, slots)
    out = paged.paged_decode_attention(q, pool, torch.from_numpy(table).to(cuda),
                                       torch.from_numpy(ctx.astype(np.int32)).to(cuda), scale,
                                       total_pages=int(need.sum()), seq_order=order)
    kg, vg = paged.kv_gather(pool, slots)
    assert torch.equal(kg, kn) and torch.equal(vg, vn)
    for b in (int(np.argmin(lengths)), int(np.argmax(lengths)), 7):
        pages = torch.from_numpy(table[b, :need[b]].astype(np.int64)).to(cuda)
        sub = pool[pages].float().cpu().numpy()
        k, v = oatt.pool_read_pages(sub, np.arange(need[b]), int(ctx[b]), hkv, P, D)
        want, _ = oatt.decode_attention(q[b].float().cpu().numpy(), k, v, scale)
        np.testing.assert_allclose(out[b].float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)
    del pool
    torch.cuda.empty_cache()


def _fused_case(rng, cuda, lengths, hq, hkv, D, num_pages, width):
    """A pool holding each sequence's first L-1 tokens, the new token's K/V and slots."""
    P = paged.PAGE_SIZE
    pool, q, table = _build_case(rng, lengths, hq, hkv, D, num_pages, cuda, pages_per_seq=width)
    B = len(lengths)
    k_new = torch.randn((B, hkv, D), device=cuda).to(torch.bfloat16)
    v_new = torch.randn((B, hkv, D), device=cuda).to(torch.bfloat16)
    slots = np.array([table[b, (L - 1) // P] * P + (L - 1) % P if L > 0 else -1
                      for b, L in enumerate(lengths)], np.int64)
    return pool, q, table, k_new, v_new, torch.from_numpy(slots).to(cuda)


# 64 one-page splits always merge in the separate kernel; with in_kernel_merge, 16 (the
# in-kernel cap) and 8 splits merge in the last split of each sequence; 64 pages per
# split is one split.
@pytest.mark.parametrize("in_kernel_merge", [False, True])
@pytest.mark.parametrize("pages_per_split", [1, 4, 8, 64])
def test_fused_layer_equals_append_then_attention(cuda, pages_per_split, in_kernel_merge):
    """Append + split-K (+ the merge) against kv_append followed by the unfused
    attention: the pool bit for bit, the output within tolerance of the oracle over the
    appended context, the counters back at zero, and a repeated call (counters reused)
    bit-identical."""
    from shellsmith_b200 import _capi

    rng = np.random.default_rng(40 + pages_per_split)
    hq, hkv, D = 16, 2, 256
    lengths = [1, 15, 16, 17, 33, 200, 517, 0, 64, 1000]
    pool, q, table, k_new, v_new, slots = _fused_case(rng, cuda, lengths, hq, hkv, D, 200, 64)
    bt = torch.from_numpy(table).to(cuda)
    ctx = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    ref_pool = pool.clone()
    paged.kv_append(k_new, v_new, ref_pool, slots)
    want_out = paged.paged_decode_attention(q, ref_pool, bt, ctx, 1 / 16,
                                            pages_per_split=pages_per_split)
    ws = paged.AttentionWorkspace(len(lengths), hq, D, 64, device=cuda)
    lse = torch.empty(len(lengths) * hq, dtype=torch.float32, device=cuda)
    got = paged.paged_decode_attention_fused(q, k_new, v_new, slots, pool, bt, ctx, 1 / 16,
                                             pages_per_split=pages_per_split, workspace=ws,
                                             lse_out=lse, in_kernel_merge=in_kernel_merge)
    torch.cuda.synchronize()
    assert torch.equal(pool, ref_pool)
    assert torch.count_nonzero(ws.counters) == 0
    want, want_lse = _oracle(ref_pool.float().cpu().numpy(), q.float().cpu().numpy(), table,
                             lengths, hkv, D, 1 / 16)
    np.testing.assert_allclose(got.float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(lse.cpu().numpy().reshape(want_lse.shape), want_lse, atol=1e-3)
    np.testing.assert_allclose(got.float().cpu().numpy(), want_out.float().cpu().numpy(),
                               rtol=RTOL, atol=ATOL)
    again = paged.paged_decode_attention_fused(q, k_new, v_new, slots, pool, bt, ctx, 1 / 16,
                                               pages_per_split=pages_per_split, workspace=ws,
                                               in_kernel_merge=in_kernel_merge)
    torch.cuda.synchronize()
    assert torch.equal(again, got) and torch.count_nonzero(ws.counters) == 0
    _capi.check_device()


def test_fused_layer_packed_many_splits_and_launch_order(cuda):
    """Packed rows; more splits than one merge window holds (1,100 one-page splits of
    one sequence); any launch order; rows with no new token (slot -1)."""
    from shellsmith_b200 import _capi

    rng = np.random.default_rng(47)
    hq, hkv, D = 8, 1, 128
    lengths = [17600, 300, 1, 45]
    pool, q, table, k_new, v_new, slots = _fused_case(rng, cuda, lengths, hq, hkv, D, 1200,
                                                      1100)
    slots[2] = -1                  # row 2 appends nothing: its one cached token stays
    bt = torch.from_numpy(table).to(cuda)
    ctx = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    ref_pool = pool.clone()
    paged.kv_append(k_new, v_new, ref_pool, slots)
    ws = paged.AttentionWorkspace(len(lengths), hq, D, 1100, device=cuda)
    packed = torch.empty((len(lengths) * hq, D + 1), dtype=torch.float32, device=cuda)
    order = torch.tensor([2, 0, 3, 1], dtype=torch.int32, device=cuda)
    paged.paged_decode_attention_fused(q, k_new, v_new, slots, pool, bt, ctx, 1 / 16,
                                       pages_per_split=1, workspace=ws, packed=packed,
                                       seq_order=order)
    torch.cuda.synchronize()
    assert torch.equal(pool, ref_pool) and torch.count_nonzero(ws.counters) == 0
    want, want_lse = _oracle(ref_pool.float().cpu().numpy(), q.float().cpu().numpy(), table,
                             lengths, hkv, D, 1 / 16)
    got = packed.cpu().numpy().reshape(len(lengths), hq, D + 1)
    np.testing.assert_allclose(got[..., :D], want, rtol=RTOL, atol=ATOL)
    np.testing.assert_allclose(got[..., D], want_lse, atol=1e-3)
    _capi.check_device()
