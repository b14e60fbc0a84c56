"""8-bit KV pages on the GPU against the CPU oracle.

Bars: the codes, scales and biases the append kernel stores are bit-exact
with oracle.attention.quantize_q8 on the same bf16 inputs (fp32 IEEE
arithmetic on both sides). Attention over an 8-bit pool is compared with the
float64 oracle over the DEQUANTISED K/V at the bf16 path's bar (rtol 2e-2 /
atol 2e-3, lse 1e-3): the kernel feeds codes to fp16 tensor cores and applies
scale and bias per token and group, which is exact algebra up to fp32 sums
and one fp16 rounding of the scaled probabilities.
"""

import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from shellsmith_b200 import paged

pytestmark = pytest.mark.gpu

RTOL, ATOL = 2e-2, 2e-3
P = paged.PAGE_SIZE


def _bf16(x):
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16)


def _fill(rng, lengths, hkv, D, num_pages, cuda, width=None, scale=1.0):
    """Random bf16 K/V appended into a fresh 8-bit pool; returns pool, table, and the
    oracle's dequantised K/V per sequence."""
    need = [math.ceil(L / P) for L in lengths]
    width = width or max(1, max(need))
    perm = rng.permutation(num_pages)
    table = np.zeros((len(lengths), width), np.int32)
    pool = paged.new_pool_q8(num_pages, hkv, D, device=cuda)
    pool.random_(0, 256)  # stale bytes everywhere (rows past a context stay garbage)
    cursor, deq = 0, []
    for b, (L, n) in enumerate(zip(lengths, need)):
        table[b, :n] = perm[cursor:cursor + n]
        cursor += n
        k = (rng.standard_normal((L, hkv, D)) * scale).astype(np.float32)
        v = (rng.standard_normal((L, hkv, D)) * scale).astype(np.float32)
        kb, vb = _bf16(k), _bf16(v)
        slots = (table[b, np.arange(L) // P].astype(np.int64) * P + np.arange(L) % P)
        paged.kv_append(kb.to(cuda), vb.to(cuda), pool, torch.from_numpy(slots).to(cuda))
        kq = oatt.dequantize_q8(*oatt.quantize_q8(kb.float().numpy()))
        vq = oatt.dequantize_q8(*oatt.quantize_q8(vb.float().numpy()))
        deq.append((kq, vq))
    return pool, table, deq


@pytest.mark.parametrize("D", [128, 256])
def test_append_codes_and_scales_bit_exact(cuda, D):
    rng = np.random.default_rng(D)
    hkv, ntok, num_pages = 2, 70, 9
    x = rng.standard_normal((ntok, hkv, D)).astype(np.float32) * 3
    x[5, 0, :64] = 0.75            # a constant group: scale 0, codes 0, bias exact
    x[6, 1, 64:128] = -2.0
    k, v = _bf16(x), _bf16(x[::-1].copy())
    slots = rng.permutation(num_pages * P)[:ntok].astype(np.int64)
    slots[3] = -1
    pool = paged.new_pool_q8(num_pages, hkv, D, device=cuda)
    pool.zero_()
    slot_t = torch.from_numpy(slots).to(cuda)
    paged.kv_append(k.to(cuda), v.to(cuda), pool, slot_t)
    codes, sb = paged.kv_gather_q8(pool, slot_t)
    codes, sb = codes.cpu().numpy(), sb.float().cpu().numpy()
    for which, src in ((0, k), (1, v)):
        want_c, want_s, want_b = oatt.quantize_q8(src.float().numpy())
        keep = slots >= 0
        assert np.array_equal(codes[keep, :, which], want_c[keep])
        assert np.array_equal(sb[keep, :, which, :, 0], want_s[keep])
        assert np.array_equal(sb[keep, :, which, :, 1], want_b[keep])
        assert not codes[~keep].any()
    assert (sb[5, 0, 0, 0, 0], sb[5, 0, 0, 0, 1]) == (0.0, 0.75)
    # Copy-on-write page copy keeps blocks bit-exact.
    before = pool.clone()
    paged.kv_copy_pages(pool, torch.tensor([1, 4], dtype=torch.int32, device=cuda),
                        torch.tensor([8, 0], dtype=torch.int32, device=cuda))
    assert torch.equal(pool[8], before[1]) and torch.equal(pool[0], before[4])
    assert torch.equal(pool[2:8], before[2:8])


@pytest.mark.parametrize("hq,hkv,D", [(16, 2, 256), (24, 4, 256), (8, 8, 128), (12, 2, 128)])
@pytest.mark.parametrize("pages_per_split", [1, 3, 64])
def test_q8_attention_matches_oracle_on_dequantised_cache(cuda, hq, hkv, D, pages_per_split):
    rng = np.random.default_rng(hq * 100 + hkv * 10 + D + pages_per_split)
    lengths = [1, 15, 16, 17, 33, 200, 517, 64]
    pool, table, deq = _fill(rng, lengths, hkv, D, 160, cuda, width=40)
    scale = 1.0 / math.sqrt(D)
    q = torch.randn((len(lengths), hq, D), device=cuda).to(torch.bfloat16)
    ctx = torch.tensor(lengths, dtype=torch.int32, device=cuda)
    lse = torch.empty(len(lengths) * hq, dtype=torch.float32, device=cuda)
    out = paged.paged_decode_attention(q, pool, torch.from_numpy(table).to(cuda), ctx, scale,
                                       pages_per_split=pages_per_split, lse_out=lse)
    qn = q.float().cpu().numpy()
    for b, (kq, vq) in enumerate(deq):
        want, want_lse = oatt.decode_attention(qn[b], kq, vq, scale)
        np.testing.assert_allclose(out[b].float().cpu().numpy(), want, rtol=RTOL, atol=ATOL)
        np.testing.assert_allclose(lse.cpu().numpy().reshape(len(lengths), hq)[b], want_lse,
                                   atol=1e-3)


def test_q8_known_answer_and_empty_sequence(cuda):
    """Constant V rows quantise exactly (scale 0, bias = the value): q = 0 averages
    v = [1, 3, 8] to 4 exactly, as in the reference's attention oracle test."""
    D = 128
    pool = paged.new_pool_q8(4, 1, D, device=cuda)
    pool.random_(0, 256)
    k = torch.zeros((3, 1, D), dtype=torch.bfloat16, device=cuda)
    v = torch.zeros((3, 1, D), dtype=torch.bfloat16, device=cuda)
    v[:, 0, :] = torch.tensor([1.0, 3.0, 8.0], device=cuda)[:, None]
    paged.kv_append(k, v, pool, torch.tensor([32, 33, 34], dtype=torch.int64, device=cuda))
    q = torch.zeros((2, 2, D), dtype=torch.bfloat16, device=cuda)
    out = paged.paged_decode_attention(q, pool, torch.tensor([[2], [2]], dtype=torch.int32,
                                                             device=cuda),
                                       torch.tensor([3, 0], dtype=torch.int32, device=cuda), 1.0)
    assert torch.all(out[0].float() == 4.0)
    assert torch.count_nonzero(out[1]) == 0


def test_q8_split_combine_equals_single_pass_on_a_long_sequence(cuda):
    """Splitting equals one pass, and over 3000 tokens the answer stays within
    5e-3 of the oracle on the dequantised cache."""
    rng = np.random.default_rng(12)
    L, hq, hkv, D = 3000, 16, 2, 256
    pool, table, deq = _fill(rng, [L], hkv, D, 200, cuda)
    q = torch.randn((1, hq, D), device=cuda).to(torch.bfloat16)
    ctx = torch.tensor([L], dtype=torch.int32, device=cuda)
    bt = torch.from_numpy(table).to(cuda)
    one = paged.paged_decode_attention(q, pool, bt, ctx, 0.0625, pages_per_split=4096)
    many = paged.paged_decode_attention(q, pool, bt, ctx, 0.0625, pages_per_split=5)
    np.testing.assert_allclose(one.float().cpu().numpy(), many.float().cpu().numpy(), rtol=RTOL,
                               atol=ATOL)
    kq, vq = deq[0]
    exact, _ = oatt.decode_attention(q[0].float().cpu().numpy(), kq, vq, 0.0625)
    assert np.abs(one[0].float().cpu().numpy() - exact).max() < 5e-3


def test_q8_bad_page_index_sets_device_status(cuda):
    from shellsmith_b200 import _capi

    _capi.device_status()
    pool = paged.new_pool_q8(4, 1, 128, device=cuda)
    pool.zero_()
    q = torch.randn((1, 2, 128), device=cuda).to(torch.bfloat16)
    table = torch.tensor([[0, 99]], dtype=torch.int32, device=cuda)
    paged.paged_decode_attention(q, pool, table, torch.tensor([20], dtype=torch.int32,
                                                              device=cuda), 0.1)
    with pytest.raises(_capi.DeviceFault):
        _capi.check_device()
    assert _capi.device_status() == 0
