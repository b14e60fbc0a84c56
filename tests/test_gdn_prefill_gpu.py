"""K2/K3 chunked GDN prefill (tcgen05) on the GPU vs the float64 sequential oracle.

Bars: fp32 state within 1e-4 (absolute) of the float64 recurrence, bf16
outputs within rtol 2e-2 / atol 2e-3.
"""

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from shellsmith_b200 import numerics
from shellsmith_b200.workloads import bf16_np, gdn_sequence_inputs, to_device

pytestmark = pytest.mark.gpu

STATE_ATOL = 1e-4
RTOL, ATOL = 2e-2, 2e-3


def _run(q, k, v, g, beta, s0, cu=None, T=None, slots=None, state_rows=None):
    qd, kd, vd = to_device(q, k, v)
    gd, bd = to_device(g, beta, dtype=torch.float32)
    state = torch.from_numpy(np.ascontiguousarray(
        s0 if state_rows is None else state_rows, dtype=np.float32)).cuda()
    cu_t = None if cu is None else torch.tensor(cu, dtype=torch.int32, device="cuda")
    sl = None if slots is None else torch.tensor(slots, dtype=torch.int32, device="cuda")
    out = numerics.gdn_chunk_prefill(qd, kd, vd, gd, bd, state, sl, cu_t, T=T)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), state.cpu().numpy()


# 420 tokens = 7 chunks, the last partial: the K/Q tiles' three buffers wrap twice and
# the prep / state-chain hand-off barriers change phase several times.
@pytest.mark.parametrize("T", [1, 63, 64, 65, 200, 256, 420])
def test_fixed_length_matches_sequential(cuda, T):
    rng = np.random.default_rng(T)
    B, Hk, Hv, d = 2, 2, 4, 128
    q, k, v, g, beta = gdn_sequence_inputs(rng, B, T, Hk, Hv, d, d)
    s0 = (rng.standard_normal((B, Hv, d, d)) * 0.1).astype(np.float32)
    out, state = _run(q.reshape(B * T, Hk, d), k.reshape(B * T, Hk, d), v.reshape(B * T, Hv, d),
                      g.reshape(B * T, Hv), beta.reshape(B * T, Hv), s0, T=T)
    y, s = ogdn.sequential(q, k, v, g, beta, s0)
    np.testing.assert_allclose(out.reshape(B, T, Hv, d), y, rtol=RTOL, atol=ATOL)
    assert np.abs(state - s).max() <= STATE_ATOL, np.abs(state - s).max()


@pytest.mark.parametrize("gates", ["slow", "unit"])
def test_slow_and_unit_gates_keep_state_precision(cuda, gates):
    """Gates near 1 (the reference test's U(.96,.995)) carry the state across chunks."""
    rng = np.random.default_rng(17)
    B, T, Hk, Hv, d = 1, 193, 1, 2, 128
    q, k, v, _, beta = gdn_sequence_inputs(rng, B, T, Hk, Hv, d, d)
    g = (np.ones((B, T, Hv), np.float32) if gates == "unit"
         else rng.uniform(0.96, 0.995, (B, T, Hv)).astype(np.float32))
    s0 = (rng.standard_normal((B, Hv, d, d)) * 0.02).astype(np.float32)
    out, state = _run(q[0], k[0], v[0], g[0], beta[0], s0, T=T)
    y, s = ogdn.sequential(q, k, v, g, beta, s0)
    np.testing.assert_allclose(out, y[0], rtol=RTOL, atol=ATOL)
    assert np.abs(state - s).max() <= STATE_ATOL, np.abs(state - s).max()


def test_varlen_packed_sequences_with_slots(cuda):
    rng = np.random.default_rng(5)
    lengths = [1, 64, 130, 7]
    Hk, Hv, d = 2, 4, 128
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    n = int(cu[-1])
    q, k, v, g, beta = gdn_sequence_inputs(rng, 1, n, Hk, Hv, d, d)
    rows = (rng.standard_normal((6, Hv, d, d)) * 0.1).astype(np.float32)
    slots = [4, 0, 5, 2]
    out, state = _run(q[0], k[0], v[0], g[0], beta[0], None, cu=list(cu), slots=slots,
                      state_rows=rows)
    for b, L in enumerate(lengths):
        a, e = cu[b], cu[b + 1]
        y, s = ogdn.sequential(q[:, a:e], k[:, a:e], v[:, a:e], g[:, a:e], beta[:, a:e],
                               rows[slots[b]][None])
        np.testing.assert_allclose(out[a:e], y[0], rtol=RTOL, atol=ATOL)
        assert np.abs(state[slots[b]] - s[0]).max() <= STATE_ATOL
    untouched = [r for r in range(6) if r not in slots]
    assert np.array_equal(state[untouched], rows[untouched])


def test_varlen_ranked_two_waves_with_ties_empty_and_skipped(cuda):
    """40 packed sequences x 4 value heads = 160 CTAs (two waves on 148 SMs), launched
    longest first with tied lengths ranked by index; empty sequences and a skipped slot
    (-1) leave their state rows untouched."""
    rng = np.random.default_rng(8)
    lengths = list(rng.choice([0, 1, 17, 64, 65, 100], size=40))
    Hk, Hv, d = 2, 4, 128
    cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    n = int(cu[-1])
    q, k, v, g, beta = gdn_sequence_inputs(rng, 1, n, Hk, Hv, d, d)
    rows = (rng.standard_normal((44, Hv, d, d)) * 0.1).astype(np.float32)
    slots = [int(x) for x in rng.permutation(44)[:40]]
    skipped = next(b for b, L in enumerate(lengths) if L > 0)
    slots[skipped] = -1
    out, state = _run(q[0], k[0], v[0], g[0], beta[0], None, cu=list(cu), slots=slots,
                      state_rows=rows)
    for b, L in enumerate(lengths):
        if L == 0 or slots[b] < 0:
            continue
        a, e = cu[b], cu[b + 1]
        y, s = ogdn.sequential(q[:, a:e], k[:, a:e], v[:, a:e], g[:, a:e], beta[:, a:e],
                               rows[slots[b]][None])
        np.testing.assert_allclose(out[a:e], y[0], rtol=RTOL, atol=ATOL)
        assert np.abs(state[slots[b]] - s[0]).max() <= STATE_ATOL
    untouched = [r for r in range(44)
                 if r not in [sl for b, sl in enumerate(slots) if sl >= 0 and lengths[b] > 0]]
    assert np.array_equal(state[untouched], rows[untouched])


def test_config1_shapes_one_sequence(cuda):
    """Config-1 head shapes (16 key / 32 value heads) on a 1k-token sequence."""
    rng = np.random.default_rng(1)
    B, T, Hk, Hv, d = 1, 1024, 16, 32, 128
    q, k, v, g, beta = gdn_sequence_inputs(rng, B, T, Hk, Hv, d, d)
    s0 = np.zeros((B, Hv, d, d), np.float32)
    out, state = _run(q[0], k[0], v[0], g[0], beta[0], s0, T=T)
    y, s = ogdn.sequential(q, k, v, g, beta, s0)
    np.testing.assert_allclose(out, y[0], rtol=RTOL, atol=ATOL)
    assert np.abs(state - s).max() <= STATE_ATOL


def test_prefill_then_decode_continues_the_recurrence(cuda):
    rng = np.random.default_rng(9)
    B, T, Hk, Hv, d = 2, 100, 2, 4, 128
    q, k, v, g, beta = gdn_sequence_inputs(rng, B, T + 3, Hk, Hv, d, d)
    qd, kd, vd = to_device(q[:, :T].reshape(B * T, Hk, d), k[:, :T].reshape(B * T, Hk, d),
                           v[:, :T].reshape(B * T, Hv, d))
    gd, bd = to_device(g[:, :T].reshape(B * T, Hv), beta[:, :T].reshape(B * T, Hv),
                       dtype=torch.float32)
    state = torch.zeros((B, Hv, d, d), dtype=torch.float32, device=cuda)
    numerics.gdn_chunk_prefill(qd, kd, vd, gd, bd, state, T=T)
    for t in range(T, T + 3):
        tq, tk, tv = to_device(q[:, t], k[:, t], v[:, t])
        tg, tb = to_device(g[:, t], beta[:, t], dtype=torch.float32)
        o = numerics.gdn_decode(tq, tk, tv, tg, tb, state)
    y, s = ogdn.sequential(q, k, v, g, beta, np.zeros((B, Hv, d, d)))
    np.testing.assert_allclose(o.float().cpu().numpy(), y[:, -1], rtol=RTOL, atol=ATOL)
    assert np.abs(state.cpu().numpy() - s).max() <= STATE_ATOL


def test_reference_signature(cuda):
    rng = np.random.default_rng(3)
    B, T, Hk, Hv, d = 2, 70, 1, 2, 128
    q, k, v, g, beta = gdn_sequence_inputs(rng, B, T, Hk, Hv, d, d)
    s0 = bf16_np(rng.standard_normal((B, Hv, d, d)) * 0.02)
    qd, kd, vd, s0d = to_device(q, k, v, s0)
    gd, bd = to_device(g, beta, dtype=torch.float32)
    y, s = numerics.gated_delta_chunked(qd, kd, vd, gd, bd, s0d)
    want_y, want_s = ogdn.sequential(q, k, v, g, beta, s0)
    assert y.dtype == torch.bfloat16 and s.dtype == torch.float32
    np.testing.assert_allclose(y.float().cpu().numpy(), want_y, rtol=RTOL, atol=ATOL)
    assert np.abs(s.cpu().numpy() - want_s).max() <= STATE_ATOL
    with pytest.raises(ValueError):
        numerics.gated_delta_chunked(qd, kd, vd, gd, bd, s0d, chunk=32)


def test_config1_full_size_sampled_chains(cuda):
    """Config 1 at full size (B = 8, T = 4096, 16 key / 32 value heads, 256 chains of 64
    chunks, 537 MB of v): every chain runs on the GPU and six (sequence, value head)
    chains — the first and last of the grid and four drawn at random — are checked
    against the float64 sequential recurrence over all 4,096 tokens."""
    from shellsmith_b200.workloads import gdn_token_inputs_device

    B, T, Hk, Hv, d = 8, 4096, 16, 32, 128
    gen = torch.Generator(device=cuda)
    gen.manual_seed(1)
    q, k, v, decay, beta = gdn_token_inputs_device(gen, B * T, Hk, Hv, d, d, device=cuda)
    state = torch.zeros((B, Hv, d, d), dtype=torch.float32, device=cuda)
    out = numerics.gdn_chunk_prefill(q, k, v, decay, beta, state, T=T)
    torch.cuda.synchronize()
    rng = np.random.default_rng(11)
    picks = [(0, 0), (B - 1, Hv - 1)] + [(int(rng.integers(B)), int(rng.integers(Hv)))
                                         for _ in range(4)]
    group = Hv // Hk
    for b, h in picks:
        rows = slice(b * T, (b + 1) * T)
        kh = h // group
        qs = q[rows, kh].float().cpu().numpy()[None, :, None]
        ks = k[rows, kh].float().cpu().numpy()[None, :, None]
        vs = v[rows, h].float().cpu().numpy()[None, :, None]
        gs = decay[rows, h].cpu().numpy()[None, :, None]
        bs = beta[rows, h].cpu().numpy()[None, :, None]
        y, s = ogdn.sequential(qs, ks, vs, gs, bs, np.zeros((1, 1, d, d)))
        np.testing.assert_allclose(out[rows, h].float().cpu().numpy(), y[0, :, 0],
                                   rtol=RTOL, atol=ATOL, err_msg=f"chain {(b, h)}")
        err = np.abs(state[b, h].cpu().numpy() - s[0, 0]).max()
        assert err <= STATE_ATOL, (b, h, err)
