"""`gated_delta_chunks` (the reference's chunked prefill from gate and beta logits,
numerics/gdn_fused.py:86-122) on the GPU, against the CPU oracle.

Bars.
  * The gates (sc_gdn_sampler_gates) equal oracle.front.sampler_gates bit for bit
    (numerics/metal/gdn_chunk_common.metal:61-75), except on elements the oracle
    marks as rounding ties (a value within 16 fp32 ulps of a bf16 rounding
    boundary, where the device's exp or log, a few ulps from the correctly rounded
    result, may pick the neighbouring bf16): those stay within 2 % and number
    under 1 %.
  * y within rtol 2e-2 / atol 2e-3 and the fp32 state within 1e-4 of the float64
    recurrence fed the oracle's gates.
  * The reference test's own bar (tests/test_gdn_chunk.py:67-78): relative L2 error
    below 0.02 against the recurrence with gates made in fp32 from the logits.
"""

import math

import numpy as np
import pytest
import torch

from oracle import front as ofront
from oracle import gdn as ogdn
from shellsmith_b200 import numerics

pytestmark = pytest.mark.gpu

bf = ofront.bf


def _inputs(rng, batch, length, key_heads, heads):
    """The distributions of the reference test's _inputs (tests/test_gdn_chunk.py:23-37)."""
    def unit(shape):
        x = rng.standard_normal(shape)
        return x / np.sqrt((x * x).sum(-1, keepdims=True))

    q = bf((unit((batch, length, key_heads, 128)) / math.sqrt(128)).astype(np.float32))
    k = bf(unit((batch, length, key_heads, 128)).astype(np.float32))
    v = bf(rng.standard_normal((batch, length, heads, 128)).astype(np.float32))
    a = bf((2 * rng.standard_normal((batch, length, heads)) - 2).astype(np.float32))
    b = bf(rng.standard_normal((batch, length, heads)).astype(np.float32))
    a_log = rng.uniform(-2.0, 1.0, heads).astype(np.float32)
    dt_bias = (0.5 * rng.standard_normal(heads)).astype(np.float32)
    state = bf((0.1 * rng.standard_normal((batch, heads, 128, 128))).astype(np.float32))
    return q, k, v, a, b, a_log, dt_bias, state


def _dev(x, cuda, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda, dtype)


def test_sampler_gates_bit_exact_with_edges(cuda):
    rng = np.random.default_rng(5)
    rows, Hv = 4096, 8
    a = (2 * rng.standard_normal((rows, Hv)) - 2).astype(np.float32)
    b = rng.standard_normal((rows, Hv)).astype(np.float32) * 3
    # Large |a + dt_bias| on both sides (softplus ~ 0 and ~ x), huge logits whose gate
    # underflows below the 1e-6 clamp, and the +-inf of padded rows.
    edges = np.array([-np.inf, np.inf, 0.0, -0.0, 10.0, -10.0, 17.0, -17.0, 20.0, -20.0, 30.0,
                      -30.0, 60.0, -60.0, 88.0, -88.0, 100.0, -100.0, 1e4, -1e4, 3e38,
                      -3e38, 1e-30, -1e-30], np.float32)
    a[:len(edges)] = edges[:, None]
    b[:len(edges)] = edges[:, None]
    a, b = bf(a), bf(b)
    a_log = np.array([-2.0, -0.5, 0.0, 0.3, 1.0, 2.5, 4.0, 6.0], np.float32)
    dt_bias = np.array([0.0, 0.5, -0.7, 1.3, -2.0, 0.1, 3.0, -4.0], np.float32)
    g, beta = numerics.gdn_sampler_gates(_dev(a, cuda), _dev(b, cuda), _dev(a_log, cuda,
                                                                               torch.float32),
                                         _dev(dt_bias, cuda, torch.float32))
    got_g, got_b = g.cpu().numpy(), beta.cpu().numpy()
    want_g, _, want_b, tie = ofront.sampler_gates(a, b, a_log, dt_bias)
    assert tie.mean() < 0.01
    exact = ~tie
    assert np.array_equal(got_g[exact].view(np.uint32), want_g[exact].view(np.uint32))
    assert np.array_equal(got_b[exact].view(np.uint32), want_b[exact].view(np.uint32))
    np.testing.assert_allclose(got_g[tie], want_g[tie], rtol=2e-2, atol=1e-30)
    np.testing.assert_allclose(got_b[tie], want_b[tie], rtol=2e-2, atol=1e-30)
    # The edges: padded rows (a = b = -inf) give gate 1 and beta 0; a gate below
    # 1e-6 is kept as its bf16 value (the chunk kernel clamps it before its log).
    assert np.all(got_g[0] == 1.0) and np.all(got_b[0] == 0.0)
    assert np.all(got_g[1] < 1e-6) and np.all(got_b[1] == 1.0)
    assert (got_g < 1e-6).sum() > Hv


def _sequential_sampler(q, k, v, a, b, a_log, dt_bias, state):
    """The float64 recurrence fed the sampler's gates (clamped at 1e-6)."""
    _, log_gate, beta, _ = ofront.sampler_gates(a, b, a_log, dt_bias)
    return ogdn.sequential(q, k, v, np.exp(log_gate.astype(np.float64)), beta, state)


def _rel_l2(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum()))


# The reference test's shapes (tests/test_gdn_chunk.py:20): (batch, length, key
# heads, value heads); 200 is not a multiple of 64.
@pytest.mark.parametrize("shape", [(1, 128, 2, 6), (1, 200, 1, 3), (2, 64, 2, 2)])
def test_gated_delta_chunks_matches_the_recurrence(cuda, shape):
    rng = np.random.default_rng(sum(shape))
    q, k, v, a, b, a_log, dt_bias, state = _inputs(rng, *shape)
    s = _dev(state, cuda, torch.float32)
    y, s_out = numerics.gated_delta_chunks(_dev(q, cuda), _dev(k, cuda), _dev(v, cuda),
                                           _dev(a, cuda), _dev(b, cuda),
                                           _dev(a_log, cuda, torch.float32),
                                           _dev(dt_bias, cuda, torch.float32), s)
    torch.cuda.synchronize()
    assert s_out is s and y.shape == v.shape and y.dtype == torch.bfloat16
    want_y, want_s = _sequential_sampler(q, k, v, a, b, a_log, dt_bias, state)
    np.testing.assert_allclose(y.float().cpu().numpy(), want_y, rtol=2e-2, atol=2e-3)
    assert np.abs(s.cpu().numpy() - want_s).max() <= 1e-4
    # The reference test's bar: gates in fp32 straight from the logits, rel-L2 < 0.02.
    log_gate = np.maximum(-np.exp(a_log.astype(np.float64))
                          * np.logaddexp(a.astype(np.float64) + dt_bias, 0.0), math.log(1e-6))
    beta32 = 1.0 / (1.0 + np.exp(-b.astype(np.float64)))
    ref_y, ref_s = ogdn.sequential(q, k, v, np.exp(log_gate), beta32, state)
    assert _rel_l2(y.float().cpu().numpy(), ref_y) < 0.02
    assert _rel_l2(s.cpu().numpy(), ref_s) < 0.02


def test_gated_delta_chunks_bf16_state_and_asserts(cuda):
    """A bf16 state (the reference's dtype) is left untouched and the returned state is
    the fp32 run rounded once; shape and dtype violations raise AssertionError."""
    rng = np.random.default_rng(9)
    q, k, v, a, b, a_log, dt_bias, state = _inputs(rng, 1, 100, 2, 4)
    args = [_dev(x, cuda) for x in (q, k, v, a, b)] + [_dev(a_log, cuda, torch.float32),
                                                        _dev(dt_bias, cuda, torch.float32)]
    s16 = _dev(state, cuda)
    before = s16.clone()
    y16, out16 = numerics.gated_delta_chunks(*args, s16)
    s32 = _dev(state, cuda, torch.float32)
    y32, out32 = numerics.gated_delta_chunks(*args, s32)
    torch.cuda.synchronize()
    assert torch.equal(s16, before) and out16.dtype == torch.bfloat16
    assert torch.equal(out16, out32.to(torch.bfloat16)) and torch.equal(y16, y32)
    with pytest.raises(AssertionError):
        numerics.gated_delta_chunks(*args[:3], args[3].float(), *args[4:], s32)
    with pytest.raises(AssertionError):
        numerics.gated_delta_chunks(args[0][..., :64], *args[1:], s32)
