"""K1 gdn_decode parity on the GPU against the float64 CPU oracle.

Tolerances: fp32 state within 1e-4 of the float64
recurrence; bf16 outputs within rtol 2e-2 / atol 2e-3. The bf16-state
variant is held to the reference test's own bound (rel-L2 < 0.015,
tests/test_bf16_token_decode.py:12-40 of the reference).
"""

import numpy as np
import pytest
import torch

from oracle import gdn as ogdn
from shellsmith_b200 import numerics
from shellsmith_b200.workloads import bf16_np, gdn_token_inputs, to_device

pytestmark = pytest.mark.gpu

STATE_ATOL = 1e-4
OUT_RTOL, OUT_ATOL = 2e-2, 2e-3


def _dev(q, k, v, g, beta):
    qd, kd, vd = to_device(q, k, v)
    gd, bd = to_device(g, beta, dtype=torch.float32)
    return qd, kd, vd, gd, bd


def test_config0_256_steps_fp32_state(cuda):
    """Config 0: B=4, 8 heads, 128x128, 256 steps, S0 = 0, seed 0."""
    rng = np.random.default_rng(0)
    B, H, d = 4, 8, 128
    state = torch.zeros((B, H, d, d), dtype=torch.float32, device=cuda)
    ref = np.zeros((B, H, d, d))
    for step in range(256):
        q, k, v, g, beta = gdn_token_inputs(rng, B, H, H, d, d)
        out = numerics.gdn_decode(*_dev(q, k, v, g, beta), state)
        want, ref = ogdn.token_step(q, k, v, g, beta, ref)
        np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=OUT_RTOL, atol=OUT_ATOL,
                                   err_msg=f"step {step}")
    torch.cuda.synchronize()
    err = np.abs(state.cpu().numpy() - ref).max()
    assert err <= STATE_ATOL, err


@pytest.mark.parametrize("B,Hk,Hv,dk,dv", [(1, 2, 6, 32, 16), (2, 2, 6, 128, 128),
                                           (3, 16, 32, 128, 128), (2, 1, 2, 64, 64),
                                           (2, 4, 8, 256, 128)])
def test_gqa_shapes_fp32_state(cuda, B, Hk, Hv, dk, dv):
    rng = np.random.default_rng(B * 1000 + dk + dv)
    s0 = rng.standard_normal((B, Hv, dv, dk)) * 0.1
    state = torch.from_numpy(s0.astype(np.float32)).to(cuda)
    ref = s0.astype(np.float32).astype(np.float64)
    for step in range(6):
        q, k, v, g, beta = gdn_token_inputs(rng, B, Hk, Hv, dk, dv)
        out = numerics.gdn_decode(*_dev(q, k, v, g, beta), state)
        want, ref = ogdn.token_step(q, k, v, g, beta, ref)
        np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=OUT_RTOL, atol=OUT_ATOL)
    assert np.abs(state.cpu().numpy() - ref).max() <= STATE_ATOL


@pytest.mark.parametrize("batch,keys,values", [(1, 32, 16), (2, 128, 128)])
def test_reference_token_test_bf16_state(cuda, batch, keys, values):
    """The reference token test: 6 value / 2 key heads, g=0.984375, beta=0.5, 8 steps,
    bf16 state, compared each step with the float64 step from the kernel's own carry."""
    rng = np.random.default_rng(91)
    state_np = bf16_np(rng.standard_normal((batch, 6, values, keys)) * 0.02)
    state = torch.from_numpy(state_np).to(cuda, torch.bfloat16)
    for _ in range(8):
        q = bf16_np(rng.standard_normal((batch, 1, 2, keys)) * 0.05)
        k = bf16_np(rng.standard_normal(q.shape) * 0.08)
        v = bf16_np(rng.standard_normal((batch, 1, 6, values)) * 0.1)
        g = np.full((batch, 1, 6), 0.984375, np.float32)
        beta = np.full(g.shape, 0.5, np.float32)
        carry = state.float().cpu().numpy().astype(np.float64)
        qd, kd, vd, gd, bd = to_device(q, k, v, g, beta)
        out, state = numerics.gated_delta_token(qd, kd, vd, gd, bd, state)
        exact_out, exact_state = ogdn.token_step(q[:, 0], k[:, 0], v[:, 0], g[:, 0], beta[:, 0],
                                                 carry)
        for actual, target in ((out[:, 0], exact_out), (state, exact_state)):
            plain = actual.float().cpu().numpy().astype(np.float64)
            assert np.linalg.norm(plain - target) / np.linalg.norm(target) < 0.015
        # The reference kernel's rounding points, restated in fp32 on the CPU.
        bf_out, bf_state = ogdn.token_step_bf16(q[:, 0], k[:, 0], v[:, 0], g[:, 0], beta[:, 0],
                                                carry.astype(np.float32))
        got = state.float().cpu().numpy()
        # Sums run in a different order, so a rare value sits one bf16 ulp away.
        assert np.mean(got != bf_state) < 0.01
        np.testing.assert_allclose(got, bf_state, rtol=2 ** -7, atol=1e-6)
        np.testing.assert_allclose(out[:, 0].float().cpu().numpy(), bf_out, rtol=2e-2, atol=2e-3)


def test_state_slots_and_skipped_rows(cuda):
    """Rows map to arbitrary state slots; a negative slot leaves everything untouched."""
    rng = np.random.default_rng(5)
    B, Hk, Hv, d, slots = 5, 2, 4, 128, 9
    s0 = (rng.standard_normal((slots, Hv, d, d)) * 0.1).astype(np.float32)
    state = torch.from_numpy(s0).to(cuda)
    slot = np.array([7, 0, -1, 3, 8], np.int32)
    q, k, v, g, beta = gdn_token_inputs(rng, B, Hk, Hv, d, d)
    out = torch.full((B, Hv, d), 7.0, dtype=torch.bfloat16, device=cuda)
    numerics.gdn_decode(*_dev(q, k, v, g, beta), state,
                        torch.from_numpy(slot).to(cuda), out=out)
    got = state.cpu().numpy()
    want = s0.astype(np.float64)
    for b, s in enumerate(slot):
        if s < 0:
            continue
        o, want[s] = (x[0] for x in ogdn.token_step(q[b:b + 1], k[b:b + 1], v[b:b + 1],
                                                     g[b:b + 1], beta[b:b + 1],
                                                     s0[s:s + 1].astype(np.float64)))
        np.testing.assert_allclose(out[b].float().cpu().numpy(), o, rtol=OUT_RTOL, atol=OUT_ATOL)
    assert np.abs(got - want).max() <= STATE_ATOL
    assert torch.all(out[2] == 7.0)


def test_bad_shapes_raise(cuda):
    q = torch.zeros((1, 1, 2, 48), dtype=torch.bfloat16, device=cuda)
    v = torch.zeros((1, 1, 6, 16), dtype=torch.bfloat16, device=cuda)
    g = torch.zeros((1, 1, 6), dtype=torch.bfloat16, device=cuda)
    state = torch.zeros((1, 6, 16, 48), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(AssertionError):  # keys % 32 != 0, as the reference asserts
        numerics.gated_delta_token(q, q, v, g, g, state)


def test_out_of_range_state_slot_is_flagged_not_read(cuda):
    from shellsmith_b200 import _capi

    _capi.device_status()
    rng = np.random.default_rng(8)
    q, k, v, g, beta = gdn_token_inputs(rng, 2, 2, 4, 128, 128)
    state = torch.zeros((2, 4, 128, 128), dtype=torch.float32, device=cuda)
    slot = torch.tensor([0, 5], dtype=torch.int32, device=cuda)
    numerics.gdn_decode(*_dev(q, k, v, g, beta), state, slot)
    with pytest.raises(_capi.DeviceFault):
        _capi.check_device()
    assert torch.count_nonzero(state[1]) == 0


def test_chained_layers_equal_plain_updates(cuda):
    """sc_gdn_decode_chained over a stack of layers (each its own state, as a model's
    GDN layers) equals the plain entry bit for bit, queued back to back with no host
    sync, for the one-chunk-per-CTA (B = 1) and bulk (B = 16) launch shapes."""
    from shellsmith_b200.workloads import gdn_token_inputs_device

    for B in (1, 16):
        gen = torch.Generator(device=cuda)
        gen.manual_seed(B)
        layers, Hk, Hv, d = 6, 16, 32, 128
        inputs = [gdn_token_inputs_device(gen, B, Hk, Hv, d, d, device=cuda)
                  for _ in range(layers)]
        start = torch.randn((layers, B, Hv, d, d), generator=gen, device=cuda) * 0.1
        results = []
        for chained in (False, True):
            state = start.clone()
            outs = []
            for step in range(3):
                for layer in range(layers):
                    outs.append(numerics.gdn_decode(*inputs[layer], state[layer],
                                                    chained=chained))
            torch.cuda.synchronize()
            results.append((state, outs))
        (s0, o0), (s1, o1) = results
        assert torch.equal(s0, s1)
        assert all(torch.equal(a, b) for a, b in zip(o0, o1))
    from shellsmith_b200 import _capi

    _capi.check_device()
