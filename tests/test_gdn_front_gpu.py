"""GDN layer glue on the GPU (conv taps, SiLU, q/k norm, gates, gated RMS norm)
against the CPU restatement in oracle.front.

Bars, stage by stage (the three-kernel decode and the prefill expose every stage):
  * tap rings are bit-exact (they are copies of the inputs);
  * the front's q, k, v, g, beta are bf16 values that the kernel computes in fp32
    and the oracle in float64 before the same roundings, so an element may land one
    bf16 step (2^-8 relative) away: at most 1 % of elements may differ and none by
    more than 2 steps;
  * the recurrence, fed the GPU's own front values and its state before the step:
    state within 1e-4, its output y within rtol 2e-2 / atol 2e-3 (the north-star
    bars; a front element one bf16 step away would move a state row by
    beta 2^-8 |v|, which is why the recurrence is checked on the GPU's own inputs);
  * the gated norm of the GPU's y: at most 1 % of elements one or two bf16 steps off.
The one-launch fused decode (experimental: measured slower than the three-kernel
step) hides its stages; it is checked end to end with looser bars (outputs
rtol/atol 3e-2, state 2e-2), as are the integration tests further down.
"""

import numpy as np
import pytest
import torch

from oracle import front as ofront
from oracle import gdn as ogdn
from shellsmith_b200 import gdn_layer, numerics
from shellsmith_b200.gdn_layer import GDNWeights

pytestmark = pytest.mark.gpu

bf = ofront.bf


def _weights(rng, Hk, Hv, cuda):
    C = (2 * Hk + Hv) * 128
    conv_w = bf((rng.standard_normal((C, 4)) * 0.5).astype(np.float32))
    a_log = np.log(rng.uniform(1, 16, Hv)).astype(np.float32)
    dt_bias = bf(rng.standard_normal(Hv).astype(np.float32))
    norm_w = bf((1 + 0.1 * rng.standard_normal(128)).astype(np.float32))
    w = GDNWeights(conv_w=torch.from_numpy(conv_w).to(cuda, torch.bfloat16),
                   a_log=torch.from_numpy(a_log).to(cuda),
                   dt_bias=torch.from_numpy(dt_bias).to(cuda),
                   norm_w=torch.from_numpy(norm_w).to(cuda, torch.bfloat16), eps=1e-6,
                   key_heads=Hk, value_heads=Hv)
    return w, (conv_w, a_log, dt_bias, norm_w)


def _inputs(rng, shape_prefix, Hk, Hv):
    C = (2 * Hk + Hv) * 128
    qkv = bf(rng.standard_normal((*shape_prefix, C)).astype(np.float32))
    z = bf(rng.standard_normal((*shape_prefix, Hv * 128)).astype(np.float32))
    a = bf(rng.standard_normal((*shape_prefix, Hv)).astype(np.float32))
    b = bf(rng.standard_normal((*shape_prefix, Hv)).astype(np.float32))
    return qkv, z, a, b


def _dev(x, cuda, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda, dtype)


def _close_bf16(got, want, name):
    """At most 1% of elements one or two bf16 steps apart, none further."""
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    step = np.maximum(np.abs(want), 1e-30) * 2.0 ** -7
    far = np.abs(got - want) > 2.01 * step
    near = np.abs(got - want) > 0
    assert not far.any(), (name, np.abs(got - want).max())
    assert near.mean() <= 0.01, (name, near.mean())


def _check_stages(front_got, front_want, y_got, state_before, state_after, z, out,
                  norm_w):
    """Per-stage bars for rows of one step (see the module docstring)."""
    q, k, v, g, beta = front_got
    for name, got, want in zip("q k v g beta".split(), front_got, front_want):
        _close_bf16(got, want, name)
    y_ref, s_ref = ogdn.token_step(q, k, v, g, beta, state_before)
    assert np.abs(state_after - s_ref).max() <= 1e-4
    np.testing.assert_allclose(y_got, y_ref, rtol=2e-2, atol=2e-3)
    B, Hv = v.shape[:2]
    want_out = ofront.gated_rms_norm(y_got, z.reshape(B, Hv, 128), norm_w, 1e-6)
    _close_bf16(out.reshape(B, Hv, 128), want_out, "gated norm")


# B = 64 with 8 value heads: 1024 update CTAs, more than are resident at once.
# (1, 3, 4): an odd number of heads (5). qkv_off passes qkv 4 bytes past an 8-byte
# boundary, which the 8-byte vector front cannot take: the per-channel kernel runs.
@pytest.mark.parametrize("Hk,Hv,B,qkv_off", [(2, 4, 3, False), (16, 32, 5, False),
                                             (2, 8, 64, False), (1, 3, 4, False),
                                             (2, 4, 3, True)])
def test_split_decode_stages_match_oracle_over_steps(cuda, Hk, Hv, B, qkv_off):
    """Five decode steps of the three-kernel form, every stage at its bar."""
    rng = np.random.default_rng(Hk * 10 + Hv)
    w, (conv_w, a_log, dt_bias, norm_w) = _weights(rng, Hk, Hv, cuda)
    slots = B + 2
    perm = rng.permutation(slots)[:B].astype(np.int32)
    idx = perm.astype(np.int64)
    taps = gdn_layer.new_taps(slots, w, device=cuda)
    state = torch.zeros((slots, Hv, 128, 128), dtype=torch.float32, device=cuda)
    ws = gdn_layer.SplitWorkspace(B, w, cuda)
    ref_taps = np.zeros((B, 3, w.channels), np.float32)
    slot_t = _dev(perm, cuda, torch.int32)
    for step in range(5):
        qkv, z, a, b = _inputs(rng, (B,), Hk, Hv)
        pos = torch.full((B,), step, dtype=torch.int32, device=cuda)
        before = state[idx].double().cpu().numpy()
        qkv_d = _dev(qkv, cuda)
        if qkv_off:  # the same values, 4 bytes past an 8-byte boundary
            wide = torch.empty(qkv_d.numel() + 2, dtype=qkv_d.dtype, device=cuda)
            qkv_d = wide[2:].view(qkv_d.shape).copy_(qkv_d)
            assert qkv_d.data_ptr() % 8 == 4
        out = gdn_layer.gdn_decode_split(qkv_d, _dev(z, cuda), _dev(a, cuda),
                                         _dev(b, cuda), w, taps, pos, state, slot_t,
                                         workspace=ws)
        torch.cuda.synchronize()
        q, k, v, y, g, beta = (t.float().cpu().numpy() for t in ws.views(B, Hk, Hv))
        *want_front, ref_taps = ofront.front(qkv[:, None], a[:, None], b[:, None], ref_taps,
                                             conv_w, a_log, dt_bias, Hk, Hv)
        _check_stages((q, k, v, g, beta), [x[:, 0] for x in want_front], y, before,
                      state[idx].double().cpu().numpy(), z, out.float().cpu().numpy(), norm_w)
        for r in range(B):
            window = gdn_layer.ring_window(taps, int(perm[r]), step + 1)
            assert np.array_equal(window.float().cpu().numpy(), ref_taps[r])
    assert torch.count_nonzero(state[np.setdiff1d(np.arange(slots), perm)]) == 0


@pytest.mark.parametrize("Hk,Hv,B", [(2, 4, 3), (16, 32, 5), (2, 8, 64)])
def test_fused_decode_matches_oracle_over_steps(cuda, Hk, Hv, B):
    """The experimental one-launch form, end to end against the oracle layer."""
    rng = np.random.default_rng(Hk * 10 + Hv)
    w, (conv_w, a_log, dt_bias, norm_w) = _weights(rng, Hk, Hv, cuda)
    slots = B + 2
    perm = rng.permutation(slots)[:B].astype(np.int32)
    taps = gdn_layer.new_taps(slots, w, device=cuda)
    state = torch.zeros((slots, Hv, 128, 128), dtype=torch.float32, device=cuda)
    ref_taps = np.zeros((B, 3, w.channels), np.float32)
    ref_state = np.zeros((B, Hv, 128, 128))
    slot_t = _dev(perm, cuda, torch.int32)
    for step in range(5):
        qkv, z, a, b = _inputs(rng, (B,), Hk, Hv)
        pos = torch.full((B,), step, dtype=torch.int32, device=cuda)
        out = gdn_layer.gdn_decode_fused(_dev(qkv, cuda), _dev(z, cuda), _dev(a, cuda),
                                         _dev(b, cuda), w, taps, pos, state, slot_t)
        want, ref_taps, ref_state = ofront.decode_layer(qkv, z, a, b, ref_taps, ref_state, conv_w,
                                                        a_log, dt_bias, norm_w, 1e-6, Hk, Hv)
        np.testing.assert_allclose(out.float().cpu().numpy(), want, rtol=3e-2, atol=3e-2)
        for r in range(B):
            window = gdn_layer.ring_window(taps, int(perm[r]), step + 1)
            assert np.array_equal(window.float().cpu().numpy(), ref_taps[r])
    got_state = state[perm.astype(np.int64)].cpu().numpy()
    assert np.abs(got_state - ref_state).max() <= 2e-2
    assert torch.count_nonzero(state[np.setdiff1d(np.arange(slots), perm)]) == 0


@pytest.mark.parametrize("path", ["fused", "split"])
def test_decode_skips_rows_and_keeps_others(cuda, path):
    Hv = 4
    rng = np.random.default_rng(4)
    Hk, B = 2, 3
    w, _ = _weights(rng, Hk, Hv, cuda)
    taps = gdn_layer.new_taps(4, w, device=cuda)
    state = torch.randn((4, Hv, 128, 128), device=cuda)
    before_state, before_taps = state.clone(), taps.clone()
    qkv, z, a, b = _inputs(rng, (B,), Hk, Hv)
    slot_t = torch.tensor([2, -1, 0], dtype=torch.int32, device=cuda)
    pos = torch.tensor([7, 7, 9], dtype=torch.int32, device=cuda)
    getattr(gdn_layer, f"gdn_decode_{path}")(_dev(qkv, cuda), _dev(z, cuda), _dev(a, cuda),
                                             _dev(b, cuda), w, taps, pos, state, slot_t)
    torch.cuda.synchronize()
    for s in (1, 3):
        assert torch.equal(state[s], before_state[s]) and torch.equal(taps[s], before_taps[s])
    # Only the write rows of positions 7 (slot 2) and 9 (slot 0) changed.
    assert torch.equal(taps[2, [0, 1, 2]], before_taps[2, [0, 1, 2]])
    assert torch.equal(taps[2, 3], _dev(qkv[0], cuda))
    assert torch.equal(taps[0, 1], _dev(qkv[2], cuda))


def _oracle_prefill(qkv, z, a, b, taps3, s0, weights_np, Hk, Hv):
    """Per-sequence oracle: front over the run, float64 recurrence, gated norm."""
    conv_w, a_log, dt_bias, norm_w = weights_np
    q, k, v, g, beta, new_taps = ofront.front(qkv[None], a[None], b[None], taps3[None], conv_w,
                                              a_log, dt_bias, Hk, Hv)
    y, s = ogdn.sequential(q, k, v, g, beta, s0[None])
    y = bf(np.asarray(y, np.float32))
    L = qkv.shape[0]
    out = ofront.gated_rms_norm(y[0], z.reshape(L, Hv, 128), norm_w, 1e-6)
    return (q[0], k[0], v[0], g[0], beta[0]), out.reshape(L, -1), new_taps[0], s[0]


def test_prefill_front_and_layer_match_oracle_ragged_with_history(cuda):
    """Two prompts (100 and 37 tokens), the second continuing at position 5 of a
    slot whose ring holds history; then the taps, the state and the output."""
    rng = np.random.default_rng(8)
    Hk, Hv = 2, 4
    w, weights_np = _weights(rng, Hk, Hv, cuda)
    C = w.channels
    lengths, starts, slots = [100, 37], [0, 5], [3, 1]
    taps = gdn_layer.new_taps(4, w, device=cuda)
    hist = bf(rng.standard_normal((3, C)).astype(np.float32))    # positions 2, 3, 4 of slot 1
    for p, row in zip((2, 3, 4), hist):
        taps[1, p % 4] = _dev(row, cuda)
    s0 = (rng.standard_normal((Hv, 128, 128)) * 0.1).astype(np.float32)
    state = torch.zeros((4, Hv, 128, 128), dtype=torch.float32, device=cuda)
    state[1] = torch.from_numpy(s0).to(cuda)
    qkv, z, a, b = _inputs(rng, (sum(lengths),), Hk, Hv)
    cu = torch.tensor([0, 100, 137], dtype=torch.int32, device=cuda)
    slot_t = torch.tensor(slots, dtype=torch.int32, device=cuda)
    start_t = torch.tensor(starts, dtype=torch.int32, device=cuda)
    front = gdn_layer.gdn_prefill_front(_dev(qkv, cuda), _dev(a, cuda), _dev(b, cuda), w, taps,
                                        cu, slot_t, start_t)
    # The recurrence on the GPU's own front values, on a copy of the state.
    state_y = state.clone()
    y = numerics.gdn_chunk_prefill(*front, state_y, slot_t, cu)
    out = gdn_layer.gdn_prefill(_dev(qkv, cuda), _dev(z, cuda), _dev(a, cuda), _dev(b, cuda), w,
                                taps, state, cu, slot_t, start_t)
    torch.cuda.synchronize()
    assert torch.equal(state, state_y)      # the layer runs the same kernels
    offs = [0, 100, 137]
    for i, (L, start, slot) in enumerate(zip(lengths, starts, slots)):
        sl = slice(offs[i], offs[i + 1])
        t3 = np.zeros((3, C), np.float32) if start == 0 else hist
        s_init = np.zeros((Hv, 128, 128)) if start == 0 else s0
        want_front, want_out, want_taps, want_s = _oracle_prefill(
            qkv[sl], z[sl], a[sl], b[sl], t3, s_init, weights_np, Hk, Hv)
        got_front = [t[sl].float().cpu().numpy() for t in front]
        for name, got, want in zip("q k v g beta".split(), got_front, want_front):
            _close_bf16(got, want, name)
        # Recurrence stage at the north-star bars, fed the GPU's front values.
        y_ref, s_ref = ogdn.sequential(*(x[None] for x in got_front), s_init[None])
        assert np.abs(state[slot].cpu().numpy() - s_ref[0]).max() <= 1e-4
        y_got = y[sl].float().cpu().numpy()
        np.testing.assert_allclose(y_got, y_ref[0], rtol=2e-2, atol=2e-3)
        _close_bf16(out[sl].float().cpu().numpy().reshape(L, Hv, 128),
                    ofront.gated_rms_norm(y_got, z[sl].reshape(L, Hv, 128), weights_np[3],
                                          1e-6), "gated norm")
        # End to end against the all-oracle layer (front roundings propagate).
        np.testing.assert_allclose(out[sl].float().cpu().numpy(), want_out, rtol=3e-2,
                                   atol=3e-2)
        window = gdn_layer.ring_window(taps, slot, start + L).float().cpu().numpy()
        assert np.array_equal(window, want_taps)
        assert np.abs(state[slot].cpu().numpy() - want_s).max() <= 2e-2


def test_prefill_then_decode_equals_longer_prefill(cuda):
    """Prefill 70 tokens then decode 3 == prefill 73 tokens (taps exact, state and
    the last outputs within tolerance)."""
    rng = np.random.default_rng(12)
    Hk, Hv = 2, 4
    w, _ = _weights(rng, Hk, Hv, cuda)
    qkv, z, a, b = (_dev(x, cuda) for x in _inputs(rng, (73,), Hk, Hv))
    zero = torch.tensor([0], dtype=torch.int32, device=cuda)
    taps = gdn_layer.new_taps(2, w, device=cuda)
    state = torch.zeros((2, Hv, 128, 128), dtype=torch.float32, device=cuda)
    slot0 = torch.tensor([0], dtype=torch.int32, device=cuda)
    slot1 = torch.tensor([1], dtype=torch.int32, device=cuda)
    gdn_layer.gdn_prefill(qkv[:70], z[:70], a[:70], b[:70], w, taps, state,
                          torch.tensor([0, 70], dtype=torch.int32, device=cuda), slot0, zero)
    outs = []
    for t in range(70, 73):
        pos = torch.tensor([t], dtype=torch.int32, device=cuda)
        outs.append(gdn_layer.gdn_decode_fused(qkv[t:t + 1], z[t:t + 1], a[t:t + 1],
                                               b[t:t + 1], w, taps, pos, state, slot0))
    full = gdn_layer.gdn_prefill(qkv, z, a, b, w, taps, state,
                                 torch.tensor([0, 73], dtype=torch.int32, device=cuda), slot1,
                                 zero)
    torch.cuda.synchronize()
    assert torch.equal(gdn_layer.ring_window(taps, 0, 73), gdn_layer.ring_window(taps, 1, 73))
    assert (state[0] - state[1]).abs().max().item() <= 2e-3
    np.testing.assert_allclose(torch.cat(outs).float().cpu().numpy(),
                               full[70:].float().cpu().numpy(), rtol=3e-2, atol=3e-2)


def test_gdn_inner_reference_call_site(cuda):
    """The reference signature: taps [B, 3, C] in and out, L = 1 and L > 1."""
    rng = np.random.default_rng(21)
    Hk, Hv, B = 2, 4, 2
    w, weights_np = _weights(rng, Hk, Hv, cuda)
    C = w.channels
    for L in (1, 9):
        qkv, z, a, b = _inputs(rng, (B, L), Hk, Hv)
        taps3 = bf(rng.standard_normal((B, 3, C)).astype(np.float32))
        s0 = (rng.standard_normal((B, Hv, 128, 128)) * 0.1).astype(np.float32)
        state = torch.from_numpy(s0).to(cuda)
        mixed, taps_out, nxt = gdn_layer.gdn_inner(
            None, _dev(qkv, cuda), _dev(z, cuda), _dev(a, cuda), _dev(b, cuda),
            _dev(taps3, cuda), state, decode_one=L == 1, weights=w)
        assert nxt is state and mixed.shape == (B, L, Hv * 128)
        for r in range(B):
            _, want_out, want_taps, want_s = _oracle_prefill(qkv[r], z[r], a[r], b[r], taps3[r],
                                                             s0[r], weights_np, Hk, Hv)
            assert np.array_equal(taps_out[r].float().cpu().numpy(), want_taps)
            np.testing.assert_allclose(mixed[r].float().cpu().numpy(), want_out, rtol=3e-2,
                                       atol=3e-2)
            assert np.abs(state[r].cpu().numpy() - want_s).max() <= 2e-2


@pytest.mark.parametrize("width", [128, 256])
def test_gated_rmsnorm_matches_oracle(cuda, width):
    rng = np.random.default_rng(width)
    y = bf(rng.standard_normal((1000, width)).astype(np.float32) * 3)
    z = bf(rng.standard_normal((1000, width)).astype(np.float32))
    wt = bf((1 + 0.1 * rng.standard_normal(width)).astype(np.float32))
    got = gdn_layer.gated_rmsnorm(_dev(y, cuda), _dev(z, cuda), _dev(wt, cuda), 1e-6)
    _close_bf16(got.float().cpu().numpy(), ofront.gated_rms_norm(y, z, wt, 1e-6), "gated")


@pytest.mark.parametrize("fused", [False, True])
def test_engine_runs_layers_from_projections_and_forks_taps(cuda, fused):
    """HybridCacheEngine with tap rings: prefill two prompts from their projections,
    decode two steps, snapshot one sequence and fork it; the fork's next step equals
    the original's next step on the same inputs (state, taps and output)."""
    from shellsmith_b200.engine import HybridCacheEngine, HybridConfig

    rng = np.random.default_rng(33)
    Hk, Hv = 2, 4
    cfg = HybridConfig(layers=4, gdn_key_heads=Hk, gdn_value_heads=Hv, q_heads=8, kv_heads=2,
                       head_dim=128, max_seqs=4, num_pages=32, max_context=256,
                       snapshot_rows=2, gdn_taps=True, gdn_glue_fused=fused)
    eng = HybridCacheEngine(cfg, device=cuda)
    weights = {l: _weights(rng, Hk, Hv, cuda) for l in cfg.gdn_layers}
    lengths = [21, 40]
    slots = [eng.admit(f"s{i}", L) for i, L in enumerate(lengths)]
    total = sum(lengths)
    proj = {l: tuple(_dev(x, cuda) for x in _inputs(rng, (total,), Hk, Hv))
            for l in cfg.gdn_layers}
    kvs = {l: (torch.randn((total, 2, 128), device=cuda).to(torch.bfloat16),
               torch.randn((total, 2, 128), device=cuda).to(torch.bfloat16))
           for l in cfg.attention_layers}
    eng.prefill_front(list(zip(slots, lengths)), lambda l, n: (*proj[l], weights[l][0]),
                      lambda l, n: kvs[l])
    ref = {}
    offs = [0, 21, 61]
    for l in cfg.gdn_layers:
        for i, slot in enumerate(slots):
            sl = slice(offs[i], offs[i + 1])
            qkv, z, a, b = (x[sl].float().cpu().numpy() for x in proj[l])
            _, _, taps3, s = _oracle_prefill(qkv, z, a, b, np.zeros((3, (2 * Hk + Hv) * 128),
                                                                    np.float32),
                                             np.zeros((Hv, 128, 128)), weights[l][1], Hk, Hv)
            ref[l, slot] = (taps3, s)

    def step(rows):
        """One decode step: inputs for every active row; returns GDN outputs per layer."""
        eng.begin_step()
        outs = {}
        for l in range(cfg.layers):
            if cfg.is_attention(l):
                q = torch.randn((cfg.max_seqs, 8, 128), device=cuda).to(torch.bfloat16)
                kn = torch.randn((cfg.max_seqs, 2, 128), device=cuda).to(torch.bfloat16)
                out = torch.empty_like(q)
                eng.attention_layer(l, q, kn, kn, out)
            else:
                qkv, z, a, b = (_dev(x, cuda) for x in rows[l])
                out = torch.empty((cfg.max_seqs, Hv * 128), dtype=torch.bfloat16, device=cuda)
                eng.gdn_layer_front(l, qkv, z, a, b, weights[l][0], out)
                outs[l] = out
        return outs

    for _ in range(2):
        rows = {l: _inputs(rng, (cfg.max_seqs,), Hk, Hv) for l in cfg.gdn_layers}
        outs = step(rows)
        for l in cfg.gdn_layers:
            for slot in slots:
                taps3, s = ref[l, slot]
                r = [x[slot:slot + 1] for x in rows[l]]
                want, taps3, s = ofront.decode_layer(*r, taps3[None], s[None], *weights[l][1],
                                                     1e-6, Hk, Hv)
                ref[l, slot] = (taps3[0], s[0])
                np.testing.assert_allclose(outs[l][slot].float().cpu().numpy(), want[0],
                                           rtol=3e-2, atol=3e-2)
    torch.cuda.synchronize()
    for l in cfg.gdn_layers:
        i = eng.gdn_index[l]
        for slot in slots:
            pos = int(eng.blocks.lengths[slot])
            assert np.array_equal(gdn_layer.ring_window(eng.taps[i], slot, pos).float().cpu()
                                  .numpy(), ref[l, slot][0])
            assert np.abs(eng.state[i, slot].cpu().numpy() - ref[l, slot][1]).max() <= 2e-2

    # Fork sequence 1 and advance both on identical inputs.
    snap = eng.snapshot(slots[1])
    fork = eng.fork(snap)
    rows = {l: _inputs(rng, (cfg.max_seqs,), Hk, Hv) for l in cfg.gdn_layers}
    for l in cfg.gdn_layers:
        for x in rows[l]:
            x[fork] = x[slots[1]]
    outs = step(rows)
    torch.cuda.synchronize()
    for l in cfg.gdn_layers:
        i = eng.gdn_index[l]
        assert torch.equal(outs[l][fork], outs[l][slots[1]])
        assert torch.equal(eng.state[i, fork], eng.state[i, slots[1]])
        assert torch.equal(eng.taps[i, fork], eng.taps[i, slots[1]])
