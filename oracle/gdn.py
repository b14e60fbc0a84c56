"""Gated-delta-net recurrence on the CPU (TEST INFRASTRUCTURE, see oracle/__init__).

Shapes (reference naming): B batch, T tokens, Hk key heads, Hv value heads,
dk key width, dv value width. The state is S[b, h, i, j] = S[value i, key j]
(the reference's [B, Hv, Dv, Dk] value-major layout, gdn_token.py:31).

The recurrence, with a = g the multiplicative decay of a token:
    S_t = g_t S_{t-1} + beta_t (v_t - g_t S_{t-1} k_t) k_t^T,   o_t = S_t q_t

Restated from (reference paths relative to the shellsmith project root):
  sequential      tests/test_gdn_sequential.py:17-36 (forward half of
                  `sequential`: repeat key heads, decay, delta rule, output)
  token_step      the one-token form of the same equations, as
                  tests/test_bf16_token_decode.py:27-35 states it
  token_step_bf16 src/studio_compute/numerics/gdn_token.py:60-77 rounding
                  points: fp32 decayed state and sums, bf16 updated state,
                  output from the rounded state
  chunked         src/studio_compute/numerics/ops.py:151-215
                  (`gated_delta_chunked`, backend "reference") with
                  `_invert_unit_lower` (ops.py:54-85, here an exact forward
                  substitution) and `_scan_forward` (ops.py:88-104)
  gates           src/studio_compute/numerics/bf16.py:98-102 and
                  tests/test_gdn_chunk.py:46-53 (fp32 gates from logits)
"""

from __future__ import annotations

import numpy as np


def bf16_round(x) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), as float32."""
    x = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    bits = x.view(np.uint32).astype(np.uint64)
    bits = ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16) << 16
    return bits.astype(np.uint32).view(np.float32).reshape(x.shape)


def _repeat_heads(x: np.ndarray, groups: int) -> np.ndarray:
    # Value head h reads key head h // groups (gdn_token.py:57, np.repeat order).
    return np.repeat(x, groups, axis=2) if groups > 1 else x


def sequential(q, k, v, g, beta, state, dtype=np.float64):
    """Token-by-token recurrence. Returns (y [B,T,Hv,dv], final state [B,Hv,dv,dk])."""
    q, k, v, g, beta, s = (np.asarray(x, dtype=dtype) for x in (q, k, v, g, beta, state))
    groups = v.shape[2] // q.shape[2]
    q, k = _repeat_heads(q, groups), _repeat_heads(k, groups)
    s = s.copy()
    ys = []
    for t in range(v.shape[1]):
        decayed = g[:, t, :, None, None] * s
        predicted = np.einsum("bhij,bhj->bhi", decayed, k[:, t])
        delta = beta[:, t, :, None] * (v[:, t] - predicted)
        s = decayed + delta[..., None] * k[:, t, :, None, :]
        ys.append(np.einsum("bhij,bhj->bhi", s, q[:, t]))
    return np.stack(ys, axis=1), s


def token_step(q, k, v, g, beta, state, dtype=np.float64):
    """One token: q, k [B,Hk,dk]; v [B,Hv,dv]; g, beta [B,Hv]; state [B,Hv,dv,dk]."""
    y, s = sequential(
        np.asarray(q)[:, None], np.asarray(k)[:, None], np.asarray(v)[:, None],
        np.asarray(g)[:, None], np.asarray(beta)[:, None], state, dtype=dtype,
    )
    return y[:, 0], s


def token_step_bf16(q, k, v, g, beta, state):
    """One token with the reference kernel's bf16 rounding points (fp32 math).

    Inputs are bf16-representable float32 arrays; returns (out, state), both
    rounded to bf16 and stored as float32.
    """
    q, k, v, g, beta, s = (np.asarray(x, dtype=np.float32) for x in (q, k, v, g, beta, state))
    groups = v.shape[1] // q.shape[1]
    q = np.repeat(q, groups, axis=1) if groups > 1 else q
    k = np.repeat(k, groups, axis=1) if groups > 1 else k
    decayed = (g[:, :, None, None] * s).astype(np.float32)
    predicted = np.einsum("bhij,bhj->bhi", decayed, k).astype(np.float32)
    delta = (beta[:, :, None] * (v - predicted)).astype(np.float32)
    updated = bf16_round(decayed + delta[..., None] * k[:, :, None, :])
    out = bf16_round(np.einsum("bhij,bhj->bhi", updated, q))
    return out, updated


def gates(a, b, a_log, dt_bias):
    """fp32 gates from logits: g = exp(-exp(A_log) softplus(a + dt_bias)), beta = sigmoid(b)."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    x = a + np.asarray(dt_bias, np.float64)
    softplus = np.maximum(x, 0.0) + np.log1p(np.exp(-np.abs(x)))
    log_gate = np.maximum(-np.exp(np.asarray(a_log, np.float64)) * softplus, np.log(1e-6))
    return np.exp(log_gate), 1.0 / (1.0 + np.exp(-b))


def _unit_lower_inverse(strict: np.ndarray) -> np.ndarray:
    """Inverse of I + strict (strict lower) over the last two axes, exact substitution."""
    n = strict.shape[-1]
    inv = np.zeros_like(strict)
    eye = np.eye(n, dtype=strict.dtype)
    for i in range(n):
        # Row i of (I + L) X = I: X_i = e_i - sum_{j<i} L_ij X_j.
        inv[..., i, :] = eye[i] - np.einsum("...j,...jk->...k", strict[..., i, :i], inv[..., :i, :])
    return inv


def chunk_transforms(q, k, v, g, beta, chunk=64, dtype=np.float64):
    """Intra-chunk WY/UT transforms of ops.py:151-199 (after head repeat and padding).

    Inputs are already [B, Hv, N, C, d] / [B, Hv, N, C]. Returns
    (mu0, q_eff, u0, kt, decay_last, ratio_last).
    """
    stable = np.clip(g, 1e-6, 1.0)
    log_decay = np.cumsum(np.log(stable), axis=-1)
    decay = np.exp(log_decay)
    c = q.shape[-2]
    lower = np.tril(np.ones((c, c), dtype=dtype))
    strict = np.tril(np.ones((c, c), dtype=dtype), -1)
    diff = log_decay[..., :, None] - log_decay[..., None, :]
    ratio = np.where(lower > 0, np.exp(np.where(lower > 0, diff, 0.0)), 0.0)
    kk = k @ np.swapaxes(k, -1, -2)
    a_strict = beta[..., :, None] * ratio * kk * strict
    x = _unit_lower_inverse(a_strict)
    u0 = x @ (beta[..., :, None] * v)
    kt = x @ ((beta * decay)[..., :, None] * k)
    m = ratio * (q @ np.swapaxes(k, -1, -2)) * lower
    q_eff = decay[..., :, None] * q - m @ kt
    mu0 = m @ u0
    return mu0, q_eff, u0, kt, decay[..., -1], np.exp(log_decay[..., -1:] - log_decay)


def scan_forward(mu0, q_eff, u0, kt, k, decay_last, ratio_last, state):
    """Inter-chunk recurrence of ops.py:88-104. Returns (outputs per chunk, final state)."""
    s = state
    outs = []
    for c in range(mu0.shape[2]):
        st = np.swapaxes(s, -1, -2)
        outs.append(mu0[:, :, c] + q_eff[:, :, c] @ st)
        uc = u0[:, :, c] - kt[:, :, c] @ st
        s = decay_last[:, :, c][..., None, None] * s + np.swapaxes(
            ratio_last[:, :, c][..., None] * uc, -1, -2) @ k[:, :, c]
    return np.stack(outs, axis=2), s


def chunked(q, k, v, g, beta, state, chunk=64, dtype=np.float64):
    """Chunked gated delta rule. Returns (y [B,T,Hv,dv], final state [B,Hv,dv,dk])."""
    q, k, v, g, beta, state = (np.asarray(x, dtype=dtype) for x in (q, k, v, g, beta, state))
    bsz, length, hk, dk = q.shape
    hv, dv = v.shape[-2:]
    groups = hv // hk
    q, k = _repeat_heads(q, groups), _repeat_heads(k, groups)
    pad = (chunk - length % chunk) % chunk
    if pad:
        q = np.concatenate([q, np.zeros((bsz, pad, hv, dk), dtype)], axis=1)
        k = np.concatenate([k, np.zeros((bsz, pad, hv, dk), dtype)], axis=1)
        v = np.concatenate([v, np.zeros((bsz, pad, hv, dv), dtype)], axis=1)
        g = np.concatenate([g, np.ones((bsz, pad, hv), dtype)], axis=1)
        beta = np.concatenate([beta, np.zeros((bsz, pad, hv), dtype)], axis=1)
    n = (length + pad) // chunk

    def blocks(x, width):
        return x.reshape(bsz, n, chunk, hv, width).transpose(0, 3, 1, 2, 4)

    qb, kb, vb = blocks(q, dk), blocks(k, dk), blocks(v, dv)
    gb = g.reshape(bsz, n, chunk, hv).transpose(0, 3, 1, 2)
    bb = beta.reshape(bsz, n, chunk, hv).transpose(0, 3, 1, 2)
    mu0, q_eff, u0, kt, decay_last, ratio_last = chunk_transforms(qb, kb, vb, gb, bb, chunk, dtype)
    y, s = scan_forward(mu0, q_eff, u0, kt, kb, decay_last, ratio_last, state)
    y = y.transpose(0, 2, 3, 1, 4).reshape(bsz, length + pad, hv, dv)[:, :length]
    return y, s
