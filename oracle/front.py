"""GDN layer glue around the recurrence on the CPU (TEST INFRASTRUCTURE, see oracle/__init__).

The decode-time GDN layer of the reference, between its projections and its
output projection (src/studio_compute/numerics/bf16.py:44-139, the unfused
branch that decode_one=True takes):

  convolution  concat(taps[B, K-1, C], qkv[B, L, C]) -> depthwise causal conv
               (MLX conv1d, kernel K = 4, weight [C, K, 1], no bias), then SiLU
               (bf16.py:78-79); the new taps are the last K-1 rows (:137)
  split        q | k | v along channels, heads of width 128 (:80-85)
  q/k norm     q = dk^-1 * rms_norm(q, eps=1e-6), k = dk^-1/2 * rms_norm(k)
               (the model's _normalize_qk; restated in
               src/shellsmith/mlx/ops.py:121-125)
  gates        beta = sigmoid(b); g = exp(-exp(A_log) * softplus(a + dt_bias)),
               every op in bf16 (bf16.py:98-102)
  update       gated_delta_token (bf16.py:103-108; recurrence in oracle.gdn)
  output       rms_norm(y, w, eps) * silu(z) (bf16.py:129-135)

Every MLX op on bf16 arrays computes in fp32 and rounds its result to bf16;
these functions round at the same points (one rounding per op: SiLU is
x * sigmoid(x), two ops, two roundings). The MLX ops themselves (conv1d,
fast.rms_norm, softplus) are library code that is not in the reference tree;
their definitions are restated here from MLX's documented semantics.
"""

from __future__ import annotations

import numpy as np

from .gdn import bf16_round as bf
from .gdn import token_step

CONV_K = 4


def sigmoid(x):
    return (1.0 / (1.0 + np.exp(-np.asarray(x, np.float64)))).astype(np.float32)


def silu_bf16(x):
    """nn.silu on bf16: x * sigmoid(x), each op rounded."""
    x = np.asarray(x, np.float32)
    return bf(x * bf(sigmoid(x)))


def rms_norm_bf16(x, weight, eps):
    """mx.fast.rms_norm over the last axis: fp32 math, one rounding."""
    x = np.asarray(x, np.float32).astype(np.float64)
    r = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)
    y = x * r if weight is None else x * r * np.asarray(weight, np.float64)
    return bf(y.astype(np.float32))


def causal_conv_silu(window, weight):
    """window [..., K, C] (oldest row first), weight [C, K] -> silu(conv) [..., C]."""
    w = np.asarray(weight, np.float64)
    y = np.einsum("...kc,ck->...c", np.asarray(window, np.float64), w)
    return silu_bf16(bf(y.astype(np.float32)))


def normalize_qk(q, k):
    """q [.., H, dk] -> dk^-1 rms_norm(q); k -> dk^-1/2 rms_norm(k) (bf16 scalars)."""
    inv_scale = q.shape[-1] ** -0.5          # a Python float, cast to bf16 by MLX
    q = bf(rms_norm_bf16(q, None, 1e-6) * bf(np.float32(inv_scale ** 2)))
    k = bf(rms_norm_bf16(k, None, 1e-6) * bf(np.float32(inv_scale)))
    return q, k


def gates_bf16(a, b, a_log, dt_bias):
    """beta = sigmoid(b); g = exp(-exp(A_log) softplus(a + dt_bias)), each op in bf16."""
    a, b = bf(a), bf(b)
    x = bf(a + bf(dt_bias))
    sp = bf(np.logaddexp(x.astype(np.float64), 0.0).astype(np.float32))
    decay_rate = bf(np.exp(bf(a_log).astype(np.float64)).astype(np.float32))
    g = bf(np.exp(bf(-decay_rate * sp).astype(np.float64)).astype(np.float32))
    beta = bf(sigmoid(b))
    return g, beta


LOG_GATE_MIN = np.float32(np.log(1e-6))    # the chunk path clamps a gate at 1e-6


def _f32(x):
    """A float64 result rounded to float32: one correctly rounded fp32 operation."""
    return np.asarray(x, np.float64).astype(np.float32)


def _near_bf16_tie(x64, margin=2.0 ** -19):
    """True where a value about to be rounded to bf16 lies within `margin` (relative,
    16 fp32 ulps) of a bf16 rounding boundary: a device exp or log that is a few fp32
    ulps from the correctly rounded result may round to the other bf16 there."""
    x = np.abs(np.asarray(x64, np.float64))
    with np.errstate(divide="ignore", invalid="ignore"):
        e = np.floor(np.log2(np.where(x > 0, x, 1.0)))
        frac = x / 2.0 ** e * 128.0                # 7 stored mantissa bits of bf16
        dist = np.abs(frac - np.floor(frac) - 0.5) / 128.0
    return np.isfinite(x) & (x > 0) & (dist < margin)


def sampler_gates(a, b, a_log, dt_bias):
    """The gates of the fused chunk path from their logits: `sampler_gate` and
    `sampler_beta` of src/studio_compute/numerics/metal/gdn_chunk_common.metal:61-75,
    called per chunk row by `load_gates` (:79-96) for gdn_fused.py:86-122
    `gated_delta_chunks`. Every step is fp32 and rounded to bf16 as MLX does:

        scale = bf16(exp(bf16(a_log)))
        x     = bf16(a + bf16(dt_bias))
        sp    = bf16(max(x, 0) + log(1 + exp(-|x|)))
        gate  = bf16(exp(bf16(-scale * sp)))
        log_gate = log(1e-6) if gate < 1e-6 else log(gate)      (fp32)
        beta  = bf16(1 / (1 + exp(-b)))

    a, b [..., H] (bf16 values, +-inf allowed: a padded row has a = b = -inf, which
    gives gate 1 and beta 0); a_log, dt_bias [H] fp32. Returns float32 arrays
    (gate, log_gate, beta) and `tie` [..., H] bool: elements where one of the steps
    rounds a value within 16 fp32 ulps of a bf16 rounding boundary, so a device exp or
    log a few ulps from the correctly rounded result may give the neighbouring bf16
    (every other element is determined bit for bit). exp and log here are correctly
    rounded fp32 operations (float64 math, one rounding)."""
    a = bf(np.asarray(a, np.float32))
    b = bf(np.asarray(b, np.float32))
    a_log = np.asarray(a_log, np.float32)
    dt_bias = np.asarray(dt_bias, np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        e_scale = np.exp(bf(a_log).astype(np.float64))
        scale = bf(_f32(e_scale))
        x = bf(_f32(a.astype(np.float64) + bf(dt_bias).astype(np.float64)))
        e = _f32(np.exp(-np.abs(x.astype(np.float64))))
        t = _f32(1.0 + e.astype(np.float64))
        lg = _f32(np.log(t.astype(np.float64)))
        sp64 = np.maximum(x, np.float32(0)).astype(np.float64) + lg.astype(np.float64)
        sp = bf(_f32(sp64))
        arg = bf(_f32(-scale.astype(np.float64) * sp.astype(np.float64)))
        g64 = np.exp(arg.astype(np.float64))
        gate = bf(_f32(g64))
        clamped = gate < np.float32(1e-6)
        log_gate = np.where(clamped, LOG_GATE_MIN,
                            _f32(np.log(np.where(clamped, 1.0, gate).astype(np.float64))))
        eb = _f32(np.exp(-b.astype(np.float64)))
        beta64 = 1.0 / _f32(1.0 + eb.astype(np.float64)).astype(np.float64)
        beta = bf(_f32(beta64))
    tie = (_near_bf16_tie(e_scale) | _near_bf16_tie(sp64) | _near_bf16_tie(g64)
           | _near_bf16_tie(beta64))
    return gate, log_gate.astype(np.float32), beta, np.broadcast_to(tie, gate.shape)


def split_heads(x, Hk, Hv, dk=128, dv=128):
    """Channels q | k | v -> q, k [..., Hk, dk], v [..., Hv, dv]."""
    q = x[..., :Hk * dk].reshape(*x.shape[:-1], Hk, dk)
    k = x[..., Hk * dk:2 * Hk * dk].reshape(*x.shape[:-1], Hk, dk)
    v = x[..., 2 * Hk * dk:].reshape(*x.shape[:-1], Hv, dv)
    return q, k, v


def front(qkv, a, b, taps, conv_w, a_log, dt_bias, Hk, Hv):
    """A run of L tokens per row: qkv [B, L, C], a, b [B, L, Hv], taps [B, K-1, C].

    Returns q, k [B, L, Hk, 128], v [B, L, Hv, 128], g, beta [B, L, Hv] (all
    bf16-representable float32) and the new taps [B, K-1, C].
    """
    qkv = np.asarray(qkv, np.float32)
    full = np.concatenate([np.asarray(taps, np.float32), qkv], axis=1)     # [B, K-1+L, C]
    L = qkv.shape[1]
    windows = np.stack([full[:, t:t + CONV_K] for t in range(L)], axis=1)  # [B, L, K, C]
    conv = causal_conv_silu(windows, conv_w)
    q, k, v = split_heads(conv, Hk, Hv)
    q, k = normalize_qk(q, k)
    g, beta = gates_bf16(a, b, a_log, dt_bias)
    return q, k, v, g, beta, full[:, -(CONV_K - 1):].copy()


def gated_rms_norm(y, z, weight, eps):
    """rms_norm(y, w, eps) * silu(z) over the last axis, with bf16.py:129-135 roundings."""
    return bf(rms_norm_bf16(y, weight, eps) * silu_bf16(z))


def decode_layer(qkv, z, a, b, taps, state, conv_w, a_log, dt_bias, norm_w, eps, Hk, Hv):
    """One decode token of one GDN layer for B rows, fp32 state (float64 recurrence).

    qkv [B, C], z [B, Hv*128], a, b [B, Hv], taps [B, K-1, C], state [B, Hv, 128, 128].
    Returns (out [B, Hv*128], new taps, new state).
    """
    q, k, v, g, beta, new_taps = front(np.asarray(qkv)[:, None], np.asarray(a)[:, None],
                                       np.asarray(b)[:, None], taps, conv_w, a_log, dt_bias,
                                       Hk, Hv)
    y, new_state = token_step(q[:, 0], k[:, 0], v[:, 0], g[:, 0], beta[:, 0], state)
    y = bf(np.asarray(y, np.float32))
    B = y.shape[0]
    out = gated_rms_norm(y, np.asarray(z, np.float32).reshape(B, Hv, -1), norm_w, eps)
    return out.reshape(B, -1), new_taps, new_state
