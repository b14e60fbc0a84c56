"""Attention on the CPU (TEST INFRASTRUCTURE, see oracle/__init__).

Restated from (paths relative to the shellsmith project root):
  attention   scripts/mlx_attention_qualify.py:234-275 `numpy_attention`
              (forward half): causal GQA, key j visible to query i when
              j <= query_offset + i, kv head of query head h is h // group,
              query_offset defaults to keys - queries.
  quantize_q8 the 8-bit cache of the cache_precision="8bit" option
              (src/studio_compute/inference.py:87-94, mlx-vlm 0.7.4
              QuantizedKVCache over mlx 0.32.3 mx.quantize: groups of 64 along
              D, scale and bias per group, w = scale * code + bias). The
              library's code is not in the reference tree; this restates the
              affine rule MLX documents for mx.quantize (scale = (max - min) /
              (2^bits - 1), bias = min, code = round((w - bias) / scale)) with
              scale and bias stored in the cache's bf16 dtype:
              scale = bf16((max - min) / 255), bias = bf16(min),
              code = clamp(rint((w - bias) / scale), 0, 255), 0 when
              scale == 0, each op in float32. Parity with the library itself is
              unpinned (it cannot run here).
  The split-K partials, their combine and the paged-pool layout have no
  counterpart in the reference (it runs one request's SDPA at a time); they
  restate the algebra softmax(x) = sum_s e^{lse_s - M} softmax_s(x) / sum_s
  e^{lse_s - M} and the pool layout documented in include/shellcache.h.
"""

from __future__ import annotations

import numpy as np


def attention(q, k, v, scale, query_offset=None):
    """q [B,Hq,Q,D], k/v [B,Hkv,K,D] -> (out [B,Hq,Q,D], lse [B,Hq,Q]) in float64."""
    q, k, v = (np.asarray(x, dtype=np.float64) for x in (q, k, v))
    bsz, heads, queries, _ = q.shape
    kv_heads, keys = k.shape[1:3]
    assert heads % kv_heads == 0 and queries <= keys
    offset = keys - queries if query_offset is None else query_offset
    assert 0 <= offset <= keys - queries
    visible = np.arange(keys)[None, :] <= (offset + np.arange(queries))[:, None]
    group = heads // kv_heads
    out = np.empty_like(q)
    lse = np.empty((bsz, heads, queries))
    for b in range(bsz):
        for h in range(heads):
            j = h // group
            scores = np.where(visible, (q[b, h] * scale) @ k[b, j].T, -np.inf)
            top = scores.max(axis=-1, keepdims=True)
            weights = np.exp(scores - top)
            total = weights.sum(axis=-1, keepdims=True)
            out[b, h] = (weights / total) @ v[b, j]
            lse[b, h] = (top + np.log(total))[:, 0]
    return out, lse


def decode_attention(q, k, v, scale):
    """One sequence, one query: q [Hq,D], k/v [L,Hkv,D] -> (out [Hq,D], lse [Hq])."""
    q = np.asarray(q, np.float64)
    if k.shape[0] == 0:
        return np.zeros_like(q), np.full(q.shape[0], -np.inf)
    out, lse = attention(q[None, :, None, :], np.asarray(k).transpose(1, 0, 2)[None],
                         np.asarray(v).transpose(1, 0, 2)[None], scale)
    return out[0, :, 0], lse[0, :, 0]


def split_partials(q, k, v, scale, tokens_per_split):
    """Normalised partial outputs and lse of consecutive key ranges (one sequence)."""
    parts_o, parts_lse = [], []
    for start in range(0, k.shape[0], tokens_per_split):
        o, l = decode_attention(q, k[start:start + tokens_per_split],
                                v[start:start + tokens_per_split], scale)
        parts_o.append(o)
        parts_lse.append(l)
    return np.stack(parts_o, axis=-2), np.stack(parts_lse, axis=-1)


def combine(parts_o, parts_lse):
    """parts_o [..., S, D], parts_lse [..., S] -> (out [..., D], lse [...])."""
    parts_o = np.asarray(parts_o, np.float64)
    parts_lse = np.asarray(parts_lse, np.float64)
    top = parts_lse.max(axis=-1, keepdims=True)
    safe = np.where(np.isfinite(top), top, 0.0)
    w = np.where(np.isfinite(parts_lse), np.exp(parts_lse - safe), 0.0)
    total = w.sum(axis=-1, keepdims=True)
    out = np.where(total > 0, (w[..., None] * parts_o).sum(axis=-2) / np.maximum(total, 1e-300),
                   0.0)
    lse = np.where(total[..., 0] > 0, (safe + np.log(np.maximum(total, 1e-300)))[..., 0], -np.inf)
    return out, lse


def pool_offsets(slot, kv_head, which, Hkv, P, D, chunk):
    """Element offset of 16-byte chunk `chunk` of a token row in the pool layout."""
    page, off = divmod(int(slot), P)
    row = (((page * Hkv + kv_head) * 2 + which) * P + off) * D
    return row + 8 * (chunk ^ (off & 7))


def pool_write(pool_flat, slots, k, v, Hkv, P, D):
    """Scatter k/v [ntok,Hkv,D] into a flat pool array (uint16 / float bits)."""
    for i, slot in enumerate(slots):
        if slot < 0:
            continue
        for h in range(Hkv):
            for which, src in ((0, k), (1, v)):
                for c in range(D // 8):
                    o = pool_offsets(slot, h, which, Hkv, P, D, c)
                    pool_flat[o:o + 8] = src[i, h, 8 * c:8 * c + 8]


def pool_read(pool_flat, slots, Hkv, P, D):
    """Gather logical k/v [ntok,Hkv,D] from a flat pool array."""
    n = len(slots)
    k = np.zeros((n, Hkv, D), dtype=pool_flat.dtype)
    v = np.zeros((n, Hkv, D), dtype=pool_flat.dtype)
    for i, slot in enumerate(slots):
        if slot < 0:
            continue
        for h in range(Hkv):
            for which, dst in ((0, k), (1, v)):
                for c in range(D // 8):
                    o = pool_offsets(slot, h, which, Hkv, P, D, c)
                    dst[i, h, 8 * c:8 * c + 8] = pool_flat[o:o + 8]
    return k, v


def pool_read_pages(pool, pages, length, Hkv, P, D):
    """Logical k/v [length,Hkv,D] of one sequence from a [num_pages,Hkv,2,P,D] pool array."""
    k = np.zeros((length, Hkv, D), dtype=pool.dtype)
    v = np.zeros((length, Hkv, D), dtype=pool.dtype)
    chunks = np.arange(D // 8)
    for t in range(length):
        page, off = pages[t // P], t % P
        perm = (chunks ^ (off & 7))
        for which, dst in ((0, k), (1, v)):
            row = pool[page, :, which, off].reshape(Hkv, D // 8, 8)
            dst[t] = row[:, perm].reshape(Hkv, D)
    return k, v


def quantize_q8(x, group=64):
    """x [..., D] (float32 values) -> codes uint8 [..., D], scale, bias [..., D/group]."""
    from .gdn import bf16_round

    x = np.asarray(x, np.float32)
    g = x.reshape(*x.shape[:-1], x.shape[-1] // group, group)
    mn, mx = g.min(axis=-1), g.max(axis=-1)
    scale = bf16_round((mx - mn) / np.float32(255.0))
    bias = bf16_round(mn)
    with np.errstate(divide="ignore", invalid="ignore"):
        codes = np.rint((g - bias[..., None]) / scale[..., None])
    codes = np.where(scale[..., None] > 0, np.clip(codes, 0, 255), 0).astype(np.uint8)
    return codes.reshape(x.shape), scale, bias


def dequantize_q8(codes, scale, bias, group=64):
    """scale * code + bias per group, in float64."""
    c = np.asarray(codes, np.float64)
    g = c.reshape(*c.shape[:-1], c.shape[-1] // group, group)
    out = g * np.asarray(scale, np.float64)[..., None] + np.asarray(bias, np.float64)[..., None]
    return out.reshape(c.shape)
