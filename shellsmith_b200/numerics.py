"""GDN recurrent-state kernels behind the reference's call-site names.

Mirrors studio_compute/numerics (reference paths relative to the shellsmith
project root):
  gated_delta_token    numerics/gdn_token.py:18-42 -- same argument names,
                       layouts and assertion behaviour; the state may be
                       bf16 (reference rounding) or fp32 (this build's
                       default), and it is updated IN PLACE (the returned
                       next state is the same tensor). The reference returns
                       a new array and its caller drops the old one
                       (mlx_decode.py:53,59-60), so the two are observably
                       equivalent at that call site.
  gdn_decode           the batched engine form: [B, H, d] rows, per-row state
                       slots into a persistent [slots, Hv, dv, dk] pool.
"""

from __future__ import annotations

import torch

from . import _capi
from ._torch import ptr, require_cuda, stream_of


def gdn_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
               beta: torch.Tensor, state: torch.Tensor, state_slot: torch.Tensor | None = None,
               out: torch.Tensor | None = None, chained: bool = False) -> torch.Tensor:
    """One-token GDN update of rows b (state row state_slot[b]), in place.

    q, k [B, Hk, dk] bf16; v [B, Hv, dv] bf16; g (decay), beta [B, Hv] fp32;
    state [slots, Hv, dv, dk] fp32 or bf16; state_slot [B] int32 or None
    (identity). Returns out [B, Hv, dv] bf16. chained (fp32 state): the work
    queued just before this call does not write these state rows (another
    layer's update, an attention layer), so the state may stream in early.
    """
    B, Hk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    for name, t in (("q", q), ("k", k), ("v", v)):
        require_cuda(name, t, torch.bfloat16, 3, align=8)
    for name, t in (("g", g), ("beta", beta)):
        require_cuda(name, t, torch.float32, 2, align=4)
    if k.shape != q.shape or v.shape[0] != B or g.shape != (B, Hv) or beta.shape != (B, Hv):
        raise ValueError("gdn_decode: inconsistent shapes")
    if state.dim() != 4 or tuple(state.shape[1:]) != (Hv, dv, dk):
        raise ValueError(f"gdn_decode: state must be [slots, {Hv}, {dv}, {dk}]")
    if state_slot is None and state.shape[0] < B:
        raise ValueError("gdn_decode: state has fewer slots than rows")
    if state_slot is not None:
        require_cuda("state_slot", state_slot, torch.int32, 1, align=4)
        if state_slot.shape[0] != B:
            raise ValueError("gdn_decode: state_slot must have one entry per row")
    if out is None:
        out = torch.empty((B, Hv, dv), dtype=torch.bfloat16, device=q.device)
    require_cuda("out", out, torch.bfloat16, 3, align=2)
    if state.dtype == torch.float32:
        require_cuda("state", state, torch.float32, 4)
        name = "sc_gdn_decode_chained" if chained else "sc_gdn_decode"
    elif state.dtype == torch.bfloat16:
        require_cuda("state", state, torch.bfloat16, 4, align=8)
        name = "sc_gdn_decode_bf16"
    else:
        raise TypeError("gdn_decode: state must be float32 or bfloat16")
    _capi.call(name, ptr(q), ptr(k), ptr(v), ptr(g), ptr(beta), ptr(state), ptr(state_slot),
               ptr(out), B, Hk, Hv, dk, dv, state.shape[0], stream_of(q))
    return out


def gated_delta_token(q_BLJK: torch.Tensor, k_BLJK: torch.Tensor, v_BLHV: torch.Tensor,
                      g_BLH: torch.Tensor, beta_BLH: torch.Tensor,
                      state_BHVK: torch.Tensor) -> tuple:
    """Apply the sequential recurrence for one autoregressive token.

    Same contract as the reference (gdn_token.py:18-42): exactly one row,
    keys % 32 == 0, heads % key_heads == 0, bf16 q/k/v. g and beta may be
    bf16 (reference) or fp32; the state may be bf16 (reference rounding) or
    fp32. Returns (output [B,1,Hv,dv] bf16, state) with the state advanced in
    place.
    """
    batch, length, key_heads, keys = q_BLJK.shape
    heads, values = v_BLHV.shape[-2:]
    assert length == 1 and keys % 32 == 0 and heads % key_heads == 0
    assert k_BLJK.shape == q_BLJK.shape and v_BLHV.shape[:2] == (batch, 1)
    assert g_BLH.shape == beta_BLH.shape == (batch, 1, heads)
    assert state_BHVK.shape == (batch, heads, values, keys)
    assert all(x.dtype == torch.bfloat16 for x in (q_BLJK, k_BLJK, v_BLHV))
    assert g_BLH.dtype in (torch.bfloat16, torch.float32)
    assert beta_BLH.dtype in (torch.bfloat16, torch.float32)
    assert state_BHVK.dtype in (torch.bfloat16, torch.float32)
    out = gdn_decode(
        q_BLJK.reshape(batch, key_heads, keys).contiguous(),
        k_BLJK.reshape(batch, key_heads, keys).contiguous(),
        v_BLHV.reshape(batch, heads, values).contiguous(),
        g_BLH.reshape(batch, heads).float().contiguous(),
        beta_BLH.reshape(batch, heads).float().contiguous(),
        state_BHVK,
    )
    return out.reshape(batch, 1, heads, values), state_BHVK


def gdn_chunk_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                      beta: torch.Tensor, state: torch.Tensor,
                      state_slot: torch.Tensor | None = None,
                      cu_seqlens: torch.Tensor | None = None, *, T: int | None = None,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """Chunked (64) GDN prefill of packed sequences on the tensor cores, state in place.

    q, k [tokens, Hk, 128] bf16; v [tokens, Hv, 128] bf16; g (decay), beta
    [tokens, Hv] fp32; state [slots, Hv, 128, 128] fp32. Sequence b is rows
    cu_seqlens[b]:cu_seqlens[b+1] (int32 [B+1]), or b*T:(b+1)*T when
    cu_seqlens is None. Returns out [tokens, Hv, 128] bf16.
    """
    tokens, Hk, dk = q.shape
    Hv, dv = v.shape[1], v.shape[2]
    for name, t in (("q", q), ("k", k), ("v", v)):
        require_cuda(name, t, torch.bfloat16, 3)
    for name, t in (("g", g), ("beta", beta)):
        require_cuda(name, t, torch.float32, 2, align=4)
    require_cuda("state", state, torch.float32, 4)
    if k.shape != q.shape or v.shape[0] != tokens or g.shape != (tokens, Hv) \
            or beta.shape != (tokens, Hv):
        raise ValueError("gdn_chunk_prefill: inconsistent shapes")
    if tuple(state.shape[1:]) != (Hv, dv, dk):
        raise ValueError(f"gdn_chunk_prefill: state must be [slots, {Hv}, {dv}, {dk}]")
    if cu_seqlens is None:
        if T is None or T <= 0 or tokens % T:
            raise ValueError("gdn_chunk_prefill: give cu_seqlens or a T dividing the tokens")
        B = tokens // T
    else:
        require_cuda("cu_seqlens", cu_seqlens, torch.int32, 1, align=4)
        B = cu_seqlens.shape[0] - 1
        T = 0
    if state_slot is not None:
        require_cuda("state_slot", state_slot, torch.int32, 1, align=4)
        if state_slot.shape[0] != B:
            raise ValueError("gdn_chunk_prefill: one state slot per sequence")
    elif state.shape[0] < B:
        raise ValueError("gdn_chunk_prefill: state has fewer slots than sequences")
    if out is None:
        out = torch.empty((tokens, Hv, dv), dtype=torch.bfloat16, device=q.device)
    require_cuda("out", out, torch.bfloat16, 3, align=2)
    _capi.call("sc_gdn_chunk_prefill", ptr(q), ptr(k), ptr(v), ptr(g), ptr(beta), ptr(state),
               ptr(state_slot), ptr(cu_seqlens), ptr(out), B, T, tokens, Hk, Hv, dk, dv,
               state.shape[0], stream_of(q))
    return out


def gated_delta_chunked(q, k, v, g, beta, state, chunk=64, *, compute_dtype=None,
                        backend=None) -> tuple:
    """Chunked gated delta rule with the reference's signature (ops.py:151).

    q, k [B, T, Hk, 128], v [B, T, Hv, 128] bf16; g (decay), beta [B, T, Hv];
    state [B, Hv, 128, 128]. Returns (y [B, T, Hv, 128] in v's dtype, final
    fp32 state). The chunk is 64 and the arithmetic is fixed (fp32
    accumulation, split-bf16 operands); `compute_dtype` and `backend` are
    accepted for call-site compatibility. An fp32 contiguous state is
    advanced in place and returned; any other state is copied first.
    """
    if chunk != 64:
        raise ValueError("gated_delta_chunked: the tensor-core kernel uses chunk = 64")
    B, T, Hk, dk = q.shape
    Hv, dv = v.shape[-2:]
    assert k.shape == q.shape and v.shape[:2] == (B, T) and Hv % Hk == 0
    assert g.shape == beta.shape == (B, T, Hv) and state.shape == (B, Hv, dv, dk)
    s = state if (state.dtype == torch.float32 and state.is_contiguous()) else \
        state.float().contiguous()
    y = gdn_chunk_prefill(
        q.to(torch.bfloat16).reshape(B * T, Hk, dk).contiguous(),
        k.to(torch.bfloat16).reshape(B * T, Hk, dk).contiguous(),
        v.to(torch.bfloat16).reshape(B * T, Hv, dv).contiguous(),
        g.float().reshape(B * T, Hv).contiguous(), beta.float().reshape(B * T, Hv).contiguous(),
        s, T=T)
    return y.reshape(B, T, Hv, dv).to(v.dtype), s


def gdn_sampler_gates(a: torch.Tensor, b: torch.Tensor, a_log: torch.Tensor,
                      dt_bias: torch.Tensor) -> tuple:
    """Gates of the fused chunk path from their logits (sc_gdn_sampler_gates).

    a, b [..., Hv] bf16 (gate and beta logits; -inf marks a padded row: gate 1,
    beta 0); a_log, dt_bias [Hv] fp32. Returns (g, beta) fp32 of a's shape: g is
    the bf16 gate value exp(-exp(A_log) softplus(a + dt_bias)) and beta =
    sigmoid(b), each step rounded to bf16 as the reference's sampler_gate /
    sampler_beta round them (numerics/metal/gdn_chunk_common.metal:61-75).
    """
    Hv = a.shape[-1]
    require_cuda("a", a, torch.bfloat16, None, align=2)
    require_cuda("b", b, torch.bfloat16, None, align=2)
    for name, t in (("a_log", a_log), ("dt_bias", dt_bias)):
        require_cuda(name, t, torch.float32, 1, align=4)
        if t.shape[0] != Hv:
            raise ValueError(f"gdn_sampler_gates: {name} must be [{Hv}]")
    if b.shape != a.shape:
        raise ValueError("gdn_sampler_gates: a and b must have the same shape")
    g = torch.empty(a.shape, dtype=torch.float32, device=a.device)
    beta = torch.empty_like(g)
    _capi.call("sc_gdn_sampler_gates", ptr(a), ptr(b), ptr(a_log), ptr(dt_bias), ptr(g),
               ptr(beta), a.numel() // max(1, Hv), Hv, stream_of(a))
    return g, beta


HEAD_WIDTH = 128


def gated_delta_chunks(q_BLGD: torch.Tensor, k_BLGD: torch.Tensor, v_BLHD: torch.Tensor,
                       a_BLH: torch.Tensor, b_BLH: torch.Tensor, a_log_H: torch.Tensor,
                       dt_bias_H: torch.Tensor, state_BHDD: torch.Tensor) -> tuple:
    """The chunked gated delta rule of one GDN layer from its gate and beta logits.

    Same contract as the reference (numerics/gdn_fused.py:86-122): normalized q, k
    [B, L, G, 128] for G key heads, v [B, L, H, 128], gate logits a and beta logits b
    [B, L, H], all bf16; the per-head A_log and dt_bias [H]; the state [B, H, 128,
    128]. Returns (y [B, L, H, 128] bf16, final state) for g = exp(-exp(A_log)
    softplus(a + dt_bias)) and beta = sigmoid(b), made with the reference's bf16
    rounding points (gdn_sampler_gates). Violations raise AssertionError as there.

    The reference pads L to a multiple of 64 with rows of g = 1 and beta = 0; the
    tensor-core kernel stops at the sequence's last row instead, which leaves the
    state and the real rows' outputs the same. The state may be bf16 (the
    reference's dtype: the update runs on an fp32 copy, rounded back once at the
    end) or fp32 (this build's pools: advanced in place). a_log and dt_bias may
    be fp32 or bf16 (the gates round them to bf16 first either way).
    """
    batch, length, key_heads, width = q_BLGD.shape
    heads = v_BLHD.shape[2]
    assert width == HEAD_WIDTH == v_BLHD.shape[3] and heads % key_heads == 0
    assert k_BLGD.shape == q_BLGD.shape and a_BLH.shape == b_BLH.shape
    assert v_BLHD.shape[:2] == (batch, length) and a_BLH.shape == (batch, length, heads)
    assert all(value.dtype == torch.bfloat16
               for value in (q_BLGD, k_BLGD, v_BLHD, a_BLH, b_BLH))
    assert state_BHDD.dtype in (torch.bfloat16, torch.float32)
    assert state_BHDD.shape == (batch, heads, HEAD_WIDTH, HEAD_WIDTH)
    assert a_log_H.shape == dt_bias_H.shape == (heads,)
    a_log = a_log_H.float().contiguous()
    dt_bias = dt_bias_H.float().contiguous()
    g, beta = gdn_sampler_gates(a_BLH.contiguous(), b_BLH.contiguous(), a_log, dt_bias)
    in_place = state_BHDD.dtype == torch.float32 and state_BHDD.is_contiguous()
    state = state_BHDD if in_place else state_BHDD.float().contiguous()
    tokens = batch * length
    y = gdn_chunk_prefill(q_BLGD.reshape(tokens, key_heads, width).contiguous(),
                          k_BLGD.reshape(tokens, key_heads, width).contiguous(),
                          v_BLHD.reshape(tokens, heads, width).contiguous(),
                          g.view(tokens, heads), beta.view(tokens, heads), state, T=length)
    if not in_place:
        if state_BHDD.dtype == torch.float32:
            return y.view(batch, length, heads, width), state
        state = state.to(torch.bfloat16)
    return y.view(batch, length, heads, width), state
