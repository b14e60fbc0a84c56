"""The GDN layer between its projections and its output projection, on the GPU.

Mirrors studio_compute/numerics/bf16.py:44-139 (`gdn_inner`): causal-conv
taps + SiLU, q/k normalisation, gates, the gated-delta recurrence and the
gated RMS norm. Two forms:

  gdn_decode_fused     the engine form: one launch per layer and decode step,
                       state rows and tap rings in persistent slot pools,
                       rows addressed by state slot and absolute position
  gdn_prefill          the prefill form: front kernel -> chunked tcgen05
                       recurrence -> gated norm, then the tap rings
  gdn_inner            the reference's call-site signature (taps [B, K-1, C],
                       state [B, Hv, dv, dk], decode_one) over the kernels above

A tap ring is taps[slot][4][C]: the token at absolute position t reads rows
(t-3)&3, (t-2)&3, (t-1)&3 and writes row t&3, so the reference's
taps[B, 3, C] are the ring rows of positions t-3..t-1 in order.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _capi, numerics
from ._torch import ptr, require_cuda, stream_of

HEAD = 128
CONV_K = 4
RING = 4


@dataclass
class GDNWeights:
    """Frozen per-layer parameters the glue reads (reference attribute in brackets)."""

    conv_w: torch.Tensor      # [C, 4] bf16            (conv1d.weight [C, 4, 1])
    a_log: torch.Tensor       # [Hv] fp32              (A_log)
    dt_bias: torch.Tensor     # [Hv] fp32              (dt_bias)
    norm_w: torch.Tensor      # [128] bf16             (norm.weight)
    eps: float                #                        (norm.eps)
    key_heads: int            #                        (num_k_heads)
    value_heads: int          #                        (num_v_heads)

    @property
    def channels(self) -> int:
        return (2 * self.key_heads + self.value_heads) * HEAD

    def check(self) -> None:
        C, Hv = self.channels, self.value_heads
        require_cuda("conv_w", self.conv_w, torch.bfloat16, 2, align=8)
        if tuple(self.conv_w.shape) != (C, CONV_K):
            raise ValueError(f"conv_w must be [{C}, {CONV_K}]")
        for name, t in (("a_log", self.a_log), ("dt_bias", self.dt_bias)):
            require_cuda(name, t, torch.float32, 1, align=4)
            if t.shape[0] != Hv:
                raise ValueError(f"{name} must be [{Hv}]")
        require_cuda("norm_w", self.norm_w, torch.bfloat16, 1, align=8)
        if self.norm_w.shape[0] != HEAD:
            raise ValueError(f"norm_w must be [{HEAD}]")
        if Hv % self.key_heads:
            raise ValueError("value heads must be a multiple of key heads")

    @classmethod
    def from_linear(cls, linear, device=None) -> "GDNWeights":
        """From an object with the reference GatedDeltaNet's attribute names."""
        w = linear.conv1d.weight
        C = w.shape[0]
        return cls(conv_w=w.reshape(C, -1).to(device=device, dtype=torch.bfloat16).contiguous(),
                   a_log=linear.A_log.to(device=device, dtype=torch.float32).contiguous(),
                   dt_bias=linear.dt_bias.to(device=device, dtype=torch.float32).contiguous(),
                   norm_w=linear.norm.weight.to(device=device, dtype=torch.bfloat16).contiguous(),
                   eps=float(linear.norm.eps), key_heads=linear.num_k_heads,
                   value_heads=linear.num_v_heads)


def new_taps(slots: int, weights: GDNWeights, device="cuda") -> torch.Tensor:
    """A zeroed tap-ring pool [slots, 4, C] bf16 (a new sequence's taps are zero)."""
    return torch.zeros((slots, RING, weights.channels), dtype=torch.bfloat16, device=device)


def ring_window(taps: torch.Tensor, slot: int, position: int) -> torch.Tensor:
    """The reference's taps[K-1, C] of a slot before the token at `position`."""
    rows = [(position - d) % RING for d in (3, 2, 1)]
    return taps[slot, rows]


def _check_decode(qkv, z, a, b, weights, taps, position, state, state_slot) -> tuple:
    """Validate one decode step's operands; returns (B, C, Hk, Hv, slots)."""
    weights.check()
    B, C = qkv.shape
    Hk, Hv = weights.key_heads, weights.value_heads
    require_cuda("qkv", qkv, torch.bfloat16, 2, align=2)
    require_cuda("z", z, torch.bfloat16, 2, align=2)
    for name, t in (("a", a), ("b", b)):
        require_cuda(name, t, torch.bfloat16, 2, align=2)
        if tuple(t.shape) != (B, Hv):
            raise ValueError(f"gdn decode: {name} must be [{B}, {Hv}]")
    if C != weights.channels or tuple(z.shape) != (B, Hv * HEAD):
        raise ValueError("gdn decode: qkv must be [B, C] and z [B, Hv*128]")
    require_cuda("taps", taps, torch.bfloat16, 3, align=2)
    require_cuda("state", state, torch.float32, 4)
    slots = state.shape[0]
    if tuple(taps.shape) != (slots, RING, C) or tuple(state.shape[1:]) != (Hv, HEAD, HEAD):
        raise ValueError(f"gdn decode: taps must be [{slots}, 4, {C}], "
                         f"state [{slots}, {Hv}, 128, 128]")
    require_cuda("position", position, torch.int32, 1, align=4)
    if position.shape[0] != B:
        raise ValueError("gdn decode: one position per row")
    if state_slot is not None:
        require_cuda("state_slot", state_slot, torch.int32, 1, align=4)
        if state_slot.shape[0] != B:
            raise ValueError("gdn decode: one state slot per row")
    elif slots < B:
        raise ValueError("gdn decode: fewer state slots than rows")
    return B, C, Hk, Hv, slots


def gdn_decode_fused(qkv: torch.Tensor, z: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                     weights: GDNWeights, taps: torch.Tensor, position: torch.Tensor,
                     state: torch.Tensor, state_slot: torch.Tensor | None = None,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """One decode token of one GDN layer for B rows: front, update, gated norm.

    qkv [B, C], z [B, Hv*128], a, b [B, Hv] bf16; taps [slots, 4, C] bf16 and
    state [slots, Hv, 128, 128] fp32 updated in place; position [B] int32
    (absolute position of each row's token); state_slot [B] int32 (-1 skips a
    row) or None (row b uses slot b). Returns out [B, Hv*128] bf16.
    """
    B, C, Hk, Hv, slots = _check_decode(qkv, z, a, b, weights, taps, position, state,
                                        state_slot)
    if out is None:
        out = torch.empty((B, Hv * HEAD), dtype=torch.bfloat16, device=qkv.device)
    require_cuda("out", out, torch.bfloat16, 2, align=2)
    _capi.call("sc_gdn_decode_fused", ptr(qkv), ptr(z), ptr(a), ptr(b), ptr(weights.conv_w),
               ptr(weights.a_log), ptr(weights.dt_bias), ptr(weights.norm_w), weights.eps,
               ptr(taps), ptr(position), ptr(state), ptr(state_slot), ptr(out), B, Hk, Hv, slots,
               stream_of(qkv))
    return out


class SplitWorkspace:
    """Device workspace of the three-kernel decode step for up to `rows` rows (reused
    per call, so a captured CUDA graph sees fixed addresses)."""

    def __init__(self, rows: int, weights: "GDNWeights", device="cuda"):
        self.rows = rows
        self.nbytes = int(_capi.lib().sc_gdn_decode_glue_workspace(rows, weights.key_heads,
                                                                    weights.value_heads))
        self.buffer = torch.empty(self.nbytes, dtype=torch.uint8, device=device)

    def views(self, B: int, Hk: int, Hv: int) -> tuple:
        """The intermediates of the last call over B rows, in the layout
        sc_gdn_decode_glue documents: q, k [B, Hk, 128], v and the recurrence output
        y [B, Hv, 128] bf16, g and beta [B, Hv] fp32 (for checking each stage)."""
        def up(n):
            return (n + 255) // 256 * 256

        qk, vy, gb = up(B * Hk * HEAD * 2), up(B * Hv * HEAD * 2), up(B * Hv * 4)
        buf = self.buffer

        def part(off, n, dtype, shape):
            size = n * torch.empty((), dtype=dtype).element_size()
            return buf[off:off + size].view(dtype).view(shape)

        return (part(0, B * Hk * HEAD, torch.bfloat16, (B, Hk, HEAD)),
                part(qk, B * Hk * HEAD, torch.bfloat16, (B, Hk, HEAD)),
                part(2 * qk, B * Hv * HEAD, torch.bfloat16, (B, Hv, HEAD)),
                part(2 * qk + vy, B * Hv * HEAD, torch.bfloat16, (B, Hv, HEAD)),
                part(2 * qk + 2 * vy, B * Hv, torch.float32, (B, Hv)),
                part(2 * qk + 2 * vy + gb, B * Hv, torch.float32, (B, Hv)))


def gdn_decode_split(qkv: torch.Tensor, z: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                     weights: GDNWeights, taps: torch.Tensor, position: torch.Tensor,
                     state: torch.Tensor, state_slot: torch.Tensor | None = None,
                     out: torch.Tensor | None = None,
                     workspace: SplitWorkspace | None = None) -> torch.Tensor:
    """gdn_decode_fused's result in three kernels (sc_gdn_decode_glue): the front over
    the rows (each a one-token sequence at its position; it also stores the new tap
    rows), the bulk-copy state update launched as its programmatic dependent (its
    state loads overlap the front) and the gated norm. Rows' slots must differ."""
    B, _, Hk, Hv, slots = _check_decode(qkv, z, a, b, weights, taps, position, state,
                                        state_slot)
    ws = workspace if workspace is not None and workspace.rows >= B else SplitWorkspace(
        B, weights, qkv.device)
    if out is None:
        out = torch.empty((B, Hv * HEAD), dtype=torch.bfloat16, device=qkv.device)
    require_cuda("out", out, torch.bfloat16, 2, align=8)
    _capi.call("sc_gdn_decode_glue", ptr(qkv), ptr(z), ptr(a), ptr(b), ptr(weights.conv_w),
               ptr(weights.a_log), ptr(weights.dt_bias), ptr(weights.norm_w), weights.eps,
               ptr(taps), ptr(position), ptr(state), ptr(state_slot), ptr(out), ptr(ws.buffer),
               ws.nbytes, B, Hk, Hv, slots, stream_of(qkv))
    return out


def gdn_prefill_front(qkv: torch.Tensor, a: torch.Tensor, b: torch.Tensor, weights: GDNWeights,
                      taps: torch.Tensor, cu_seqlens: torch.Tensor, seq_slot: torch.Tensor,
                      seq_start: torch.Tensor) -> tuple:
    """Conv + SiLU + q/k norm + gates of packed prompt tokens (no tap writes).

    Returns (q, k [tokens, Hk, 128], v [tokens, Hv, 128] bf16, g, beta [tokens, Hv] fp32).
    """
    weights.check()
    T, C = qkv.shape
    Hk, Hv = weights.key_heads, weights.value_heads
    require_cuda("qkv", qkv, torch.bfloat16, 2, align=2)
    for name, t in (("a", a), ("b", b)):
        require_cuda(name, t, torch.bfloat16, 2, align=2)
        if tuple(t.shape) != (T, Hv):
            raise ValueError(f"gdn_prefill_front: {name} must be [{T}, {Hv}]")
    if C != weights.channels:
        raise ValueError(f"gdn_prefill_front: qkv must have {weights.channels} channels")
    require_cuda("taps", taps, torch.bfloat16, 3, align=2)
    for name, t in (("cu_seqlens", cu_seqlens), ("seq_slot", seq_slot),
                    ("seq_start", seq_start)):
        require_cuda(name, t, torch.int32, 1, align=4)
    nseq = seq_slot.shape[0]
    if cu_seqlens.shape[0] != nseq + 1 or seq_start.shape[0] != nseq:
        raise ValueError("gdn_prefill_front: cu_seqlens [n+1], seq_slot and seq_start [n]")
    dev = qkv.device
    q = torch.empty((T, Hk, HEAD), dtype=torch.bfloat16, device=dev)
    k = torch.empty_like(q)
    v = torch.empty((T, Hv, HEAD), dtype=torch.bfloat16, device=dev)
    g = torch.empty((T, Hv), dtype=torch.float32, device=dev)
    beta = torch.empty_like(g)
    _capi.call("sc_gdn_prefill_front", ptr(qkv), ptr(a), ptr(b), ptr(weights.conv_w),
               ptr(weights.a_log), ptr(weights.dt_bias), ptr(taps), ptr(cu_seqlens),
               ptr(seq_slot), ptr(seq_start), ptr(q), ptr(k), ptr(v), ptr(g), ptr(beta), nseq, T,
               Hk, Hv, taps.shape[0], stream_of(qkv))
    return q, k, v, g, beta


def gdn_taps_store(qkv: torch.Tensor, taps: torch.Tensor, cu_seqlens: torch.Tensor,
                   seq_slot: torch.Tensor, seq_start: torch.Tensor) -> None:
    """Each prompt's last min(3, n) inputs into its slot's tap ring (cu_seqlens None:
    sequence s is token s, a decode batch)."""
    require_cuda("qkv", qkv, torch.bfloat16, 2, align=2)
    require_cuda("taps", taps, torch.bfloat16, 3, align=2)
    if taps.shape[2] != qkv.shape[1] or taps.shape[1] != RING:
        raise ValueError("gdn_taps_store: taps must be [slots, 4, C] with qkv's C")
    _capi.call("sc_gdn_taps_store", ptr(qkv), ptr(taps), ptr(cu_seqlens), ptr(seq_slot),
               ptr(seq_start), seq_slot.shape[0], qkv.shape[1], taps.shape[0], stream_of(qkv))


def gated_rmsnorm(y: torch.Tensor, z: torch.Tensor, weight: torch.Tensor, eps: float,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """rms_norm(y, weight, eps) * silu(z) over the last axis (bf16 in and out)."""
    width = weight.shape[0]
    for name, t in (("y", y), ("z", z)):
        if t.dtype != torch.bfloat16 or not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"gated_rmsnorm: {name} must be a contiguous CUDA bf16 tensor")
    if y.numel() != z.numel() or y.numel() % width:
        raise ValueError("gated_rmsnorm: y and z must hold whole rows of the weight's width")
    require_cuda("weight", weight, torch.bfloat16, 1, align=8)
    if out is None:
        out = torch.empty_like(y)
    if (out.dtype != torch.bfloat16 or not out.is_cuda or not out.is_contiguous()
            or out.numel() != y.numel()):
        raise ValueError("gated_rmsnorm: out must be a contiguous CUDA bf16 tensor like y")
    _capi.call("sc_gated_rmsnorm", ptr(y), ptr(z), ptr(weight), float(eps), ptr(out),
               y.numel() // width, width, stream_of(y))
    return out


def gdn_prefill(qkv: torch.Tensor, z: torch.Tensor, a: torch.Tensor, b: torch.Tensor,
                weights: GDNWeights, taps: torch.Tensor, state: torch.Tensor,
                cu_seqlens: torch.Tensor, seq_slot: torch.Tensor, seq_start: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Prefill of packed prompts through one GDN layer: front, chunked recurrence on
    the tensor cores (state rows seq_slot, in place), gated norm, tap rings.
    Returns out [tokens, Hv*128] bf16."""
    q, k, v, g, beta = gdn_prefill_front(qkv, a, b, weights, taps, cu_seqlens, seq_slot,
                                         seq_start)
    y = numerics.gdn_chunk_prefill(q, k, v, g, beta, state, seq_slot, cu_seqlens)
    gdn_taps_store(qkv, taps, cu_seqlens, seq_slot, seq_start)
    out = gated_rmsnorm(y, z, weights.norm_w, weights.eps, out=out)
    return out.view(qkv.shape[0], -1)


def gdn_inner(linear, qkv_BLD, z_BLD, a_BLH, beta_BLH, conv_BCD, state_BHVK, *,
              decode_one: bool = False, gate_activation: str = "silu", weights=None) -> tuple:
    """The reference call site (bf16.py:44-139): returns (mixed [B, L, Hv*128],
    taps [B, K-1, C], next state). The state is fp32 and advanced in place (the
    reference returns a new array); taps are returned as a new tensor.
    """
    if gate_activation != "silu":
        raise ValueError("Unsupported GDN output gate activation.")
    weights = weights or GDNWeights.from_linear(linear, device=qkv_BLD.device)
    B, L, C = qkv_BLD.shape
    Hv = weights.value_heads
    assert conv_BCD.shape == (B, CONV_K - 1, C) and state_BHVK.shape == (B, Hv, HEAD, HEAD)
    assert not decode_one or L == 1
    dev = qkv_BLD.device
    ring = torch.zeros((B, RING, C), dtype=torch.bfloat16, device=dev)
    ring[:, :CONV_K - 1] = conv_BCD          # positions 0..2 hold the carried taps
    slots = torch.arange(B, dtype=torch.int32, device=dev)
    start = torch.full((B,), CONV_K - 1, dtype=torch.int32, device=dev)
    if L == 1:
        out = gdn_decode_fused(qkv_BLD[:, 0].contiguous(), z_BLD[:, 0].contiguous(),
                               a_BLH[:, 0].contiguous(), beta_BLH[:, 0].contiguous(), weights,
                               ring, start, state_BHVK)
    else:
        cu = torch.arange(0, (B + 1) * L, L, dtype=torch.int32, device=dev)
        out = gdn_prefill(qkv_BLD.reshape(B * L, C).contiguous(),
                          z_BLD.reshape(B * L, -1).contiguous(),
                          a_BLH.reshape(B * L, Hv).contiguous(),
                          beta_BLH.reshape(B * L, Hv).contiguous(), weights, ring, state_BHVK,
                          cu, slots, start)
    end = CONV_K - 1 + L                      # the next token's position
    taps = torch.stack([ring[:, (end - d) % RING] for d in (3, 2, 1)], dim=1)
    return out.view(B, L, -1), taps, state_BHVK
