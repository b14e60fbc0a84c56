"""The cache path's C ABI registered as PyTorch operators: torch.ops.shellcache.*.

Each operator calls the same libshellcache.so entry point as the Python shims
(numerics, paged) and has a fake (meta) kernel, so shapes and dtypes propagate
under FakeTensorMode and torch.compile tracing without running a kernel. State
and page pools are mutated in place, as the C ABI does; an operator never
returns an alias of its inputs, so the ones the reference names with a
(output, next_state) result return the output and advance `state`.

  shellcache::gdn_decode                 sc_gdn_decode / _bf16 (numerics.gdn_decode)
  shellcache::gated_delta_token          gdn_token.py:18-42 call site, state in place
  shellcache::gated_delta_chunked        ops.py:151 call site, fp32 state in place
  shellcache::gated_delta_chunks         gdn_fused.py:86-122 call site, fp32 state in place
  shellcache::kv_append                  sc_kv_append / _q8
  shellcache::paged_decode_attention     sc_paged_decode_attention / _q8
  shellcache::paged_decode_attention_fused  append + split-K + merge in one launch

Importing this module registers the operators (once per process).
"""

from __future__ import annotations

from typing import Optional

import torch

from . import numerics, paged

_LIB = "shellcache"


@torch.library.custom_op(f"{_LIB}::gdn_decode", mutates_args=("state",))
def gdn_decode(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
               beta: torch.Tensor, state: torch.Tensor,
               state_slot: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One-token GDN update of rows b (state row state_slot[b]); returns out [B, Hv, dv]."""
    return numerics.gdn_decode(q, k, v, g, beta, state, state_slot)


@gdn_decode.register_fake
def _(q, k, v, g, beta, state, state_slot=None):
    return q.new_empty((q.shape[0], v.shape[1], v.shape[2]), dtype=torch.bfloat16)


@torch.library.custom_op(f"{_LIB}::gated_delta_token", mutates_args=("state_BHVK",))
def gated_delta_token(q_BLJK: torch.Tensor, k_BLJK: torch.Tensor, v_BLHV: torch.Tensor,
                      g_BLH: torch.Tensor, beta_BLH: torch.Tensor,
                      state_BHVK: torch.Tensor) -> torch.Tensor:
    """The reference's token step; returns out [B, 1, Hv, dv] and advances the state."""
    out, _ = numerics.gated_delta_token(q_BLJK, k_BLJK, v_BLHV, g_BLH, beta_BLH, state_BHVK)
    return out


@gated_delta_token.register_fake
def _(q_BLJK, k_BLJK, v_BLHV, g_BLH, beta_BLH, state_BHVK):
    return v_BLHV.new_empty(v_BLHV.shape, dtype=torch.bfloat16)


def _require_fp32_state(state: torch.Tensor, name: str) -> None:
    if state.dtype != torch.float32 or not state.is_contiguous():
        raise ValueError(f"shellcache::{name} advances a contiguous fp32 state in place")


@torch.library.custom_op(f"{_LIB}::gated_delta_chunked", mutates_args=("state",))
def gated_delta_chunked(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, g: torch.Tensor,
                        beta: torch.Tensor, state: torch.Tensor) -> torch.Tensor:
    """The reference's chunked recurrence; returns y [B, T, Hv, dv], state in place."""
    _require_fp32_state(state, "gated_delta_chunked")
    y, _ = numerics.gated_delta_chunked(q, k, v, g, beta, state)
    return y


@gated_delta_chunked.register_fake
def _(q, k, v, g, beta, state):
    return v.new_empty(v.shape)


@torch.library.custom_op(f"{_LIB}::gated_delta_chunks", mutates_args=("state",))
def gated_delta_chunks(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, a: torch.Tensor,
                       b: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor,
                       state: torch.Tensor) -> torch.Tensor:
    """The reference's chunked prefill from gate logits; returns y, state in place."""
    _require_fp32_state(state, "gated_delta_chunks")
    y, _ = numerics.gated_delta_chunks(q, k, v, a, b, a_log, dt_bias, state)
    return y


@gated_delta_chunks.register_fake
def _(q, k, v, a, b, a_log, dt_bias, state):
    return v.new_empty(v.shape, dtype=torch.bfloat16)


@torch.library.custom_op(f"{_LIB}::kv_append", mutates_args=("kv_pool",))
def kv_append(k: torch.Tensor, v: torch.Tensor, kv_pool: torch.Tensor,
              slot_mapping: torch.Tensor) -> None:
    """Write k/v [ntok, Hkv, D] into the pool at slot_mapping (int64, < 0 skips)."""
    paged.kv_append(k, v, kv_pool, slot_mapping)


@kv_append.register_fake
def _(k, v, kv_pool, slot_mapping):
    return None


@torch.library.custom_op(f"{_LIB}::paged_decode_attention", mutates_args=())
def paged_decode_attention(q: torch.Tensor, kv_pool: torch.Tensor, block_table: torch.Tensor,
                           ctx_len: torch.Tensor, scale: float,
                           pages_per_split: Optional[int] = None,
                           max_pages_in_batch: Optional[int] = None,
                           total_pages: Optional[int] = None) -> torch.Tensor:
    """Split-K decode attention of q [B, Hq, D] over each row's pages; returns out."""
    return paged.paged_decode_attention(q, kv_pool, block_table, ctx_len, scale,
                                        pages_per_split=pages_per_split,
                                        max_pages_in_batch=max_pages_in_batch,
                                        total_pages=total_pages)


@paged_decode_attention.register_fake
def _(q, kv_pool, block_table, ctx_len, scale, pages_per_split=None, max_pages_in_batch=None,
      total_pages=None):
    return torch.empty_like(q)


@torch.library.custom_op(f"{_LIB}::paged_decode_attention_fused", mutates_args=("kv_pool",))
def paged_decode_attention_fused(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                                 slot_mapping: torch.Tensor, kv_pool: torch.Tensor,
                                 block_table: torch.Tensor, ctx_len: torch.Tensor,
                                 scale: float, pages_per_split: Optional[int] = None,
                                 max_pages_in_batch: Optional[int] = None,
                                 total_pages: Optional[int] = None) -> torch.Tensor:
    """The new tokens' KV append and split-K attention in one launch; returns out."""
    return paged.paged_decode_attention_fused(q, k_new, v_new, slot_mapping, kv_pool,
                                              block_table, ctx_len, scale,
                                              pages_per_split=pages_per_split,
                                              max_pages_in_batch=max_pages_in_batch,
                                              total_pages=total_pages)


@paged_decode_attention_fused.register_fake
def _(q, k_new, v_new, slot_mapping, kv_pool, block_table, ctx_len, scale,
      pages_per_split=None, max_pages_in_batch=None, total_pages=None):
    return torch.empty_like(q)


OPERATORS = ("gdn_decode", "gated_delta_token", "gated_delta_chunked", "gated_delta_chunks",
             "kv_append", "paged_decode_attention", "paged_decode_attention_fused")
