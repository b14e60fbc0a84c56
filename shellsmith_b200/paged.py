"""Paged KV pool and split-K decode attention (device side).

The reference keeps one concatenating KV buffer per request
(studio_compute/mlx_request_cache.py:48-100 `OwnedKV`) and runs one SDPA per
request (mlx_decode.py:80-106). Here every attention layer owns one page pool
kv_pool[num_pages, Hkv, 2, P, D] (bf16) shared by all sequences; the host
block manager hands out pages, and these functions move and read them:

  kv_append               scatter new tokens' K/V through a slot mapping
  kv_gather               read logical K/V back (inverse of kv_append)
  kv_copy_pages           page-level copy-on-write of forked prefixes
  paged_decode_attention  split-K attention of one query per sequence over
                          its ragged pages, then the (out, lse) combine
  attention_combine       merge per-part (out, lse), e.g. across GPUs

8-bit pools (cache_precision "8bit"): uint8 [num_pages, Hkv, 34 * D], one
quantised block per (page, kv head) (new_pool_q8); kv_append, kv_copy_pages
and paged_decode_attention take either kind of pool and pick the kernels by
its dtype; kv_gather_q8 reads codes and scales back.
"""

from __future__ import annotations

import math

import torch

from . import _capi
from ._torch import ptr, require_cuda, stream_of

PAGE_SIZE = 16


def new_pool(num_pages: int, kv_heads: int, head_dim: int, page_size: int = PAGE_SIZE,
             device: str | torch.device = "cuda") -> torch.Tensor:
    """Allocate one layer's pool [num_pages, Hkv, 2, P, D] bf16 (uninitialised)."""
    return torch.empty((num_pages, kv_heads, 2, page_size, head_dim), dtype=torch.bfloat16,
                       device=device)


Q8_BYTES_PER_DIM = 34     # per (page, kv head): 2 x 16 x D codes + 4 x 16 x D/64 bf16


def new_pool_q8(num_pages: int, kv_heads: int, head_dim: int,
                device: str | torch.device = "cuda") -> torch.Tensor:
    """One layer's 8-bit pool [num_pages, Hkv, 34 * D] uint8 (uninitialised)."""
    if head_dim not in (128, 256):
        raise ValueError("8-bit pages need D in {128, 256}")
    return torch.empty((num_pages, kv_heads, Q8_BYTES_PER_DIM * head_dim), dtype=torch.uint8,
                       device=device)


def _q8_dims(kv_pool: torch.Tensor):
    require_cuda("kv_pool", kv_pool, torch.uint8, 3, align=16)
    num_pages, hkv, block = kv_pool.shape
    dim = block // Q8_BYTES_PER_DIM
    if block != Q8_BYTES_PER_DIM * dim or dim not in (128, 256):
        raise ValueError("an 8-bit pool must be [num_pages, Hkv, 34 * D], D in {128, 256}")
    return num_pages, hkv, PAGE_SIZE, dim


def _pool_dims(kv_pool: torch.Tensor):
    if kv_pool.dtype == torch.uint8:
        return _q8_dims(kv_pool)
    require_cuda("kv_pool", kv_pool, torch.bfloat16, 5)
    num_pages, hkv, two, page, dim = kv_pool.shape
    if two != 2:
        raise ValueError("kv_pool must be [num_pages, Hkv, 2, P, D]")
    return num_pages, hkv, page, dim


def kv_append(k: torch.Tensor, v: torch.Tensor, kv_pool: torch.Tensor,
              slot_mapping: torch.Tensor) -> None:
    """Write k/v [ntok, Hkv, D] into the pool at slot_mapping [ntok] (int64, <0 skips)."""
    num_pages, hkv, page, dim = _pool_dims(kv_pool)
    require_cuda("k", k, torch.bfloat16, 3)
    require_cuda("v", v, torch.bfloat16, 3)
    require_cuda("slot_mapping", slot_mapping, torch.int64, 1, align=8)
    ntok = k.shape[0]
    if k.shape != (ntok, hkv, dim) or v.shape != k.shape or slot_mapping.shape[0] != ntok:
        raise ValueError("kv_append: k/v must be [ntok, Hkv, D] with one slot per token")
    name = "sc_kv_append_q8" if kv_pool.dtype == torch.uint8 else "sc_kv_append"
    _capi.call(name, ptr(k), ptr(v), ptr(kv_pool), ptr(slot_mapping), ntok, hkv, dim, page,
               num_pages, stream_of(kv_pool))
    _count(1 if ntok else 0)


def kv_gather_q8(kv_pool: torch.Tensor, slot_mapping: torch.Tensor) -> tuple:
    """An 8-bit pool's tokens at slot_mapping in plain order: codes [ntok, Hkv, 2, D]
    uint8 (K, V) and scale_bias [ntok, Hkv, 2, D/64, 2] bf16 (zeros for slots < 0)."""
    num_pages, hkv, page, dim = _q8_dims(kv_pool)
    require_cuda("slot_mapping", slot_mapping, torch.int64, 1, align=8)
    ntok = slot_mapping.shape[0]
    codes = torch.empty((ntok, hkv, 2, dim), dtype=torch.uint8, device=kv_pool.device)
    sb = torch.empty((ntok, hkv, 2, dim // 64, 2), dtype=torch.bfloat16, device=kv_pool.device)
    _capi.call("sc_kv_gather_q8", ptr(kv_pool), ptr(slot_mapping), ntok, hkv, dim, page,
               num_pages, ptr(codes), ptr(sb), stream_of(kv_pool))
    return codes, sb


def kv_gather(kv_pool: torch.Tensor, slot_mapping: torch.Tensor) -> tuple:
    """Logical k, v [ntok, Hkv, D] stored at slot_mapping (zeros for negative slots)."""
    if kv_pool.dtype == torch.uint8:
        raise TypeError("kv_gather reads bf16 pools; use kv_gather_q8 for 8-bit pools")
    num_pages, hkv, page, dim = _pool_dims(kv_pool)
    require_cuda("slot_mapping", slot_mapping, torch.int64, 1, align=8)
    ntok = slot_mapping.shape[0]
    k = torch.empty((ntok, hkv, dim), dtype=torch.bfloat16, device=kv_pool.device)
    v = torch.empty_like(k)
    _capi.call("sc_kv_gather", ptr(kv_pool), ptr(slot_mapping), ptr(k), ptr(v), ntok, hkv, dim,
               page, num_pages, stream_of(kv_pool))
    return k, v


def kv_copy_pages(kv_pool: torch.Tensor, src: torch.Tensor, dst: torch.Tensor) -> None:
    """Copy pages src[i] -> dst[i] (int32), every head, K and V."""
    num_pages, hkv, page, dim = _pool_dims(kv_pool)
    require_cuda("src", src, torch.int32, 1, align=4)
    require_cuda("dst", dst, torch.int32, 1, align=4)
    if src.shape != dst.shape:
        raise ValueError("kv_copy_pages: src and dst must match")
    name = "sc_kv_copy_pages_q8" if kv_pool.dtype == torch.uint8 else "sc_kv_copy_pages"
    _capi.call(name, ptr(kv_pool), ptr(src), ptr(dst), src.shape[0], hkv, dim, page, num_pages,
               stream_of(kv_pool))


_SM_COUNT: dict = {}

# Kernels launched so far by the attention entry points of this module (appends, split-K
# kernels and their merges; a merge runs only when some sequence spans more than one
# split). Benchmarks read the difference over a timed region to count their launches.
attention_launches = 0


def _count(n: int) -> None:
    global attention_launches
    attention_launches += n


def sm_count(device) -> int:
    index = torch.device(device).index or 0
    if index not in _SM_COUNT:
        _SM_COUNT[index] = torch.cuda.get_device_properties(index).multi_processor_count
    return _SM_COUNT[index]


def split_plan(max_pages_in_batch: int, pages_per_split: int | None = None,
               total_work: int | None = None, sms: int | None = None, waves: int = 2,
               cap: int = 256, rows: int | None = None,
               min_pages: int | None = None) -> tuple:
    """(pages_per_split, num_splits) for a batch whose longest sequence has that many pages.

    sms is the SM count of the device that runs the launch (`sm_count(device)`);
    it is required whenever the size adapts to the batch (total_work given).

    Without an explicit size, a split is the largest power of two of pages, at
    most `cap`, whose CTAs still fill `waves` waves (one CTA per SM). The CTA
    count is estimated as total_work / pps, plus half a split per row for the
    rounding of each sequence when `rows` (sequences x head groups) is given;
    total_work = sum over sequences of pages x kv heads x head groups. Large
    splits keep the per-CTA overhead, the partials and their combine small (with
    the sequences launched longest first the last wave stays short); enough
    waves keep the SMs evenly loaded and a single long sequence spread over all
    of them. bf16 pages use three waves and up to 1,024 pages (16 MiB of K/V per
    kv head at D = 256); 8-bit pages, which carry half the bytes per page and
    more work per byte, measured best at two waves of at most 256 pages.

    min_pages: a split then grows to at least this many pages while the CTAs still
    number half a wave. Last, with `rows` given, a split doubles while its CTAs still
    fill one wave and an average sequence still spans three splits: config 2's share of
    32 sequences (U[1k, 32k]) took 0.214-0.215 ms per step with 128-page splits against
    0.202-0.204 ms with 256 (at 16 sequences the two tie, 0.120-0.123 ms), while config
    3's shorter sequences (64 of U[512, 16k]: under two 256-page splits each) keep 128. Small batches of long sequences meet the wave target only with
    short splits, and there each CTA's start, partial write and merge cost more than
    the extra waves gain: for bf16 pages at D = 256, 8 or 16 sequences of U[1k, 32k]
    tokens took 0.071 / 0.119 ms with 128-page splits against 0.088 / 0.126 ms with the
    wave rule's 32 / 64.
    """
    if pages_per_split:
        pps = pages_per_split
    elif total_work:
        if not sms or sms < 1:
            raise ValueError("split_plan: an adaptive split needs the device's SM count (sms)")

        def ctas(p):
            return total_work / p + (rows / 2 if rows else 0)
        pps = 16
        while pps * 2 <= cap and ctas(pps * 2) >= waves * sms:
            pps *= 2
        while min_pages and pps < min_pages and pps * 2 <= cap and \
                total_work / (pps * 2) >= sms / 2:
            pps *= 2
        # Long sequences: while the CTAs still fill a wave and a sequence still spans
        # three splits on average, fewer and longer splits cut the per-CTA start, the
        # partials and the merge more than the extra waves gain.
        while rows and pps * 2 <= cap and ctas(pps * 2) >= sms and \
                total_work / rows / (pps * 2) >= 3:
            pps *= 2
    else:
        pps = 64
    return pps, max(1, math.ceil(max(1, max_pages_in_batch) / pps))


def decode_plan(batch: int, q_heads: int, kv_heads: int, max_pages_in_batch: int,
                pages_per_split: int | None, total_pages: int | None, sms: int,
                q8: bool = False) -> tuple:
    """(pages_per_split, num_splits) that paged_decode_attention and its fused form pick
    for a batch: bf16 pages three waves, splits up to 1,024 pages and at least 128
    while half a wave remains; 8-bit pages two waves up to 256 pages."""
    groups = kv_heads * ((q_heads // kv_heads + 7) // 8)
    return split_plan(max_pages_in_batch, pages_per_split,
                      None if total_pages is None else total_pages * groups, sms,
                      waves=2 if q8 else 3, cap=256 if q8 else 1024,
                      rows=None if q8 else batch * groups, min_pages=None if q8 else 128)


class AttentionWorkspace:
    """Reusable split-K scratch (partials and their lse) for one layer shape."""

    def __init__(self, batch: int, q_heads: int, head_dim: int, num_splits: int,
                 device: str | torch.device = "cuda"):
        self.num_splits = num_splits
        self.part_out = torch.empty((batch, q_heads, num_splits, head_dim), dtype=torch.float32,
                                    device=device)
        self.part_lse = torch.empty((batch, q_heads, num_splits), dtype=torch.float32,
                                    device=device)
        # Arrival counters of the one-launch layer (one per sequence, kv head and head
        # group: at most one per query head); every launch leaves them zero.
        self.counters = torch.zeros(batch * q_heads, dtype=torch.int32, device=device)

    def fits(self, batch: int, q_heads: int, head_dim: int, num_splits: int) -> bool:
        b, h, s, d = self.part_out.shape
        return b >= batch and h == q_heads and d == head_dim and s >= num_splits

    def views(self, batch: int, num_splits: int) -> tuple:
        """Contiguous [batch, Hq, num_splits, D] / [batch, Hq, num_splits] views of the scratch."""
        b, h, s, d = self.part_out.shape
        n = batch * h * num_splits
        return (self.part_out.view(-1)[:n * d].view(batch, h, num_splits, d),
                self.part_lse.view(-1)[:n].view(batch, h, num_splits))


def paged_decode_attention(q: torch.Tensor, kv_pool: torch.Tensor, block_table: torch.Tensor,
                           ctx_len: torch.Tensor, scale: float, *,
                           max_pages_in_batch: int | None = None,
                           pages_per_split: int | None = None,
                           total_pages: int | None = None,
                           workspace: AttentionWorkspace | None = None,
                           out: torch.Tensor | None = None,
                           lse_out: torch.Tensor | None = None,
                           seq_order: torch.Tensor | None = None,
                           sms: int | None = None) -> torch.Tensor:
    """Decode attention of q [B, Hq, D] over each sequence's ctx_len[b] cached tokens.

    sms overrides the SM count the split size is planned for (default: the count
    of q's device).

    seq_order [B] int32 (a permutation) launches the sequences' CTAs in that
    order; longest first shortens the last wave of a ragged batch.

    block_table [B, max_pages] int32 lists each sequence's pages in token
    order. max_pages_in_batch (host-known) sizes the grid; when omitted the
    block-table width is used, which never syncs the device. total_pages
    (host-known sum of the sequences' pages) lets the split size adapt.
    """
    num_pages, hkv, page, dim = _pool_dims(kv_pool)
    require_cuda("q", q, torch.bfloat16, 3)
    require_cuda("block_table", block_table, torch.int32, 2, align=4)
    require_cuda("ctx_len", ctx_len, torch.int32, 1, align=4)
    B, hq, d = q.shape
    if d != dim or hq % hkv or block_table.shape[0] != B or ctx_len.shape[0] != B:
        raise ValueError("paged_decode_attention: inconsistent shapes")
    max_pages = block_table.shape[1]
    q8 = kv_pool.dtype == torch.uint8
    pps, nsplit = decode_plan(B, hq, hkv, max_pages_in_batch or max_pages, pages_per_split,
                              total_pages, sms or sm_count(q.device), q8=q8)
    if out is None:
        out = torch.empty((B, hq, dim), dtype=torch.bfloat16, device=q.device)
    require_cuda("out", out, torch.bfloat16, 3)
    if lse_out is not None:
        require_cuda("lse_out", lse_out, torch.float32, 1, align=4)
    if seq_order is not None:
        require_cuda("seq_order", seq_order, torch.int32, 1, align=4)
        if seq_order.shape[0] != B:
            raise ValueError("paged_decode_attention: seq_order needs one entry per sequence")
    part_out = part_lse = None
    if nsplit > 1:
        if workspace is None or not workspace.fits(B, hq, dim, nsplit):
            workspace = AttentionWorkspace(B, hq, dim, nsplit, device=q.device)
        part_out, part_lse = workspace.views(B, nsplit)
    name = ("sc_paged_decode_attention_q8" if kv_pool.dtype == torch.uint8
            else "sc_paged_decode_attention")
    _capi.call(name, ptr(q), ptr(kv_pool), num_pages, ptr(block_table), ptr(ctx_len),
               ptr(seq_order), B, hq, hkv, dim, page, max_pages, pps, nsplit, float(scale),
               ptr(part_out), ptr(part_lse), ptr(out), ptr(lse_out), stream_of(q))
    _count(1 + (nsplit > 1) if B else 0)
    return out


def paged_decode_attention_fused(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                                 slot_mapping: torch.Tensor, kv_pool: torch.Tensor,
                                 block_table: torch.Tensor, ctx_len: torch.Tensor, scale: float,
                                 *, max_pages_in_batch: int | None = None,
                                 pages_per_split: int | None = None,
                                 total_pages: int | None = None,
                                 workspace: AttentionWorkspace | None = None,
                                 out: torch.Tensor | None = None,
                                 lse_out: torch.Tensor | None = None,
                                 packed: torch.Tensor | None = None,
                                 seq_order: torch.Tensor | None = None,
                                 sms: int | None = None,
                                 in_kernel_merge: bool = False) -> torch.Tensor:
    """kv_append of each row's new token folded into paged_decode_attention
    (sc_paged_decode_attention_fused): one launch, plus the merge kernel when a
    sequence spans several splits. in_kernel_merge: the last split of each sequence
    merges them instead (at most 16 splits), which measured slower on B200 (the
    arrival round trip keeps every split CTA resident longer than the separate merge
    costs), so it is off by default.

    k_new, v_new [B, Hkv, D] bf16 and slot_mapping [B] int64 (< 0: no append) are
    the step's new tokens; ctx_len counts them. With `packed` ([B * Hq, D + 1] fp32)
    the rows come out as the packed per-device partial instead of bf16 `out`.
    Other arguments as paged_decode_attention (bf16 pools only).
    """
    if kv_pool.dtype != torch.bfloat16:
        raise TypeError("paged_decode_attention_fused takes bf16 pools")
    num_pages, hkv, page, dim = _pool_dims(kv_pool)
    require_cuda("q", q, torch.bfloat16, 3)
    require_cuda("k_new", k_new, torch.bfloat16, 3)
    require_cuda("v_new", v_new, torch.bfloat16, 3)
    require_cuda("slot_mapping", slot_mapping, torch.int64, 1, align=8)
    require_cuda("block_table", block_table, torch.int32, 2, align=4)
    require_cuda("ctx_len", ctx_len, torch.int32, 1, align=4)
    B, hq, d = q.shape
    if (d != dim or hq % hkv or block_table.shape[0] != B or ctx_len.shape[0] != B
            or k_new.shape != (B, hkv, dim) or v_new.shape != k_new.shape
            or slot_mapping.shape[0] != B):
        raise ValueError("paged_decode_attention_fused: inconsistent shapes")
    max_pages = block_table.shape[1]
    pps, nsplit = decode_plan(B, hq, hkv, max_pages_in_batch or max_pages, pages_per_split,
                              total_pages, sms or sm_count(q.device))
    if packed is None:
        if out is None:
            out = torch.empty((B, hq, dim), dtype=torch.bfloat16, device=q.device)
        require_cuda("out", out, torch.bfloat16, 3)
    else:
        require_cuda("packed", packed, torch.float32, 2, align=4)
        if tuple(packed.shape) != (B * hq, dim + 1) or out is not None:
            raise ValueError("paged_decode_attention_fused: packed is [B * Hq, D + 1], "
                             "given instead of out")
    if lse_out is not None:
        require_cuda("lse_out", lse_out, torch.float32, 1, align=4)
    if seq_order is not None:
        require_cuda("seq_order", seq_order, torch.int32, 1, align=4)
        if seq_order.shape[0] != B:
            raise ValueError("paged_decode_attention_fused: seq_order needs one entry per "
                             "sequence")
    part_out = part_lse = counters = None
    if nsplit > 1:
        if workspace is None or not workspace.fits(B, hq, dim, nsplit):
            workspace = AttentionWorkspace(B, hq, dim, nsplit, device=q.device)
        part_out, part_lse = workspace.views(B, nsplit)
        counters = workspace.counters
    merge_in_kernel = bool(in_kernel_merge) and 1 < nsplit <= 16
    _capi.call("sc_paged_decode_attention_fused", ptr(q), ptr(k_new), ptr(v_new),
               ptr(slot_mapping), ptr(kv_pool), num_pages, ptr(block_table), ptr(ctx_len),
               ptr(seq_order), B, hq, hkv, dim, page, max_pages, pps, nsplit, float(scale),
               ptr(part_out), ptr(part_lse), ptr(counters), ptr(out), ptr(lse_out), ptr(packed),
               int(merge_in_kernel), stream_of(q))
    _count(1 + (nsplit > 1 and not merge_in_kernel) if B else 0)
    return packed if packed is not None else out


def append_and_attend(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                      slot_mapping: torch.Tensor, kv_pool: torch.Tensor,
                      block_table: torch.Tensor, ctx_len: torch.Tensor, scale: float, *,
                      max_pages_in_batch: int | None = None,
                      pages_per_split: int | None = None, total_pages: int | None = None,
                      workspace: AttentionWorkspace | None = None,
                      out: torch.Tensor | None = None, seq_order: torch.Tensor | None = None,
                      sms: int | None = None) -> torch.Tensor:
    """One decode step of an attention layer: append each row's new token, then attend.

    When every sequence fits one split (the plan has one), the append is folded into
    the attention launch (paged_decode_attention_fused: one kernel). Otherwise
    kv_append, the split-K kernel and the merge run as three launches: on B200 that
    sequence measured faster than the fused kernel with its splits merged either in
    the kernel or by the merge kernel (config 2 shares of 8-64 sequences: 1.5-6 %).
    8-bit pools always take the two kernels of their own.
    """
    if kv_pool.dtype == torch.bfloat16:
        num_pages, hkv, page, dim = _pool_dims(kv_pool)
        _, nsplit = decode_plan(q.shape[0], q.shape[1], hkv,
                                max_pages_in_batch or block_table.shape[1], pages_per_split,
                                total_pages, sms or sm_count(q.device))
        if nsplit == 1:
            return paged_decode_attention_fused(
                q, k_new, v_new, slot_mapping, kv_pool, block_table, ctx_len, scale,
                max_pages_in_batch=max_pages_in_batch, pages_per_split=pages_per_split,
                total_pages=total_pages, workspace=workspace, out=out, seq_order=seq_order,
                sms=sms)
    kv_append(k_new, v_new, kv_pool, slot_mapping)
    return paged_decode_attention(q, kv_pool, block_table, ctx_len, scale,
                                  max_pages_in_batch=max_pages_in_batch,
                                  pages_per_split=pages_per_split, total_pages=total_pages,
                                  workspace=workspace, out=out, seq_order=seq_order, sms=sms)


def attention_combine(part_out: torch.Tensor, part_lse: torch.Tensor,
                      out: torch.Tensor | None = None,
                      lse_out: torch.Tensor | None = None) -> tuple:
    """Merge part_out [rows, S, D] fp32 with part_lse [rows, S] -> (out bf16, lse fp32)."""
    require_cuda("part_out", part_out, torch.float32, 3)
    require_cuda("part_lse", part_lse, torch.float32, 2, align=4)
    rows, nparts, dim = part_out.shape
    if part_lse.shape != (rows, nparts):
        raise ValueError("attention_combine: part_lse must be [rows, S]")
    if out is None:
        out = torch.empty((rows, dim), dtype=torch.bfloat16, device=part_out.device)
    if lse_out is None:
        lse_out = torch.empty((rows,), dtype=torch.float32, device=part_out.device)
    _capi.call("sc_attention_combine", ptr(part_out), ptr(part_lse), rows, nparts, dim, ptr(out),
               ptr(lse_out), stream_of(part_out))
    return out, lse_out


def paged_decode_attention_packed(q: torch.Tensor, kv_pool: torch.Tensor,
                                  block_table: torch.Tensor, ctx_len: torch.Tensor, scale: float,
                                  *, packed: torch.Tensor | None = None,
                                  max_pages_in_batch: int | None = None,
                                  pages_per_split: int | None = None,
                                  total_pages: int | None = None,
                                  workspace: AttentionWorkspace | None = None) -> torch.Tensor:
    """Like paged_decode_attention, but returns fp32 packed [B * Hq, D + 1]: each row's
    normalised output and, at index D, its natural-log lse (a device's partial)."""
    if kv_pool.dtype == torch.uint8:
        raise TypeError("paged_decode_attention_packed takes bf16 pools")
    num_pages, hkv, page, dim = _pool_dims(kv_pool)
    require_cuda("q", q, torch.bfloat16, 3)
    require_cuda("block_table", block_table, torch.int32, 2, align=4)
    require_cuda("ctx_len", ctx_len, torch.int32, 1, align=4)
    B, hq, d = q.shape
    if d != dim or hq % hkv or block_table.shape[0] != B or ctx_len.shape[0] != B:
        raise ValueError("paged_decode_attention_packed: inconsistent shapes")
    max_pages = block_table.shape[1]
    groups = hkv * ((hq // hkv + 7) // 8)
    pps, nsplit = split_plan(max_pages_in_batch or max_pages, pages_per_split,
                             None if total_pages is None else total_pages * groups,
                             sm_count(q.device))
    if packed is None:
        packed = torch.empty((B * hq, dim + 1), dtype=torch.float32, device=q.device)
    require_cuda("packed", packed, torch.float32, 2, align=4)
    part_out = part_lse = None
    if nsplit > 1:
        if workspace is None or not workspace.fits(B, hq, dim, nsplit):
            workspace = AttentionWorkspace(B, hq, dim, nsplit, device=q.device)
        part_out, part_lse = workspace.views(B, nsplit)
    _capi.call("sc_paged_decode_attention_packed", ptr(q), ptr(kv_pool), num_pages,
               ptr(block_table), ptr(ctx_len), B, hq, hkv, dim, page, max_pages, pps, nsplit,
               float(scale), ptr(part_out), ptr(part_lse), ptr(packed), stream_of(q))
    _count(1 + (nsplit > 1) if B else 0)
    return packed


def attention_combine_packed(gathered: torch.Tensor, out: torch.Tensor | None = None,
                             lse_out: torch.Tensor | None = None) -> tuple:
    """Merge gathered packed parts [nparts, rows, D + 1] -> (out [rows, D] bf16, lse [rows])."""
    require_cuda("gathered", gathered, torch.float32, 3, align=4)
    nparts, rows, width = gathered.shape
    dim = width - 1
    if out is None:
        out = torch.empty((rows, dim), dtype=torch.bfloat16, device=gathered.device)
    if lse_out is None:
        lse_out = torch.empty((rows,), dtype=torch.float32, device=gathered.device)
    _capi.call("sc_attention_combine_packed", ptr(gathered), nparts, rows, dim, ptr(out),
               ptr(lse_out), stream_of(gathered))
    return out, lse_out
