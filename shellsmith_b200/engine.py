"""Hybrid GDN / full-attention cache engine: the decode cache step on one GPU.

The reference's decode step (studio_compute/mlx_decode.py:18-77
`decode_rows`) walks the layers; GDN layers concatenate every request's
recurrent cache, run the token kernel and split the caches back (42-60), and
attention layers run one request at a time (`_attention_rows`, 80-106). Here
the caches are persistent device pools and one launch covers every row:

  GDN layer        sc_gdn_decode over all rows, state rows = sequence slots
  attention layer  the new token's KV append and split-K attention over each
                   row's pages: one launch (sc_paged_decode_attention_fused) when
                   every sequence fits one split, else sc_kv_append,
                   sc_paged_decode_attention and its merge (8-bit pages:
                   sc_kv_append_q8 then sc_paged_decode_attention_q8)

A sequence's slot is its batch row, its block-table row and its GDN state row,
so no gather/scatter of caches happens per step; inactive rows are skipped by
the kernels (state slot -1, slot mapping -1, context length 0).
Projections, norms and the MLP are outside the cache path and are not run.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch

from . import gdn_layer, numerics, paged
from .block_manager import BlockManager


@dataclass
class HybridConfig:
    layers: int = 48
    attention_every: int = 4          # layer l is full attention when l % 4 == 3 (3:1)
    gdn_key_heads: int = 16
    gdn_value_heads: int = 32
    key_dim: int = 128
    value_dim: int = 128
    q_heads: int = 16
    kv_heads: int = 2
    head_dim: int = 256
    page_size: int = paged.PAGE_SIZE
    max_seqs: int = 256
    num_pages: int = 150_000
    max_context: int = 16_384 + 2_048 + 1_024
    state_dtype: torch.dtype = torch.float32
    pages_per_split: int | None = None   # None: adapt to the batch (paged.split_plan)
    snapshot_rows: int = 0               # extra GDN state rows for prefix snapshots
    gdn_taps: bool = False               # keep conv tap rings (layers run with their glue)
    gdn_glue_fused: bool = False         # one-launch cluster kernel instead of the 3-kernel step
    kv_precision: str = "bf16"           # "8bit": quantised pages (paged.new_pool_q8)
    sms: int | None = None               # SM count the split size is planned for (None: device's)

    def is_attention(self, layer: int) -> bool:
        return layer % self.attention_every == self.attention_every - 1

    @property
    def gdn_layers(self) -> list:
        return [l for l in range(self.layers) if not self.is_attention(l)]

    @property
    def attention_layers(self) -> list:
        return [l for l in range(self.layers) if self.is_attention(l)]

    @property
    def max_pages_per_seq(self) -> int:
        return math.ceil(self.max_context / self.page_size)

    def state_bytes(self) -> int:
        elem = torch.finfo(self.state_dtype).bits // 8
        return (len(self.gdn_layers) * self.max_seqs * self.gdn_value_heads * self.value_dim
                * self.key_dim * elem)

    def kv_token_bytes(self) -> float:
        """Bytes one cached token holds per attention layer (K and V of every kv head)."""
        if self.kv_precision == "8bit":   # codes + bf16 scale and bias per group of 64
            return self.kv_heads * (2 * self.head_dim + 8 * self.head_dim / 64)
        return self.kv_heads * self.head_dim * 2 * 2

    def kv_bytes(self) -> int:
        return int(len(self.attention_layers) * self.num_pages * self.page_size
                   * self.kv_token_bytes())


class HybridCacheEngine:
    """Device pools + block manager for one GPU's share of sequences."""

    def __init__(self, cfg: HybridConfig, device: torch.device | str = "cuda", seed: int = 0):
        self.cfg = cfg
        self.device = torch.device(device)
        dev = self.device
        n_gdn, n_attn = len(cfg.gdn_layers), len(cfg.attention_layers)
        self.gdn_index = {l: i for i, l in enumerate(cfg.gdn_layers)}
        self.attn_index = {l: i for i, l in enumerate(cfg.attention_layers)}
        self.state = torch.zeros((n_gdn, cfg.max_seqs + cfg.snapshot_rows, cfg.gdn_value_heads,
                                  cfg.value_dim, cfg.key_dim), dtype=cfg.state_dtype, device=dev)
        self._free_snapshot_rows = list(range(cfg.max_seqs + cfg.snapshot_rows - 1,
                                              cfg.max_seqs - 1, -1))
        # Conv tap rings [n_gdn, rows, 4, C] (gdn_layer): rows as the state's.
        channels = (2 * cfg.gdn_key_heads * cfg.key_dim + cfg.gdn_value_heads * cfg.value_dim)
        self.taps = (torch.zeros((n_gdn, self.state.shape[1], gdn_layer.RING, channels),
                                 dtype=torch.bfloat16, device=dev) if cfg.gdn_taps else None)
        self._glue_ws = None
        if cfg.kv_precision not in ("bf16", "8bit"):
            raise ValueError("Unsupported inference cache precision.")
        if cfg.kv_precision == "8bit":
            self.kv = torch.empty((n_attn, cfg.num_pages, cfg.kv_heads,
                                   paged.Q8_BYTES_PER_DIM * cfg.head_dim), dtype=torch.uint8,
                                  device=dev)
        else:
            self.kv = torch.empty((n_attn, cfg.num_pages, cfg.kv_heads, 2, cfg.page_size,
                                   cfg.head_dim), dtype=torch.bfloat16, device=dev)
        self.blocks = BlockManager(cfg.num_pages, cfg.page_size, cfg.max_seqs,
                                   cfg.max_pages_per_seq, seed=seed)
        # The step's tables: pinned host mirrors in one buffer, copied to the device's
        # buffer of the same layout in one transfer per step. int32 words: the block
        # table, then the slot mapping (int64), context lengths, state slots,
        # positions and the longest-first order, each segment 16-byte aligned.
        S, P = cfg.max_seqs, cfg.max_pages_per_seq
        seg = -(-S // 4) * 4
        n_table = -(-S * P // 4) * 4
        words = n_table + 6 * seg
        self._h_stage = torch.zeros(words, dtype=torch.int32, pin_memory=True)
        self._d_stage = torch.zeros(words, dtype=torch.int32, device=dev)

        def views(buf):
            o = n_table + 2 * seg
            return (buf[:S * P].view(S, P), buf[n_table:n_table + 2 * S].view(torch.int64),
                    buf[o:o + S], buf[o + seg:o + seg + S], buf[o + 2 * seg:o + 2 * seg + S],
                    buf[o + 3 * seg:o + 3 * seg + S])

        (self._h_table, self._h_slot_map, self._h_ctx, self._h_state_slot, self._h_position,
         self._h_order) = views(self._h_stage)
        (self.table, self.slot_map, self.ctx_len, self.state_slot, self.position,
         self.seq_order) = views(self._d_stage)
        self.blocks.table = self._h_table.numpy()
        # numpy views of the host mirrors, written in place every step
        self._n_slot_map, self._n_ctx, self._n_state_slot, self._n_position, self._n_order = (
            t.numpy() for t in (self._h_slot_map, self._h_ctx, self._h_state_slot,
                                self._h_position, self._h_order))
        self._h_slot_map.fill_(-1)
        self._h_state_slot.fill_(-1)
        self._h_order.copy_(torch.arange(S, dtype=torch.int32))
        self._d_stage.copy_(self._h_stage)
        self._staged = torch.cuda.Event()
        self._staged.record()
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        # Scratch for the smallest split size the plan can pick (16 pages).
        _, nsplit = paged.split_plan(cfg.max_pages_per_seq, cfg.pages_per_split or 16)
        self.workspace = paged.AttentionWorkspace(cfg.max_seqs, cfg.q_heads, cfg.head_dim, nsplit,
                                                  device=dev)
        self.max_pages_in_batch = 1
        self.total_pages = 0
        self.rows = cfg.max_seqs  # rows the step's kernels cover (set by begin_step)

    # ------------------------------------------------------------ lifecycle
    def admit(self, owner, prompt_len: int) -> int:
        """Reserve a slot and pages for a prompt; its GDN state starts at zero."""
        slot = self.blocks.admit(owner, prompt_len)
        self.state[:, slot].zero_()
        if self.taps is not None:
            self.taps[:, slot].zero_()
        return slot

    def _copy_rows(self, dst: int, src: int) -> None:
        """GDN state (and tap ring) row src -> dst in every GDN layer."""
        self.state[:, dst].copy_(self.state[:, src])
        if self.taps is not None:
            self.taps[:, dst].copy_(self.taps[:, src])

    def release(self, slot: int) -> None:
        self.blocks.release(slot)

    def extend(self, slot: int, tokens: int) -> None:
        """Hold `tokens` cached tokens in a sequence (pages for a prompt's remainder)."""
        self.blocks.extend(slot, tokens)

    # ------------------------------------------------------------ prefix snapshots
    def _copy_pages(self, src: list, dst: list) -> None:
        """Copy pages src[i] -> dst[i] in every attention layer's pool (one launch)."""
        if not src:
            return
        n_attn, num_pages = self.kv.shape[0], self.kv.shape[1]
        offs = np.arange(n_attn, dtype=np.int64)[:, None] * num_pages
        s = torch.from_numpy((offs + np.asarray(src)[None]).astype(np.int32).ravel())
        d = torch.from_numpy((offs + np.asarray(dst)[None]).astype(np.int32).ravel())
        flat = self.kv.view(n_attn * num_pages, *self.kv.shape[2:])
        paged.kv_copy_pages(flat, s.to(self.device), d.to(self.device))

    def _share_prefix(self, pages: list, tokens: int, copy_partial: bool) -> list:
        """Own the pages of a `tokens`-long prefix: full pages shared, the partial
        last page shared or copied into a fresh page."""
        P = self.cfg.page_size
        full = tokens // P
        owned = list(pages[:full])
        self.blocks.share(owned)
        if tokens % P:
            if copy_partial:
                fresh = self.blocks.take_pages(1)
                self._copy_pages([pages[full]], fresh)
                owned += fresh
            else:
                self.blocks.share([pages[full]])
                owned.append(pages[full])
        return owned

    def snapshot(self, slot: int) -> "PagedSnapshot":
        """An immutable copy of a live sequence's cache: full pages shared, the partial
        last page (which the sequence keeps writing) and the GDN state copied."""
        if not self._free_snapshot_rows:
            raise MemoryError("no free snapshot state row")
        tokens = int(self.blocks.lengths[slot])
        pages = self._share_prefix(self.blocks.pages[slot], tokens, copy_partial=True)
        row = self._free_snapshot_rows.pop()
        self._copy_rows(row, slot)
        return PagedSnapshot(self, pages, tokens, row)

    def fork(self, snap: "PagedSnapshot", owner=None) -> int:
        """A new sequence slot holding the snapshot's prefix: full pages shared, the
        partial last page copied (the fork appends to it), the GDN state copied."""
        pages = self._share_prefix(snap.pages, snap.tokens, copy_partial=True)
        slot = self.blocks.adopt(owner, pages, snap.tokens)
        self._copy_rows(slot, snap.row)
        return slot

    def copy_snapshot(self, snap: "PagedSnapshot") -> "PagedSnapshot":
        """Another owner of the same immutable prefix (every page shared)."""
        if not self._free_snapshot_rows:
            raise MemoryError("no free snapshot state row")
        pages = self._share_prefix(snap.pages, snap.tokens, copy_partial=False)
        row = self._free_snapshot_rows.pop()
        self._copy_rows(row, snap.row)
        return PagedSnapshot(self, pages, snap.tokens, row)

    def drop_snapshot(self, snap: "PagedSnapshot") -> None:
        if snap.row is None:
            return
        self.blocks.drop(snap.pages)
        self._free_snapshot_rows.append(snap.row)
        snap.row = None

    def cache_bytes(self, tokens: int) -> int:
        """Bytes a cache of `tokens` tokens holds: K/V of every attention layer plus the
        GDN state of every GDN layer (what a prefix snapshot is charged)."""
        c = self.cfg
        kv = tokens * c.kv_token_bytes() * len(c.attention_layers)
        elem = torch.finfo(c.state_dtype).bits // 8
        st = c.gdn_value_heads * c.value_dim * c.key_dim * elem * len(c.gdn_layers)
        if self.taps is not None:
            st += self.taps.shape[2] * self.taps.shape[3] * 2 * len(c.gdn_layers)
        return int(kv + st)

    def prefill(self, new: list, gdn_inputs, kv_inputs, out=None) -> int:
        """Run admitted prompts through every layer's cache work.

        new: [(slot, prompt_len)] of sequences admitted this step (their GDN
        state rows start at zero), or [(slot, start, stop)] to continue a prompt
        from position `start` (a prefix-cache fork: its state row holds the state
        after `start` tokens). gdn_inputs(layer, ntok) -> (q, k, v, decay, beta)
        packed [ntok, ...] in `new` order; kv_inputs(layer, ntok) -> (k, v)
        [ntok, Hkv, D]. GDN layers run the chunked prefill kernel over all
        prompts at once (one launch per layer, varlen); attention layers write
        the prompts' K/V into their pages. Returns the kernels launched.
        """
        if not new:
            return 0
        spans = [(e[0], 0, e[1]) if len(e) == 2 else tuple(e) for e in new]
        lengths = [stop - start for _, start, stop in spans]
        total = int(sum(lengths))
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32),
                          device=self.device)
        slots = torch.tensor([s for s, _, _ in spans], dtype=torch.int32, device=self.device)
        kv_slots = torch.from_numpy(np.concatenate(
            [self.blocks.prompt_slots(s, a, b) for s, a, b in spans])).to(self.device)
        launched = 0
        for layer in range(self.cfg.layers):
            if self.cfg.is_attention(layer):
                k, v = kv_inputs(layer, total)
                paged.kv_append(k, v, self.kv[self.attn_index[layer]], kv_slots)
            else:
                q, k, v, decay, beta = gdn_inputs(layer, total)
                numerics.gdn_chunk_prefill(q, k, v, decay, beta,
                                           self.state[self.gdn_index[layer]], slots, cu,
                                           out=None if out is None else out[:total])
            launched += 1
        return launched

    def write_prompt_kv(self, slot: int, layer: int, k: torch.Tensor, v: torch.Tensor,
                        start: int = 0) -> None:
        """Scatter prompt K/V [n, Hkv, D] of one attention layer at positions start.. ."""
        slots = self.blocks.prompt_slots(slot, start, start + k.shape[0])
        paged.kv_append(k, v, self.kv[self.attn_index[layer]],
                        torch.from_numpy(slots).to(self.device, non_blocking=True))

    def begin_step(self, rows=None) -> int:
        """Append one token to every active sequence (or to the listed slots only) and
        stage the step's tables. Rows outside the step are skipped by every kernel
        (state slot -1, slot mapping -1, context length 0).

        Returns the number of rows this step decodes.
        """
        self._staged.synchronize()  # the previous step's copies have read the staging
        blocks = self.blocks
        active = (np.flatnonzero(blocks.active) if rows is None
                  else np.asarray(sorted(int(r) for r in rows), np.int64))
        if rows is not None and not blocks.active[active].all():
            raise ValueError("begin_step: a listed slot holds no sequence")
        new_slots = blocks.append_token(active)  # raises before anything changes
        slot_map, ctx, state_slot = self._n_slot_map, self._n_ctx, self._n_state_slot
        slot_map.fill(-1)
        slot_map[active] = new_slots
        ctx.fill(0)
        ctx[active] = blocks.lengths[active]
        self._n_order[:] = np.argsort(-ctx, kind="stable")  # attention: longest first
        state_slot.fill(-1)
        state_slot[active] = active
        np.maximum(blocks.lengths - 1, 0, out=self._n_position, casting="unsafe")
        # Rows past the highest active slot hold no sequence: the step's kernels
        # cover rows [0, self.rows) only (the block manager packs slots low). The
        # longest-first order then starts with exactly those rows: inactive rows
        # tie at length 0 and keep their index order.
        self.rows = blocks.highest_active()
        self.max_pages_in_batch = max(1, int(blocks.pages_for(ctx.max())))
        self.total_pages = int(np.ceil(blocks.lengths[active] / self.cfg.page_size).sum())
        self._d_stage.copy_(self._h_stage, non_blocking=True)  # every table at once
        self._staged.record()
        return len(active)

    # ------------------------------------------------------------ decode
    def gdn_layer(self, layer: int, q, k, v, decay, beta, out, chained: bool = False) -> None:
        """The GDN state update of `layer` for every staged row. chained=True promises
        that the kernel queued just before it on the stream is another layer's update or
        an attention layer (it writes neither this layer's state rows nor the slot
        array), so the state may stream in while that kernel finishes."""
        n = self.rows
        if n == 0:
            return
        numerics.gdn_decode(q[:n], k[:n], v[:n], decay[:n], beta[:n],
                            self.state[self.gdn_index[layer]], self.state_slot[:n], out=out[:n],
                            chained=chained)

    def gdn_layer_front(self, layer: int, qkv, z, a, b, weights, out) -> None:
        """A GDN layer from its projections: conv taps, q/k norm, gates, state update
        and gated norm (gdn_layer.gdn_decode_split: three kernels, the state update
        overlapping the front; or gdn_decode_fused, one launch)."""
        i = self.gdn_index[layer]
        if self.cfg.gdn_glue_fused:
            gdn_layer.gdn_decode_fused(qkv, z, a, b, weights, self.taps[i], self.position,
                                       self.state[i], self.state_slot, out=out)
            return
        if self._glue_ws is None:
            self._glue_ws = gdn_layer.SplitWorkspace(self.cfg.max_seqs, weights, self.device)
        gdn_layer.gdn_decode_split(qkv, z, a, b, weights, self.taps[i], self.position,
                                   self.state[i], self.state_slot, out=out,
                                   workspace=self._glue_ws)

    def prefill_front(self, new: list, front_inputs, kv_inputs, out=None) -> int:
        """prefill() for layers run from their projections: front_inputs(layer, ntok)
        -> (qkv, z, a, b, weights) packed in `new` order; GDN layers run front,
        chunked recurrence, gated norm and tap store (gdn_layer.gdn_prefill)."""
        if not new:
            return 0
        spans = [(e[0], 0, e[1]) if len(e) == 2 else tuple(e) for e in new]
        lengths = [stop - start for _, start, stop in spans]
        total = int(sum(lengths))
        dev = self.device
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32), device=dev)
        slots = torch.tensor([s for s, _, _ in spans], dtype=torch.int32, device=dev)
        starts = torch.tensor([a for _, a, _ in spans], dtype=torch.int32, device=dev)
        kv_slots = torch.from_numpy(np.concatenate(
            [self.blocks.prompt_slots(s, a, b) for s, a, b in spans])).to(dev)
        launched = 0
        for layer in range(self.cfg.layers):
            if self.cfg.is_attention(layer):
                k, v = kv_inputs(layer, total)
                paged.kv_append(k, v, self.kv[self.attn_index[layer]], kv_slots)
                launched += 1
            else:
                qkv, z, a, b, weights = front_inputs(layer, total)
                i = self.gdn_index[layer]
                gdn_layer.gdn_prefill(qkv, z, a, b, weights, self.taps[i], self.state[i], cu,
                                      slots, starts, out=None if out is None else out[:total])
                launched += 4
        return launched

    def attention_layer(self, layer: int, q, k_new, v_new, out) -> None:
        """Append each row's new token and attend over its pages (paged.append_and_attend:
        one launch when the batch fits one split per sequence, else append, split-K and
        merge)."""
        n = self.rows
        if n == 0:
            return
        paged.append_and_attend(q[:n], k_new[:n], v_new[:n], self.slot_map[:n],
                                self.kv[self.attn_index[layer]], self.table[:n],
                                self.ctx_len[:n], self.scale,
                                max_pages_in_batch=self.max_pages_in_batch,
                                pages_per_split=self.cfg.pages_per_split,
                                total_pages=self.total_pages, workspace=self.workspace,
                                out=out[:n], seq_order=self.seq_order[:n], sms=self.cfg.sms)

    def decode_step(self, inputs: dict, outputs: dict) -> None:
        """Run every layer's cache work for the staged token of each active row.

        inputs[l] = (q, k, v, decay, beta) for GDN layers, (q, k, v) for
        attention layers; outputs[l] receives that layer's mixer output.
        """
        for layer in range(self.cfg.layers):
            if self.cfg.is_attention(layer):
                self.attention_layer(layer, *inputs[layer], outputs[layer])
            else:
                # Past the first layer the kernel before is this step's previous layer.
                self.gdn_layer(layer, *inputs[layer], outputs[layer], chained=layer > 0)

    # ------------------------------------------------------------ accounting
    def step_bytes(self, lengths: np.ndarray) -> dict:
        """Algorithmic HBM bytes of one decode step for active context lengths."""
        c = self.cfg
        n = len(lengths)
        gdn = len(c.gdn_layers) * n * (
            2 * c.gdn_value_heads * c.value_dim * c.key_dim * (torch.finfo(c.state_dtype).bits // 8)
            + (2 * c.gdn_key_heads * c.key_dim + 2 * c.gdn_value_heads * c.value_dim) * 2
            + 2 * c.gdn_value_heads * 4)
        row = c.kv_token_bytes()                        # K + V bytes of one token
        pages = np.ceil(lengths / c.page_size)
        attn_layer = (float(lengths.sum()) * row + n * row + n * c.q_heads * c.head_dim * 2 * 2
                      + float(pages.sum()) * 4)
        return {"gdn": float(gdn), "attention_per_layer": attn_layer,
                "attention": attn_layer * len(c.attention_layers),
                "total": float(gdn) + attn_layer * len(c.attention_layers)}


class PagedSnapshot:
    """A prefix cache entry: shared pages, a GDN state row and a token count."""

    def __init__(self, engine: HybridCacheEngine, pages: list, tokens: int, row: int):
        self.engine, self.pages, self.tokens, self.row = engine, pages, tokens, row

    @property
    def nbytes(self) -> int:
        return self.engine.cache_bytes(self.tokens)
