"""One long sequence whose KV pages are split across GPUs (the config-4 path).

The reference runs one device; a 128k-token context there is one concatenated
cache read by one SDPA (mlx_decode.py:94-103). Here each rank holds a
contiguous range of the sequence's pages in its own pool, and per attention
layer and decode token:
  1. the rank that owns the tail page appends the new token's K/V;
  2. every rank computes its split-K partial over its own pages: normalised
     fp32 output and lse, packed [Hq, D + 1] (sc_paged_decode_attention_packed);
  3. the ranks all-gather the packed partials (NCCL over NVLink; Hq (D + 1) 4
     bytes = 16.4 KB per rank at Hq 16, D 256) -- the one exchange of the path;
  4. every rank merges the gathered parts into the same bf16 output
     (sc_attention_combine_packed).
The GDN layers' state (32 heads x 128 x 128 fp32, 2 MiB) is small and is
updated identically on every rank.

`PageRanges` is the host-only partition (tested on CPU with gloo ranks);
`ShardedSequence` owns the device pools of one rank.
"""

from __future__ import annotations

import math

import torch

from . import paged


class PageRanges:
    """Contiguous split of `total_pages` pages over `world` ranks (first ranks take the rest)."""

    def __init__(self, total_pages: int, world: int):
        if total_pages < 0 or world < 1:
            raise ValueError("PageRanges: bad sizes")
        self.total_pages = total_pages
        self.world = world
        base, extra = divmod(total_pages, world)
        self.starts = [r * base + min(r, extra) for r in range(world + 1)]

    def range_of(self, rank: int) -> tuple:
        return self.starts[rank], self.starts[rank + 1]

    def owner(self, page: int) -> int:
        for r in range(self.world):
            if self.starts[r] <= page < self.starts[r + 1]:
                return r
        return self.world - 1  # pages past the split belong to the tail rank


class ShardedSequence:
    """The pages of one sequence held by this rank, for every attention layer."""

    def __init__(self, tokens: int, rank: int, world: int, *, attention_layers: int,
                 kv_heads: int, head_dim: int, q_heads: int, headroom_pages: int = 64,
                 device="cuda", group=None):
        self.rank, self.world, self.group = rank, world, group
        self.P = paged.PAGE_SIZE
        self.q_heads, self.head_dim = q_heads, head_dim
        total_pages = math.ceil(tokens / self.P)
        self.ranges = PageRanges(total_pages, world)
        first, last = self.ranges.range_of(rank)
        self.first_page = first
        self.local_pages = last - first
        self.is_tail = rank == world - 1
        capacity = self.local_pages + (headroom_pages if self.is_tail else 0)
        self.capacity = max(1, capacity)
        # Tokens this rank holds: full pages, except the tail rank's last page.
        self.local_tokens = min(tokens - first * self.P, self.local_pages * self.P) \
            if self.local_pages else 0
        self.kv = torch.empty((attention_layers, self.capacity, kv_heads, 2, self.P, head_dim),
                              dtype=torch.bfloat16, device=device)
        self.table = torch.arange(self.capacity, dtype=torch.int32,
                                  device=device).view(1, -1).contiguous()
        self.ctx = torch.tensor([self.local_tokens], dtype=torch.int32, device=device)
        self.slot = torch.full((1,), -1, dtype=torch.int64, device=device)
        # Pinned staging of the per-token scalars: copied before each step, so a
        # captured CUDA graph of the layers replays with fresh values.
        self._h_ctx = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._h_slot = torch.full((1,), -1, dtype=torch.int64).pin_memory()
        self._staged = None
        self.packed = torch.empty((q_heads, head_dim + 1), dtype=torch.float32, device=device)
        self.gathered = torch.empty((world, q_heads, head_dim + 1), dtype=torch.float32,
                                    device=device)
        self.out = torch.empty((q_heads, head_dim), dtype=torch.bfloat16, device=device)
        self.workspace = None
        self.pages_per_split = None

    def begin_token(self) -> None:
        """Stage the next decode token: the tail rank appends it after its last token.

        Only copies into the fixed device buffers `slot` and `ctx`, so the layer
        work may be a replayed CUDA graph."""
        if self._staged is not None:
            self._staged.synchronize()  # the previous copy has read the staging
        if self.is_tail:
            if self.local_tokens >= self.capacity * self.P:
                raise MemoryError("tail rank ran out of page headroom")
            self._h_slot[0] = self.local_tokens  # local page id * P + offset (identity table)
            self.local_tokens += 1
        else:
            self._h_slot[0] = -1
        self._h_ctx[0] = self.local_tokens
        self.slot.copy_(self._h_slot, non_blocking=True)
        self.ctx.copy_(self._h_ctx, non_blocking=True)
        self._staged = torch.cuda.Event()
        self._staged.record()

    def groups(self) -> int:
        hkv = self.kv.shape[2]
        return hkv * ((self.q_heads // hkv + 7) // 8)

    def attention(self, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                  scale: float, all_gather=None) -> torch.Tensor:
        """One attention layer for the staged token: q [1, Hq, D], k/v [1, Hkv, D] bf16."""
        pool = self.kv[layer]
        paged.kv_append(k_new, v_new, pool, self.slot)
        # The grid covers the whole local capacity (fixed, so the step can be
        # captured); CTAs past the context return at once. One sequence makes
        # equal CTAs, so the split is sized for exactly one wave on every SM
        # (the batch rule's two waves only add CTA overhead and partials here).
        if self.workspace is None:
            sms = paged.sm_count(q.device)
            self.pages_per_split = max(1, -(-self.capacity * self.groups() // sms))
            _, nsplit = paged.split_plan(self.capacity, self.pages_per_split)
            self.workspace = paged.AttentionWorkspace(1, self.q_heads, self.head_dim,
                                                      max(1, nsplit), device=q.device)
        paged.paged_decode_attention_packed(q, pool, self.table, self.ctx, scale,
                                            packed=self.packed, max_pages_in_batch=self.capacity,
                                            pages_per_split=self.pages_per_split,
                                            total_pages=self.capacity, workspace=self.workspace)
        if all_gather is None:
            import torch.distributed as dist

            dist.all_gather_into_tensor(self.gathered, self.packed, group=self.group)
        else:
            all_gather(self.gathered, self.packed)
        paged.attention_combine_packed(self.gathered, out=self.out)
        return self.out
