"""One long sequence whose KV pages are split across GPUs (the config-4 path).

The reference runs one device; a 128k-token context there is one concatenated
cache read by one SDPA (mlx_decode.py:94-103). Here each rank holds a
contiguous range of the sequence's pages in its own pool, and per attention
layer and decode token:
  1.+2. the rank that owns the tail page appends the new token's K/V, and every
     rank computes its split-K partial over its own pages: normalised fp32 output
     and lse packed [Hq, D + 1] (sc_paged_decode_attention_packed, or, when the
     rank's pages are one split, sc_paged_decode_attention_fused with the append
     folded in);
  3. the ranks exchange the packed partials (Hq (D + 1) 4 bytes = 16.4 KB per
     rank at Hq 16, D 256) -- the one exchange of the path: either each rank
     stores its block straight into every peer's receive buffer over NVLink and
     raises an epoch flag there (PeerExchange: sc_exchange_put / sc_exchange_wait
     over CUDA IPC mappings), or an NCCL all-gather;
  4. every rank merges the gathered parts into the same bf16 output
     (sc_attention_combine_packed).
The GDN layers' state (32 heads x 128 x 128 fp32, 2 MiB) is small and is
updated identically on every rank.

`PageRanges` is the host-only partition (tested on CPU with gloo ranks);
`ShardedSequence` owns the device pools of one rank; `PeerExchange` owns the
NVLink receive buffers.
"""

from __future__ import annotations

import math

import torch

from . import _capi, paged
from ._torch import ptr, stream_of


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


def _cudart():
    from cuda.bindings import runtime as cudart

    return cudart


def epoch_base(tokens_done: int, attention_layers: int) -> int:
    """The epoch base of a token: attention layer l of token t raises the exchange flags
    to base + l + 1 with base = t x layers. The kernels add and compare modulo 2^32, so
    the base wraps like a u32, returned as the int32 two's-complement image an int32
    device word holds."""
    e = (tokens_done * attention_layers) & 0xFFFFFFFF
    return e - (1 << 32) if e >= 1 << 31 else e


def _check(result, what):
    err = result[0]
    if int(err) != 0:
        raise RuntimeError(f"{what} failed: {err}")
    return result[1] if len(result) > 1 else None


class PeerExchange:
    """NVLink receive buffers for the packed partials of `world` ranks.

    Each rank allocates [2 parities][world][rows][D + 1] fp32 plus [world] uint32
    epoch flags in one cudaMalloc block, shares it with CUDA IPC, and maps every
    peer's block, so its put kernel stores straight into the peers' memory. The
    process group only carries the IPC handles once (all_gather_object)."""

    def __init__(self, rows: int, width: int, rank: int, world: int, group=None,
                 device="cuda"):
        import torch.distributed as dist

        cudart = _cudart()
        self.rows, self.width, self.rank, self.world = rows, width, rank, world
        self.block = rows * width * 4                                # one rank's partial
        if self.block % 16:
            raise ValueError("PeerExchange: rows * (D + 1) * 4 must be a multiple of 16")
        self.flags_off = 2 * world * self.block
        nbytes = self.flags_off + ((world * 4 + 255) // 256) * 256
        dev = torch.device(device)
        self.device = dev
        with torch.cuda.device(dev):
            self.base = int(_check(cudart.cudaMalloc(nbytes), "cudaMalloc"))
            _check(cudart.cudaMemset(self.base, 0, nbytes), "cudaMemset")
            handle = _check(cudart.cudaIpcGetMemHandle(self.base), "cudaIpcGetMemHandle")
        raw = bytes(handle.reserved)
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, raw, group=group)
        else:
            handles = [raw]
        self.peer_bases, self._opened = [], []
        with torch.cuda.device(dev):
            for r, h in enumerate(handles):
                if r == rank:
                    self.peer_bases.append(self.base)
                    continue
                mh = cudart.cudaIpcMemHandle_t()
                mh.reserved = h
                p = int(_check(cudart.cudaIpcOpenMemHandle(
                    mh, cudart.cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle"))
                self.peer_bases.append(p)
                self._opened.append(p)
        # Per parity: where this rank's block goes on each peer, and each peer's flag for it.
        self.dst = [torch.tensor([b + (par * world + rank) * self.block for b in self.peer_bases],
                                 dtype=torch.int64, device=dev) for par in (0, 1)]
        self.flag_ptrs = torch.tensor([b + self.flags_off + 4 * rank for b in self.peer_bases],
                                      dtype=torch.int64, device=dev)
        # Arrival counter of the fused attention merge (the kernel leaves it zero).
        self.counter = torch.zeros(1, dtype=torch.int32, device=dev)

    def gathered(self, parity: int) -> int:
        """Device address of this rank's received [world][rows][D + 1] blocks."""
        return self.base + parity * self.world * self.block

    def put_and_wait(self, packed: torch.Tensor, epoch: torch.Tensor, epoch_add: int,
                     parity: int) -> None:
        stream = stream_of(packed)
        _capi.call("sc_exchange_put", ptr(packed), self.block, ptr(self.dst[parity]),
                   ptr(self.flag_ptrs), ptr(epoch), epoch_add, self.world, stream)
        _capi.call("sc_exchange_wait", self.base + self.flags_off, self.world, ptr(epoch),
                   epoch_add, stream)

    def attention_put(self, q: torch.Tensor, pool: torch.Tensor, table: torch.Tensor,
                      ctx: torch.Tensor, scale: float, *, max_pages: int,
                      pages_per_split: int, num_splits: int, workspace, packed: torch.Tensor,
                      epoch: torch.Tensor, epoch_add: int, parity: int) -> None:
        """Split-K attention of this rank's pages whose merge writes the packed rows
        into `packed`; its last CTA copies them into every rank's slot for this rank and
        raises the epoch flags (one kernel pair; sc_paged_decode_attention_exchange)."""
        B, hq, d = q.shape
        num_pages, hkv, page, _ = paged._pool_dims(pool)
        part_out, part_lse = workspace.views(B, num_splits)
        _capi.call("sc_paged_decode_attention_exchange", ptr(q), ptr(pool), num_pages,
                   ptr(table), ptr(ctx), B, hq, hkv, d, page, max_pages, pages_per_split,
                   num_splits, float(scale), ptr(part_out), ptr(part_lse), ptr(packed),
                   ptr(self.dst[parity]), ptr(self.flag_ptrs), ptr(self.counter), ptr(epoch),
                   epoch_add, self.world, stream_of(q))

    def merge(self, out: torch.Tensor, epoch: torch.Tensor, epoch_add: int, parity: int) -> None:
        """Wait (bounded) for every rank's epoch, then merge the received parts into
        out [rows, D] bf16 (sc_attention_combine_exchange)."""
        _capi.call("sc_attention_combine_exchange", self.gathered(parity),
                   self.base + self.flags_off, ptr(epoch), epoch_add, self.world, self.rows,
                   self.width - 1, ptr(out), None, stream_of(out))

    def close(self) -> None:
        cudart = _cudart()
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for p in self._opened:
                cudart.cudaIpcCloseMemHandle(p)
            self._opened = []
            if self.base:
                cudart.cudaFree(self.base)
                self.base = 0


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
        self.peer = None      # PeerExchange, when enable_peer_exchange() was called
        self.peer_fused = False
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self._h_epoch = torch.zeros(1, dtype=torch.int32).pin_memory()
        self.tokens_done = 0

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
        # Exchange epochs: attention layer l of this token raises flags to base + l + 1.
        self._h_epoch[0] = epoch_base(self.tokens_done, self.kv.shape[0])
        self.tokens_done += 1
        self.slot.copy_(self._h_slot, non_blocking=True)
        self.ctx.copy_(self._h_ctx, non_blocking=True)
        self.epoch.copy_(self._h_epoch, non_blocking=True)
        self._staged = torch.cuda.Event()
        self._staged.record()

    def enable_peer_exchange(self, group=None, fused: bool = False) -> None:
        """Exchange the packed partials by NVLink stores instead of NCCL (collective:
        every rank calls it). By default a put and a wait kernel carry the packed block.
        fused: the split merge's last CTA copies the block into the peers and the final
        merge waits for them (two launches fewer per layer)."""
        if self.kv.shape[0] % 2:
            raise ValueError("peer exchange alternates receive buffers per attention layer: "
                             "it needs an even number of attention layers")
        self.peer = PeerExchange(self.q_heads, self.head_dim + 1, self.rank, self.world,
                                 group=group, device=self.kv.device)
        self.peer_fused = fused

    def close(self) -> None:
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def groups(self) -> int:
        hkv = self.kv.shape[2]
        return hkv * ((self.q_heads // hkv + 7) // 8)

    def attention(self, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                  scale: float, all_gather=None) -> torch.Tensor:
        """One attention layer for the staged token: q [1, Hq, D], k/v [1, Hkv, D] bf16."""
        pool = self.kv[layer]
        # The grid covers the whole local capacity (fixed, so the step can be
        # captured); CTAs past the context return at once. One sequence makes
        # equal CTAs, so the split is sized for one wave on every SM (the batch
        # rule's two waves only add CTA overhead and partials here), rounded up to
        # a power of two and at least 32 pages: per layer 59.0 -> 56.7 us at one
        # rank's 8,207 pages (111 -> 128), 29.6 -> 26.1 us at 1,039 (14 -> 32;
        # 16 pages: 27.1).
        if self.workspace is None:
            sms = paged.sm_count(q.device)
            one_wave = max(1, -(-self.capacity * self.groups() // sms))
            self.pages_per_split = max(32, 1 << (one_wave - 1).bit_length())
            _, self.num_splits = paged.split_plan(self.capacity, self.pages_per_split)
            self.workspace = paged.AttentionWorkspace(1, self.q_heads, self.head_dim,
                                                      max(1, self.num_splits), device=q.device)
        if self.world == 1 and all_gather is None:
            # One rank holds every page: append the token and attend; the split merge
            # writes the final rows.
            paged.append_and_attend(q, k_new, v_new, self.slot, pool, self.table, self.ctx,
                                    scale, max_pages_in_batch=self.capacity,
                                    pages_per_split=self.pages_per_split,
                                    total_pages=self.capacity, workspace=self.workspace,
                                    out=self.out.view(1, self.q_heads, self.head_dim))
            return self.out
        if self.peer is not None and self.peer_fused and self.num_splits > 1:
            paged.kv_append(k_new, v_new, pool, self.slot)
            parity = (layer + 1) & 1   # the parity of this call's epoch (even layer count)
            self.peer.attention_put(q, pool, self.table, self.ctx, scale,
                                    max_pages=self.capacity, pages_per_split=self.pages_per_split,
                                    num_splits=self.num_splits, workspace=self.workspace,
                                    packed=self.packed, epoch=self.epoch, epoch_add=layer + 1,
                                    parity=parity)
            self.peer.merge(self.out, self.epoch, layer + 1, parity)
            return self.out
        # This rank's packed partial: the append folded into the attention launch when it
        # is one split, else the append, the split-K kernel and the merge.
        plan = dict(max_pages_in_batch=self.capacity, pages_per_split=self.pages_per_split,
                    total_pages=self.capacity, workspace=self.workspace)
        if self.num_splits == 1:
            paged.paged_decode_attention_fused(q, k_new, v_new, self.slot, pool, self.table,
                                               self.ctx, scale, packed=self.packed, **plan)
        else:
            paged.kv_append(k_new, v_new, pool, self.slot)
            paged.paged_decode_attention_packed(q, pool, self.table, self.ctx, scale,
                                                packed=self.packed, **plan)
        if self.peer is not None:
            parity = (layer + 1) & 1   # the parity of this call's epoch (even layer count)
            self.peer.put_and_wait(self.packed, self.epoch, layer + 1, parity)
            _capi.call("sc_attention_combine_packed", self.peer.gathered(parity), self.world,
                       self.q_heads, self.head_dim, ptr(self.out), None, stream_of(self.out))
            return self.out
        if all_gather is None:
            import torch.distributed as dist

            dist.all_gather_into_tensor(self.gathered, self.packed, group=self.group)
        else:
            all_gather(self.gathered, self.packed)
        paged.attention_combine_packed(self.gathered, out=self.out)
        return self.out
