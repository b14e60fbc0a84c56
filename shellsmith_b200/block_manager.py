"""Host page allocator, block tables and GDN state slots for the paged cache.

The reference has no paging: each request owns a concatenating KV buffer
(studio_compute/mlx_request_cache.py:48-100) and a recurrent-cache copy, and
admission is a byte reservation (inference.py:21-56, model.py:271-288). This
block manager is the paged counterpart. Its logical effects follow the
reference -- a request is admitted or deferred, advanced one token per
decode step, and released with all of its resources -- while the physical
placement (which page, which slot) is this build's own, deterministic:

  * pages come from a LIFO free list seeded with a permutation of the pool
    (seeded RNG), and a release pushes the pages back in reverse order;
  * a page has a reference count: prefix snapshots and forked sequences share
    full pages, and a page returns to the free list when its last owner
    drops it;
  * a new sequence takes the lowest free state slot of [0, max_seqs), so the
    active slots stay packed at the bottom; a sequence's slot is also its batch
    row, its block-table row and its GDN state row;
  * a sequence of n tokens holds ceil(n / P) pages; the token at position t
    lives at slot page[t // P] * P + t % P.

Everything here is host NumPy; the device copies of the block table, the
context lengths and the slot mapping are refreshed by the engine.
"""

from __future__ import annotations

import heapq

import numpy as np


class OutOfPages(MemoryError):
    """The pool cannot hold the requested tokens."""


class BlockManager:
    def __init__(self, num_pages: int, page_size: int, max_seqs: int, max_pages_per_seq: int,
                 seed: int | None = 0):
        if num_pages < 1 or page_size < 1 or max_seqs < 1 or max_pages_per_seq < 1:
            raise ValueError("BlockManager sizes must be positive")
        self.num_pages = num_pages
        self.page_size = page_size
        self.max_seqs = max_seqs
        self.max_pages_per_seq = max_pages_per_seq
        order = (np.random.default_rng(seed).permutation(num_pages) if seed is not None
                 else np.arange(num_pages))
        # pop() takes from the end: reverse so the first page handed out is order[0].
        self._free_pages = [int(p) for p in order[::-1]]
        # Free slots as a min-heap: a new sequence takes the lowest free slot, so the
        # active rows stay packed at the bottom and a step can launch over rows
        # [0, highest active slot] only (highest_active()).
        self._free_slots = list(range(max_seqs))
        self.table = np.zeros((max_seqs, max_pages_per_seq), np.int32)
        self.refcount = np.zeros(num_pages, np.int32)
        self.lengths = np.zeros(max_seqs, np.int64)
        self.active = np.zeros(max_seqs, bool)
        self.pages: dict[int, list] = {}
        self.owner: dict[int, object] = {}
        self.dirty_rows: set = set()

    # ------------------------------------------------------------ queries
    @property
    def free_pages(self) -> int:
        return len(self._free_pages)

    @property
    def free_slots(self) -> int:
        return len(self._free_slots)

    def highest_active(self) -> int:
        """1 + the highest active slot (0 when none): a step's kernels need cover only
        rows [0, highest_active())."""
        act = np.flatnonzero(self.active)
        return int(act[-1]) + 1 if act.size else 0

    def pages_for(self, tokens: int) -> int:
        return -(-int(tokens) // self.page_size)

    def can_admit(self, tokens: int) -> bool:
        need = self.pages_for(tokens)
        return (bool(self._free_slots) and need <= len(self._free_pages)
                and need <= self.max_pages_per_seq)

    def slot_of_position(self, slot: int, position: int) -> int:
        page = self.pages[slot][position // self.page_size]
        return page * self.page_size + position % self.page_size

    # ------------------------------------------------------------ lifecycle
    def admit(self, owner, tokens: int) -> int:
        """Reserve a state slot and pages for `tokens` cached tokens; returns the slot."""
        if not self._free_slots:
            raise OutOfPages("no free sequence slot")
        need = self.pages_for(tokens)
        if need > self.max_pages_per_seq:
            raise OutOfPages(f"{tokens} tokens exceed {self.max_pages_per_seq} pages per sequence")
        if need > len(self._free_pages):
            raise OutOfPages(f"{need} pages needed, {len(self._free_pages)} free")
        slot = heapq.heappop(self._free_slots)
        pages = self.take_pages(need)
        self.pages[slot] = pages
        self.owner[slot] = owner
        self.table[slot, :need] = pages
        self.table[slot, need:] = 0
        self.lengths[slot] = tokens
        self.active[slot] = True
        self.dirty_rows.add(slot)
        return slot

    def prompt_slots(self, slot: int, start: int, stop: int) -> np.ndarray:
        """Slot mapping (int64) of positions [start, stop) of a sequence."""
        pages = np.asarray(self.pages[slot], np.int64)
        pos = np.arange(start, stop, dtype=np.int64)
        return pages[pos // self.page_size] * self.page_size + pos % self.page_size

    def append_token(self, slots: np.ndarray) -> np.ndarray:
        """Grow each listed sequence by one token; returns the new tokens' KV slots.

        A sequence whose length is a multiple of P takes one new page (LIFO).
        Raises OutOfPages before changing anything if the pool cannot cover
        every sequence that needs a page.
        """
        slots = np.asarray(slots, np.int64)
        lengths = self.lengths[slots]
        needs_page = lengths % self.page_size == 0
        if int(needs_page.sum()) > len(self._free_pages):
            raise OutOfPages("pool exhausted while appending decode tokens")
        if np.any(lengths // self.page_size + needs_page > self.max_pages_per_seq):
            raise OutOfPages("a sequence outgrew max_pages_per_seq")
        # Only a sequence at a page boundary changes its page list (about one row in
        # P per step); every other row's slot is read from the table, which mirrors
        # the page lists row for row.
        grow = np.flatnonzero(needs_page)
        if grow.size:
            # One pop for every row that needs a page, in row order (the same LIFO
            # pages a row-by-row take would give).
            new_pages = self.take_pages(int(grow.size))
            rows = slots[grow]
            self.table[rows, lengths[grow] // self.page_size] = new_pages
            for slot, page in zip(rows.tolist(), new_pages):
                self.pages[slot].append(page)
            self.dirty_rows.update(rows.tolist())
        out = (self.table[slots, lengths // self.page_size].astype(np.int64) * self.page_size
               + lengths % self.page_size)
        self.lengths[slots] = lengths + 1
        return out

    # ------------------------------------------------------------ shared pages
    def take_pages(self, n: int) -> list:
        """Pop n free pages (LIFO), each with reference count 1."""
        if n > len(self._free_pages):
            raise OutOfPages(f"{n} pages needed, {len(self._free_pages)} free")
        pages = [self._free_pages.pop() for _ in range(n)]
        self.refcount[pages] = 1
        return pages

    def share(self, pages) -> None:
        """One more owner (a prefix snapshot or a forked sequence) for each page."""
        for p in pages:
            self.refcount[p] += 1

    def drop(self, pages) -> None:
        """One owner fewer; pages nobody owns go back to the free list (reverse order)."""
        for p in reversed(list(pages)):
            self.refcount[p] -= 1
            if self.refcount[p] == 0:
                self._free_pages.append(int(p))
            elif self.refcount[p] < 0:
                raise RuntimeError(f"page {p} released more often than it was owned")

    def adopt(self, owner, pages: list, tokens: int) -> int:
        """Open a sequence slot over pages the caller already owns (a fork)."""
        if not self._free_slots:
            raise OutOfPages("no free sequence slot")
        if len(pages) > self.max_pages_per_seq or self.pages_for(tokens) != len(pages):
            raise ValueError("adopt: page count does not match the token count")
        slot = heapq.heappop(self._free_slots)
        self.pages[slot] = list(pages)
        self.owner[slot] = owner
        self.table[slot, :len(pages)] = pages
        self.table[slot, len(pages):] = 0
        self.lengths[slot] = tokens
        self.active[slot] = True
        self.dirty_rows.add(slot)
        return slot

    def extend(self, slot: int, tokens: int) -> None:
        """Grow a sequence to `tokens` cached tokens (the rest of a prompt after a
        prefix-cache hit); takes the extra pages before changing anything."""
        have = self.pages[slot]
        need = self.pages_for(tokens) - len(have)
        if tokens < self.lengths[slot]:
            raise ValueError("extend cannot shrink a sequence")
        if len(have) + need > self.max_pages_per_seq:
            raise OutOfPages(f"{tokens} tokens exceed {self.max_pages_per_seq} pages per sequence")
        if need > 0:
            fresh = self.take_pages(need)
            self.table[slot, len(have):len(have) + need] = fresh
            have.extend(fresh)
        self.lengths[slot] = tokens
        self.dirty_rows.add(slot)

    def release(self, slot: int) -> None:
        """Drop a sequence's pages (freed when no snapshot shares them) and free its slot."""
        pages = self.pages.pop(slot)
        self.drop(pages)
        self.owner.pop(slot, None)
        self.lengths[slot] = 0
        self.active[slot] = False
        heapq.heappush(self._free_slots, slot)
        self.dirty_rows.add(slot)

    def take_dirty_rows(self) -> list:
        rows = sorted(self.dirty_rows)
        self.dirty_rows.clear()
        return rows
