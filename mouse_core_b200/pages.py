"""Host-side page allocator and block table of a paged KV cache.

The reference keeps one contiguous ``[layers, B, kv_heads, capacity, hd]``
buffer per session and doubles it (allocate + copy) whenever any row
overflows (src/mouse_core/models/backbone/flex_decode.py:109-114, 140-149).
Here every row owns a list of fixed-size pages drawn from a shared pool;
growing a row appends a page id to its block-table row, so nothing is copied.
Page ids are shared by all layers (each layer has its own pool slab).

The allocator runs on the host (numpy) because the caller already knows every
row's length there; the device copy of the block table is refreshed with one
host-to-device copy per call that changes it.
"""

from __future__ import annotations

import numpy as np


class PageTable:
    """Free list + per-row page lists + refcounts for ``num_pages`` pages."""

    def __init__(self, batch_size: int, num_pages: int, page_size: int, max_pages: int):
        self.B = int(batch_size)
        self.page_size = int(page_size)
        self.num_pages = int(num_pages)
        self.table = np.full((self.B, max(int(max_pages), 1)), -1, dtype=np.int32)
        self.npages = np.zeros(self.B, dtype=np.int64)
        self.refcount = np.zeros(self.num_pages, dtype=np.int32)
        self._free = np.arange(self.num_pages - 1, -1, -1, dtype=np.int32)  # stack, top = end
        self._nfree = self.num_pages
        self.dirty = True

    @property
    def max_pages(self) -> int:
        return self.table.shape[1]

    @property
    def free_pages(self) -> int:
        return self._nfree

    def grow_pool(self, new_num_pages: int) -> None:
        """Register pages ``num_pages .. new_num_pages-1`` as free (the caller
        has already enlarged the device pools)."""
        new_num_pages = int(new_num_pages)
        if new_num_pages <= self.num_pages:
            return
        extra = np.arange(new_num_pages - 1, self.num_pages - 1, -1, dtype=np.int32)
        # The stack holds every page id: pages in use now come back later.
        free = np.empty(new_num_pages, dtype=np.int32)
        free[: extra.shape[0]] = extra
        free[extra.shape[0]: extra.shape[0] + self._nfree] = self._free[: self._nfree]
        self._free = free
        self._nfree += extra.shape[0]
        rc = np.zeros(new_num_pages, dtype=np.int32)
        rc[: self.num_pages] = self.refcount
        self.refcount = rc
        self.num_pages = new_num_pages

    def ensure_width(self, max_pages: int) -> None:
        if max_pages > self.max_pages:
            width = max(int(max_pages), 2 * self.max_pages)
            t = np.full((self.B, width), -1, dtype=np.int32)
            t[:, : self.max_pages] = self.table
            self.table = t
            self.dirty = True

    def pages_needed(self, new_lengths: np.ndarray) -> np.ndarray:
        """Pages each row must add to hold ``new_lengths`` tokens."""
        need = (np.asarray(new_lengths, dtype=np.int64) + self.page_size - 1) // self.page_size
        return np.maximum(need - self.npages, 0)

    def allocate(self, add: np.ndarray) -> None:
        """Append ``add[b]`` fresh pages to row ``b`` (enough must be free)."""
        add = np.asarray(add, dtype=np.int64)
        total = int(add.sum())
        if total == 0:
            return
        if total > self._nfree:
            raise RuntimeError(f"page pool exhausted: need {total} pages, {self._nfree} free")
        self.ensure_width(int((self.npages + add).max()))
        ids = self._free[self._nfree - total: self._nfree][::-1].copy()
        self._nfree -= total
        rows = np.repeat(np.arange(self.B), add)
        starts = np.repeat(self.npages, add)
        offs = np.arange(total) - np.repeat(np.cumsum(add) - add, add)
        self.table[rows, starts + offs] = ids
        self.refcount[ids] += 1
        self.npages += add
        self.dirty = True

    def open_pages(self, rows: np.ndarray) -> np.ndarray:
        """Append one fresh page to each of ``rows`` (distinct, ascending; the
        table must have a free column for each) and return the ids: the same
        ids ``allocate`` hands out for one page per row. ``dirty`` is left
        as it is: the caller writes the new entries into the device table."""
        k = int(rows.shape[0])
        if k > self._nfree:
            raise RuntimeError(f"page pool exhausted: need {k} pages, {self._nfree} free")
        ids = self._free[self._nfree - k: self._nfree][::-1].copy()
        self._nfree -= k
        self.table[rows, self.npages[rows]] = ids
        self.refcount[ids] += 1
        self.npages[rows] += 1
        return ids

    def release_rows(self, rows) -> None:
        """Drop every page reference of ``rows`` (pages whose refcount reaches
        zero return to the free list) and empty those rows."""
        for b in np.atleast_1d(np.asarray(rows, dtype=np.int64)):
            n = int(self.npages[b])
            if n == 0:
                continue
            ids = self.table[b, :n].copy()
            self.refcount[ids] -= 1
            freed = ids[self.refcount[ids] == 0]
            if freed.size:
                self._free[self._nfree: self._nfree + freed.size] = freed
                self._nfree += freed.size
            self.table[b, :n] = -1
            self.npages[b] = 0
            self.dirty = True

    def share(self, dst_row: int, src_row: int, n_pages: int) -> None:
        """Make the first ``n_pages`` pages of ``dst_row`` the same pages as
        ``src_row``'s (refcounted, no copy). ``dst_row`` must be empty."""
        if self.npages[dst_row] != 0:
            raise ValueError("share() needs an empty destination row")
        n = int(n_pages)
        if n == 0:
            return
        ids = self.table[src_row, :n]
        self.ensure_width(n)
        self.table[dst_row, :n] = ids
        self.refcount[ids] += 1
        self.npages[dst_row] = n
        self.dirty = True

    def take_free(self, n: int) -> np.ndarray:
        """Pop ``n`` free page ids (refcount 1) for a caller that installs them."""
        if n > self._nfree:
            raise RuntimeError(f"page pool exhausted: need {n} pages, {self._nfree} free")
        ids = self._free[self._nfree - n: self._nfree][::-1].copy()
        self._nfree -= n
        self.refcount[ids] += 1
        return ids

    def slots(self, rows: np.ndarray, positions: np.ndarray) -> np.ndarray:
        """Pool slot (page * page_size + offset) of token ``positions`` of ``rows``."""
        pg = self.table[rows, positions // self.page_size].astype(np.int64)
        return pg * self.page_size + positions % self.page_size
