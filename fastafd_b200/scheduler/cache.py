"""CPU-side KV page ledgers owned by the coordinator.

The coordinator, not the GPU worker, decides which physical page backs which token:
every plan carries explicit page grants and the worker only applies them. Two managers:

* :class:`NaivePageLedger` - free-list of pages, no sharing.
* :class:`RadixPageCache` - page-granular radix tree over token ids for prefix reuse with
  reference counts and LRU eviction of unreferenced leaves.

Reference: python/minisgl/afd_scheduler.py:47-369 (_CpuNaiveCacheManager, _CpuRadixCacheManager),
python/minisgl/kvcache/radix_cache.py:97-225.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np


class OutOfPages(RuntimeError):
    pass


class NaivePageLedger:
    """Free-list allocator. Page 0 is reserved as the dummy page of padding rows."""

    def __init__(self, num_pages: int, page_size: int):
        if num_pages < 2:
            raise ValueError("need at least 2 pages (page 0 is the dummy page)")
        self.num_pages, self.page_size = num_pages, page_size
        self._free = np.arange(num_pages - 1, 0, -1, dtype=np.int32)   # stack, pops low ids first
        self._n_free = num_pages - 1

    @property
    def free_pages(self) -> int:
        return self._n_free

    def pages_for(self, tokens: int) -> int:
        return (tokens + self.page_size - 1) // self.page_size

    def allocate(self, n: int) -> np.ndarray:
        if n > self._n_free:
            raise OutOfPages(f"need {n} pages, {self._n_free} free")
        out = self._free[self._n_free - n:self._n_free][::-1].copy()
        self._n_free -= n
        return out

    def free(self, pages: Sequence[int]) -> None:
        n = len(pages)
        if n == 0:
            return
        if self._n_free + n > self.num_pages - 1:
            raise RuntimeError("double free of KV pages")
        self._free[self._n_free:self._n_free + n] = np.asarray(pages, dtype=np.int32)[::-1]
        self._n_free += n

    # prefix-cache interface (no sharing here)
    def match_prefix(self, ids: Sequence[int]) -> Tuple[List[int], object]:
        return [], None

    def release(self, handle, ids: Sequence[int], pages: Sequence[int], cache_upto: int) -> None:
        self.free(pages)

    def check_integrity(self) -> None:
        live = self._free[:self._n_free]
        if len(np.unique(live)) != len(live) or (live <= 0).any() or (live >= self.num_pages).any():
            raise RuntimeError("page free-list corrupted")


@dataclass
class _Node:
    key: Tuple[int, ...]                 # page_size token ids
    page: int
    parent: Optional["_Node"]
    children: Dict[Tuple[int, ...], "_Node"] = field(default_factory=dict)
    ref: int = 0
    last_use: float = 0.0


_HOST_LIB = None


def _host_lib():
    """The native control-plane helpers (csrc/host/host_runtime.cpp), built on first use;
    None when no host compiler is available."""
    global _HOST_LIB
    if _HOST_LIB is None:
        import ctypes as C

        from ..build import build_host_lib
        try:
            lib = C.CDLL(str(build_host_lib()))
            for fn in (lib.afd_mismatch_i32, lib.afd_mismatch_i64):
                fn.restype = C.c_int64
                fn.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
            lib.afd_decode_out_loc.restype = C.c_int64
            lib.afd_decode_out_loc.argtypes = [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_int64, C.c_int32,
                                               C.c_int64, C.c_void_p]
            _HOST_LIB = lib
        except (OSError, RuntimeError):
            _HOST_LIB = False
    return _HOST_LIB or None


def mismatch_index(a: Sequence[int], b: Sequence[int]) -> int:
    """First index where two id sequences differ (the reference's native radix helper,
    python/minisgl/kernel/csrc/src/radix.cpp). Arrays of one integer dtype go to the native
    routine; anything else is compared with numpy."""
    a = np.asarray(a)
    b = np.asarray(b)
    n = min(len(a), len(b))
    if n == 0:
        return 0
    lib = _host_lib()
    if lib is not None and a.dtype == b.dtype and a.dtype in (np.int32, np.int64) \
            and a.flags.c_contiguous and b.flags.c_contiguous:
        fn = lib.afd_mismatch_i32 if a.dtype == np.int32 else lib.afd_mismatch_i64
        return int(fn(a.ctypes.data, b.ctypes.data, n))
    neq = np.nonzero(a[:n] != b[:n])[0]
    return int(neq[0]) if len(neq) else n


def decode_out_loc(page_table: np.ndarray, rows: np.ndarray, positions: np.ndarray, page_size: int,
                   num_pages: int) -> np.ndarray:
    """KV slot of each request's next token: page_table[row][pos // page_size] * page_size +
    pos % page_size, for int32 arrays (page_table 2-D, C-contiguous). Raises if a request's page is
    missing (negative entry) or outside the pool - the host-side twin of the bounds check that the
    store kernel makes on the device."""
    pt = np.ascontiguousarray(page_table, dtype=np.int32)
    rows = np.ascontiguousarray(rows, dtype=np.int32)
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    out = np.empty(len(rows), dtype=np.int32)
    lib = _host_lib()
    if lib is not None:
        bad = int(lib.afd_decode_out_loc(pt.ctypes.data, pt.shape[1], rows.ctypes.data, pos.ctypes.data, len(rows),
                                         page_size, num_pages, out.ctypes.data))
    else:
        col = pos // page_size
        ok = (pos >= 0) & (col < pt.shape[1])
        pages = np.where(ok, pt[rows, np.minimum(col, pt.shape[1] - 1)], -1)
        ok &= (pages >= 0) & (pages < num_pages)
        bad = int(np.argmin(ok)) if not ok.all() else -1
        out[:] = pages * page_size + pos % page_size
    if bad >= 0:
        raise IndexError(f"request {bad} (table row {int(rows[bad])}, position {int(pos[bad])}) has no valid KV page")
    return out


class RadixPageCache(NaivePageLedger):
    """Prefix cache at page granularity: a trie whose edges are whole pages of token ids.

    `match_prefix` pins the matched path (ref += 1) and returns its pages; `release` unpins
    it and inserts the request's fully written pages so later requests can share them.
    Unreferenced leaves are evicted in LRU order when the free list runs dry."""

    def __init__(self, num_pages: int, page_size: int):
        super().__init__(num_pages, page_size)
        self.root = _Node((), -1, None)
        self._cached_pages = 0

    def match_prefix(self, ids: Sequence[int]) -> Tuple[List[int], object]:
        ps, node, pages = self.page_size, self.root, []
        path: List[_Node] = []
        # never match the whole prompt: the last token must be recomputed to get logits
        limit = (len(ids) - 1) // ps
        for i in range(limit):
            key = tuple(ids[i * ps:(i + 1) * ps])
            child = node.children.get(key)
            if child is None:
                break
            path.append(child)
            pages.append(child.page)
            node = child
        now = time.monotonic()
        for n in path:
            n.ref += 1
            n.last_use = now
        return pages, path

    def allocate(self, n: int) -> np.ndarray:
        if n > self._n_free:
            self._evict(n - self._n_free)
        return super().allocate(n)

    def _evict(self, need: int) -> None:
        leaves = [x for x in self._iter_nodes() if not x.children and x.ref == 0]
        leaves.sort(key=lambda x: x.last_use)
        freed = 0
        while freed < need and leaves:
            leaf = leaves.pop(0)
            parent = leaf.parent
            del parent.children[leaf.key]
            super().free([leaf.page])
            self._cached_pages -= 1
            freed += 1
            if parent is not self.root and not parent.children and parent.ref == 0:
                leaves.append(parent)
                leaves.sort(key=lambda x: x.last_use)
        if freed < need:
            raise OutOfPages(f"need {need} more pages; cache has no evictable leaf")

    def _iter_nodes(self):
        stack = list(self.root.children.values())
        while stack:
            n = stack.pop()
            yield n
            stack.extend(n.children.values())

    def release(self, handle, ids: Sequence[int], pages: Sequence[int], cache_upto: int) -> None:
        """`pages` are all pages of the request (shared prefix first). Tokens [0, cache_upto)
        have valid KV. Shared pages are unpinned; own full pages are inserted into the tree;
        the rest is freed."""
        path: List[_Node] = handle or []
        for n in path:
            n.ref -= 1
        ps = self.page_size
        node = path[-1] if path else self.root
        full = cache_upto // ps
        now = time.monotonic()
        to_free = []
        for i in range(len(path), len(pages)):
            page = int(pages[i])
            if i < full:
                key = tuple(ids[i * ps:(i + 1) * ps])
                child = node.children.get(key)
                if child is None:
                    child = _Node(key, page, node, last_use=now)
                    node.children[key] = child
                    self._cached_pages += 1
                else:
                    to_free.append(page)     # someone inserted the same prefix meanwhile
                node = child
            else:
                to_free.append(page)
        self.free(to_free)

    @property
    def cached_pages(self) -> int:
        return self._cached_pages

    def check_integrity(self) -> None:
        super().check_integrity()
        tree_pages = [n.page for n in self._iter_nodes()]
        if len(set(tree_pages)) != len(tree_pages):
            raise RuntimeError("a page appears twice in the radix tree")
        if set(tree_pages) & set(self._free[:self._n_free].tolist()):
            raise RuntimeError("a cached page is also on the free list")
        if any(n.ref < 0 for n in self._iter_nodes()):
            raise RuntimeError("negative reference count")


def make_page_cache(kind: str, num_pages: int, page_size: int) -> NaivePageLedger:
    if kind == "naive":
        return NaivePageLedger(num_pages, page_size)
    if kind == "radix":
        return RadixPageCache(num_pages, page_size)
    raise ValueError(f"cache_type must be naive or radix, got {kind}")
