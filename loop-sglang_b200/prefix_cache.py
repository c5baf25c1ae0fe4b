"""Prefix caches with the reference's interface, over the native radix tree.

``RadixPrefixCache`` keeps the names, signatures, results and error behaviour of
the reference's ``RadixPrefixCache`` (python/loopsgl/kvcache/radix_cache.py:102-232)
and ``NoPrefixCache`` those of kvcache/no_prefix_cache.py:6-47; the result types
mirror kvcache/base.py:59-84. The tree itself is ``lsb_radix_*`` in
``libloopsgl_b200.so`` (host C++, ``csrc/radix.cpp``): a walk, split, lock or
eviction is one native call instead of a Python loop over nodes with a tensor
comparison per node.

Token ids are compared as int32 (vocabularies are far below 2**31); KV locations
are int32 as in the page table. The tree keeps the locations on the host; a
handle's ``get_matched_indices`` and ``evict`` return int32 tensors on the cache's
device, as the reference's do.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import NamedTuple

import numpy as np
import torch

from . import _lib


class SizeInfo(NamedTuple):
    evictable_size: int
    protected_size: int

    @property
    def total_size(self) -> int:
        return self.evictable_size + self.protected_size


@dataclass(frozen=True)
class RadixCacheHandle:
    """A matched or inserted prefix: its length and the tree node it ends at."""

    cached_len: int
    node: int
    cache: "RadixPrefixCache" = field(repr=False, compare=False)

    def get_matched_indices(self) -> torch.Tensor:
        return self.cache._indices(self.node, self.cached_len)


class InsertResult(NamedTuple):
    cached_len: int  # length already in the cache before insertion (the caller frees it)
    handle: RadixCacheHandle


class MatchResult(NamedTuple):
    cuda_handle: RadixCacheHandle


def _ids(x: torch.Tensor | np.ndarray | list) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        x = x.detach().cpu().numpy()
    a = np.ascontiguousarray(np.asarray(x), dtype=np.int32)
    if a.ndim != 1:
        raise ValueError("prefix cache keys must be 1-D")
    return a


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data if a.size else 0)


class RadixPrefixCache:
    """Radix tree of cached prefixes matched at page granularity."""

    def __init__(self, device: torch.device | str, page_size: int = 1) -> None:
        self.device = torch.device(device)
        self.page_size = int(page_size)
        self.empty_tensor = torch.empty(0, dtype=torch.int32, device=self.device)
        tree = ctypes.c_void_p()
        _lib.check(_lib.lib().lsb_radix_create(self.page_size, ctypes.byref(tree)), "radix_create")
        self._tree = tree

    def __del__(self) -> None:
        tree = getattr(self, "_tree", None)
        if tree is not None and tree.value:
            self._tree = None
            try:
                _lib.lib().lsb_radix_destroy(tree)
            except Exception:  # interpreter shutdown: the library may already be unloaded
                pass

    # -- the BasePrefixCache interface (kvcache/base.py:86-154) --

    def lock_handle(self, handle: RadixCacheHandle, unlock: bool = False) -> None:
        if not isinstance(handle, RadixCacheHandle) or handle.cache is not self:
            raise TypeError("lock_handle: not a handle of this cache")
        _lib.check(_lib.lib().lsb_radix_lock(self._tree, handle.node, int(bool(unlock))),
                   "radix_lock")

    def match_prefix(self, input_ids: torch.Tensor) -> MatchResult:
        ids = _ids(input_ids)
        node, pre = ctypes.c_int64(), ctypes.c_int64()
        _lib.check(_lib.lib().lsb_radix_match(self._tree, _ptr(ids), ids.size, ctypes.byref(node),
                                              ctypes.byref(pre)), "radix_match")
        return MatchResult(RadixCacheHandle(pre.value, node.value, self))

    def insert_prefix(self, input_ids: torch.Tensor, indices: torch.Tensor) -> InsertResult:
        ids, loc = _ids(input_ids), _ids(indices)
        if loc.size < ids.size:
            raise ValueError("insert_prefix: fewer indices than input ids")
        node, pre, ins = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        _lib.check(_lib.lib().lsb_radix_insert(self._tree, _ptr(ids), _ptr(loc), ids.size,
                                               ctypes.byref(node), ctypes.byref(pre),
                                               ctypes.byref(ins)), "radix_insert")
        return InsertResult(pre.value, RadixCacheHandle(ins.value, node.value, self))

    def evict(self, size: int) -> torch.Tensor:
        if size == 0:
            return self.empty_tensor
        evictable = self.size_info.evictable_size
        if size > evictable:
            raise RuntimeError(f"Cannot evict {size}, only {evictable} is evictable")
        out = np.empty(evictable, dtype=np.int32)
        n = ctypes.c_int64()
        _lib.check(_lib.lib().lsb_radix_evict(self._tree, int(size), _ptr(out), out.size,
                                              ctypes.byref(n)), "radix_evict")
        return torch.from_numpy(out[: n.value].copy()).to(self.device)

    def reset(self) -> None:
        raise NotImplementedError("RadixManager.reset is not implemented")

    @property
    def size_info(self) -> SizeInfo:
        e, p = ctypes.c_int64(), ctypes.c_int64()
        _lib.check(_lib.lib().lsb_radix_size_info(self._tree, ctypes.byref(e), ctypes.byref(p)),
                   "radix_size_info")
        return SizeInfo(evictable_size=e.value, protected_size=p.value)

    def check_integrity(self) -> None:
        """Recount the tree (links, keys, lock counts, size totals); raises on corruption."""
        _lib.check(_lib.lib().lsb_radix_check(self._tree), "radix_check")

    # -- helpers --

    def _indices(self, node: int, cached_len: int) -> torch.Tensor:
        if cached_len == 0:
            return self.empty_tensor
        out = np.empty(cached_len, dtype=np.int32)
        n = ctypes.c_int64()
        _lib.check(_lib.lib().lsb_radix_indices(self._tree, node, _ptr(out), out.size,
                                                ctypes.byref(n)), "radix_indices")
        return torch.from_numpy(out[: n.value].copy()).to(self.device)


def fast_compare_key(x: torch.Tensor, y: torch.Tensor) -> int:
    """Length of the common prefix of two 1-D int32/int64 CPU tensors
    (kernel/radix.py:18-20)."""
    for t in (x, y):
        if t.dim() != 1 or not t.is_contiguous() or t.device.type != "cpu" or \
                t.dtype not in (torch.int32, torch.int64):
            raise RuntimeError("Both tensors must be 1D CPU int tensors.")
    if x.dtype != y.dtype:
        raise RuntimeError("Both tensors must have the same dtype.")
    out = ctypes.c_int64()
    _lib.check(_lib.lib().lsb_fast_compare_key(
        ctypes.c_void_p(x.data_ptr()), x.numel(), ctypes.c_void_p(y.data_ptr()), y.numel(),
        32 if x.dtype == torch.int32 else 64, ctypes.byref(out)), "fast_compare_key")
    return out.value


@dataclass(frozen=True)
class NoPrefixCacheHandle:
    cached_len: int = 0
    empty_tensor: torch.Tensor | None = field(default=None, repr=False, compare=False)

    def get_matched_indices(self) -> torch.Tensor:
        return self.empty_tensor


class NoPrefixCache:
    """The prefix-cache interface without retaining or matching prefixes."""

    def __init__(self, device: torch.device | str) -> None:
        self.device = torch.device(device)
        self.empty_tensor = torch.empty(0, dtype=torch.int32, device=self.device)

    def lock_handle(self, handle, unlock: bool = False) -> None:
        pass

    def match_prefix(self, input_ids: torch.Tensor) -> MatchResult:
        return MatchResult(NoPrefixCacheHandle(0, self.empty_tensor))

    def insert_prefix(self, input_ids: torch.Tensor, indices: torch.Tensor) -> InsertResult:
        return InsertResult(0, NoPrefixCacheHandle(0, self.empty_tensor))

    def evict(self, size: int) -> torch.Tensor:
        if size == 0:
            return self.empty_tensor
        raise NotImplementedError("NoPrefixCache has no cached prefixes to evict.")

    def reset(self) -> None:
        pass

    @property
    def size_info(self) -> SizeInfo:
        return SizeInfo(evictable_size=0, protected_size=0)

    def check_integrity(self) -> None:
        pass


def create_prefix_cache(device: torch.device | str, disable_radix_cache: bool = False,
                        page_size: int = 1):
    """The radix cache or its no-reuse stand-in (kvcache/__init__.py:60-68; the
    reference reads the page size from its global context)."""
    if disable_radix_cache:
        return NoPrefixCache(device=device)
    return RadixPrefixCache(device=device, page_size=page_size)


# ------------------------------------------------------- shared-prefix groups --

@dataclass
class SharedPrefixGroups:
    """Decode rows grouped by the leading KV pages they share, in the CSR form
    ``lsb_paged_attention_shared_prefix`` reads (int32 device tensors).

    ``group_rows[group_ptr[g]:group_ptr[g + 1]]`` are group g's member rows, whose first
    ``group_prefix[g]`` keys are the same pages; ``row_prefix[r]`` is the prefix of row r's
    group (0 for rows in none).
    """

    group_ptr: torch.Tensor
    group_rows: torch.Tensor
    group_prefix: torch.Tensor
    row_prefix: torch.Tensor
    max_group_rows: int
    max_group_prefix: int

    @property
    def num_groups(self) -> int:
        return self.group_ptr.numel() - 1


def find_shared_prefixes(page_table: np.ndarray, seq_lens: np.ndarray, page_size: int,
                         device: torch.device | str, min_pages: int = 1,
                         max_rows: int = 64) -> SharedPrefixGroups | None:
    """Groups of decode rows whose page tables start with the same pages.

    What the radix cache gives requests that matched one prefix
    (kvcache/radix_cache.py:92-99, 133-147): the same page ids at the start of their
    tables. Rows are keyed by their first page; a group's prefix is the run of whole pages
    every member has in common, kept inside each member's context minus its last key (so
    each row keeps keys of its own). Groups of one row or with fewer than ``min_pages``
    shared pages are dropped, and groups of more than ``max_rows`` rows are cut into groups
    of at most ``max_rows`` over the same prefix. Host arrays in (taken when a batch is
    formed: a group stays valid while its rows only grow); None when nothing is shared.
    """
    page_table = np.asarray(page_table)
    seq_lens = np.asarray(seq_lens, dtype=np.int64)
    rows = page_table.shape[0]
    whole = (seq_lens - 1) // page_size  # whole pages strictly before each row's last key
    cand = np.flatnonzero(whole >= max(1, min_pages))
    if cand.size < 2:
        return None
    first = page_table[cand, 0]
    order = np.argsort(first, kind="stable")
    cand, first = cand[order], first[order]
    bounds = np.flatnonzero(np.diff(first)) + 1
    ptr, members, prefix = [0], [], []
    row_prefix = np.zeros(rows, np.int32)
    for rs in np.split(cand, bounds):
        if rs.size < 2:
            continue
        limit = int(whole[rs].min())
        block = page_table[rs, :limit]
        same = np.all(block == block[0], axis=0)  # pages common to every member
        common = limit if same.all() else int(np.argmin(same))
        if common < min_pages:
            continue
        for i in range(0, rs.size, max_rows):
            part = rs[i:i + max_rows]
            if part.size < 2:  # a lone remainder reads its prefix itself
                continue
            members.extend(part.tolist())
            ptr.append(len(members))
            prefix.append(common * page_size)
            row_prefix[part] = common * page_size
    if not prefix:
        return None
    sizes = np.diff(np.asarray(ptr))
    dev = torch.device(device)
    as_i32 = lambda a: torch.as_tensor(np.asarray(a, np.int32), device=dev)  # noqa: E731
    return SharedPrefixGroups(group_ptr=as_i32(ptr), group_rows=as_i32(members),
                              group_prefix=as_i32(prefix), row_prefix=as_i32(row_prefix),
                              max_group_rows=int(sizes.max()), max_group_prefix=int(max(prefix)))
