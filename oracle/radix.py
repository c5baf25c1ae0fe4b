"""The radix prefix tree restated in plain Python (TEST INFRASTRUCTURE ONLY).

Follows python/loopsgl/kvcache/radix_cache.py: nodes hold a run of ids and their KV
locations (:18-86), children are keyed by the first page of their run (:235-238), a walk
matches whole pages and splits a node matched part-way, stamping the walked path with the
walk's time (:206-232, :70-82), insertion adds the unmatched page-aligned tail as a new
node (:137-147), lock counts move path lengths between the evictable and protected totals
(:114-131), and eviction pops unlocked leaves oldest first, a parent joining once it has
become an unlocked leaf (:149-176). Time is a counter (the reference reads a monotonic
clock; only the order matters). Pinned to the reference's recorded sequences in
``tests/golden/radix.json``; the native tree (``csrc/radix.cpp``) is fuzzed against it.
"""

from __future__ import annotations

import heapq
import itertools


class _Node:
    __slots__ = ("key", "value", "parent", "children", "ref", "stamp")

    def __init__(self, stamp: int) -> None:
        self.key: list[int] = []
        self.value: list[int] = []
        self.parent: _Node | None = None
        self.children: dict[tuple, _Node] = {}
        self.ref = 0
        self.stamp = stamp

    def __lt__(self, other: "_Node") -> bool:
        return self.stamp < other.stamp


class RadixTree:
    def __init__(self, page_size: int) -> None:
        self.page = page_size
        self._clock = itertools.count(1)
        self.root = _Node(next(self._clock))
        self.root.ref = 1
        self.evictable = 0
        self.protected = 0

    def _key(self, ids) -> tuple:
        return tuple(ids[: self.page])

    def _split(self, node: _Node, pos: int) -> _Node:
        up = _Node(node.stamp)
        up.key, up.value = node.key[:pos], node.value[:pos]
        up.parent, up.ref = node.parent, node.ref
        node.parent.children[self._key(up.key)] = up
        node.key, node.value = node.key[pos:], node.value[pos:]
        node.parent = up
        up.children[self._key(node.key)] = node
        return up

    def _walk(self, ids: list[int]) -> tuple[_Node, int]:
        tic = next(self._clock)
        node, pre = self.root, 0
        while len(ids) - pre >= self.page:
            child = node.children.get(self._key(ids[pre:]))
            if child is None:
                break
            n = min(len(child.key), len(ids) - pre)
            common = next((i for i in range(n) if child.key[i] != ids[pre + i]), n)
            m = common // self.page * self.page
            pre += m
            if m != len(child.key):
                up = self._split(child, m)
                up.stamp = tic
                return up, pre
            child.stamp = tic
            node = child
        return node, pre

    def match(self, ids: list[int]) -> tuple[_Node, int]:
        return self._walk(list(ids))

    def insert(self, ids: list[int], locs: list[int]) -> tuple[int, _Node, int]:
        n = len(ids) // self.page * self.page
        ids, locs = list(ids[:n]), list(locs[:n])
        node, pre = self._walk(ids)
        if pre != n:
            new = _Node(next(self._clock))
            new.key, new.value = ids[pre:], locs[pre:]
            new.parent = node
            node.children[self._key(new.key)] = new
            self.evictable += n - pre
            node = new
        return pre, node, n

    def lock(self, node: _Node, unlock: bool = False) -> None:
        while node.parent is not None:
            if unlock:
                node.ref -= 1
                if node.ref == 0:
                    self.evictable += len(node.key)
                    self.protected -= len(node.key)
            else:
                if node.ref == 0:
                    self.evictable -= len(node.key)
                    self.protected += len(node.key)
                node.ref += 1
            node = node.parent

    @staticmethod
    def indices(node: _Node) -> list[int]:
        parts = []
        while node.parent is not None:
            parts.append(node.value)
            node = node.parent
        return [x for p in reversed(parts) for x in p]

    def evict(self, size: int) -> list[int]:
        if size == 0:
            return []
        if size > self.evictable:
            raise RuntimeError(f"Cannot evict {size}, only {self.evictable} is evictable")
        leaves, stack = [], [self.root]
        while stack:
            n = stack.pop()
            if not n.children:
                if n.ref == 0:
                    leaves.append(n)
            else:
                stack.extend(n.children.values())
        heapq.heapify(leaves)
        out: list[int] = []
        while len(out) < size:
            n = heapq.heappop(leaves)
            out.extend(n.value)
            self.evictable -= len(n.key)
            parent = n.parent
            del parent.children[self._key(n.key)]
            if not parent.children and parent.ref == 0:
                heapq.heappush(leaves, parent)
        return out
