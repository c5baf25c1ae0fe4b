"""The native radix tree against the oracle restatement, beyond the recorded sequences.

1. The oracle (``oracle/radix.py``) reproduces the reference's recorded sequences
   (``tests/golden/radix.json``) exactly -- the same pin the native tree has.
2. Seeded random sequences (page sizes 1, 2, 4 and 16; small alphabets, so partial matches
   and splits are frequent; matches, locked inserts, releases, evictions of random sizes,
   unlocked probes) run through both; every result must agree and the native tree must
   pass its structural check after every step.
3. Several threads drive one native tree at once (calls are serialised inside); afterwards
   its structure and totals are consistent and everything unlocked is evictable.
"""

from __future__ import annotations

import json
import sys
import threading
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from __graft_entry__ import load_package  # noqa: E402
from oracle.radix import RadixTree  # noqa: E402

load_package()
from loop_sglang_b200.prefix_cache import RadixPrefixCache  # noqa: E402

CASES = json.loads((ROOT / "tests" / "golden" / "radix.json").read_text())["cases"]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"page{c['page_size']}")
def test_oracle_replays_reference_sequence(case: dict) -> None:
    tree = RadixTree(case["page_size"])
    handles = {}
    for i, op in enumerate(case["ops"]):
        want = op["want"]
        if op["kind"] == "request":
            node, pre = tree.match(op["ids"])
            tree.lock(node)
            matched = tree.indices(node)
            assert (pre, matched) == (want["match_len"], want["matched"]), i
            locs = matched + op["fresh"][pre:len(op["ids"])]
            cached, new, n = tree.insert(op["ids"], locs)
            tree.lock(node, unlock=True)
            tree.lock(new)
            handles[i] = new
            assert (cached, n, tree.indices(new)) == (want["cached_len"], want["insert_len"],
                                                      want["inserted"]), i
        elif op["kind"] == "finish":
            tree.lock(handles.pop(op["ref"]), unlock=True)
        elif op["kind"] == "evict":
            assert tree.evict(op["size"]) == want["evicted"], i
        else:
            node, pre = tree.match(op["ids"])
            assert (pre, tree.indices(node)) == (want["match_len"], want["matched"]), i
        assert [tree.evictable, tree.protected] == want["size_info"], i


def _ops(rng: np.random.Generator, page: int, n_ops: int):
    prefixes = [rng.integers(0, 3, int(rng.integers(1, 6)) * page).tolist() for _ in range(3)]
    for _ in range(n_ops):
        r = rng.random()
        if r < 0.5:
            ids = list(prefixes[int(rng.integers(0, 3))])[: int(rng.integers(0, 6 * page + 1))]
            ids += rng.integers(0, 3, int(rng.integers(0, 3 * page + 2))).tolist()
            yield "request", ids
        elif r < 0.75:
            yield "finish", float(rng.random())
        elif r < 0.9:
            yield "evict", float(rng.random())
        else:
            yield "probe", rng.integers(0, 3, int(rng.integers(0, 4 * page + 1))).tolist()


@pytest.mark.parametrize("page", [1, 2, 4, 16])
@pytest.mark.parametrize("seed", range(6))
def test_native_tree_matches_oracle(page: int, seed: int) -> None:
    rng = np.random.default_rng(1000 * page + seed)
    native, oracle = RadixPrefixCache("cpu", page_size=page), RadixTree(page)
    live: list[tuple] = []  # (native handle, oracle node)
    next_loc = page
    for kind, arg in _ops(rng, page, 250):
        if kind == "request":
            ids = torch.tensor(arg, dtype=torch.int32)
            h = native.match_prefix(ids).cuda_handle
            node, pre = oracle.match(arg)
            assert h.cached_len == pre
            native.lock_handle(h)
            oracle.lock(node)
            matched = h.get_matched_indices().tolist()
            assert matched == oracle.indices(node)
            fresh = list(range(next_loc, next_loc + len(arg) - pre))
            next_loc += len(fresh) + page
            locs = matched + fresh
            ins = native.insert_prefix(ids, torch.tensor(locs, dtype=torch.int32))
            cached, new, n = oracle.insert(arg, locs)
            assert (ins.cached_len, ins.handle.cached_len) == (cached, n)
            native.lock_handle(h, unlock=True)
            oracle.lock(node, unlock=True)
            native.lock_handle(ins.handle)
            oracle.lock(new)
            assert ins.handle.get_matched_indices().tolist() == oracle.indices(new)
            live.append((ins.handle, new))
        elif kind == "finish" and live:
            h, node = live.pop(int(arg * len(live)))
            native.lock_handle(h, unlock=True)
            oracle.lock(node, unlock=True)
        elif kind == "evict":
            size = int(arg * oracle.evictable)
            assert native.evict(size).tolist() == oracle.evict(size)
        elif kind == "probe":
            h = native.match_prefix(torch.tensor(arg, dtype=torch.int32)).cuda_handle
            node, pre = oracle.match(arg)
            assert (h.cached_len, h.get_matched_indices().tolist()) == (pre, oracle.indices(node))
        assert tuple(native.size_info) == (oracle.evictable, oracle.protected)
        native.check_integrity()


def test_threads_share_one_tree() -> None:
    cache = RadixPrefixCache("cpu", page_size=4)
    errors: list[BaseException] = []

    def worker(tid: int) -> None:
        try:
            rng = np.random.default_rng(tid)
            base = 1_000_000 * (tid + 1)
            for j in range(300):
                ids = torch.tensor(rng.integers(0, 3, int(rng.integers(4, 40))), dtype=torch.int32)
                h = cache.match_prefix(ids).cuda_handle
                cache.lock_handle(h)
                locs = torch.cat([h.get_matched_indices(),
                                  torch.arange(base + 64 * j, base + 64 * j + len(ids) - h.cached_len,
                                               dtype=torch.int32)])
                ins = cache.insert_prefix(ids, locs)
                cache.lock_handle(h, unlock=True)
                cache.lock_handle(ins.handle)
                cache.lock_handle(ins.handle, unlock=True)
        except BaseException as exc:  # reported below
            errors.append(exc)

    threads = [threading.Thread(target=worker, args=(t,)) for t in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    cache.check_integrity()
    info = cache.size_info
    assert info.protected_size == 0 and info.evictable_size > 0
    assert len(cache.evict(info.evictable_size)) == info.evictable_size
    assert tuple(cache.size_info) == (0, 0)
    cache.check_integrity()
