"""The native radix prefix cache against the reference's own tree.

``tests/golden/radix.json`` holds, for page sizes 1 and 4, a seeded scheduler-like
sequence (match, lock, insert with fresh page-aligned locations, unlock, evict,
unlocked probes) and every result the reference's ``RadixPrefixCache``
(kvcache/radix_cache.py:102-232) gave: match and insert lengths, matched and
inserted locations, evicted locations in eviction order, and the size totals after
each step. The replay here must reproduce all of them exactly, and the tree must
pass its own structural check after every step. Host code only: no GPU.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from __graft_entry__ import load_package  # noqa: E402

load_package()
from loop_sglang_b200.prefix_cache import (  # noqa: E402
    NoPrefixCache,
    RadixPrefixCache,
    create_prefix_cache,
    fast_compare_key,
)

CASES = json.loads((ROOT / "tests" / "golden" / "radix.json").read_text())["cases"]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"page{c['page_size']}")
def test_radix_replay_matches_reference(case: dict) -> None:
    cache = RadixPrefixCache("cpu", page_size=case["page_size"])
    handles = {}
    for i, op in enumerate(case["ops"]):
        want = op["want"]
        if op["kind"] == "request":
            ids = torch.tensor(op["ids"], dtype=torch.int32)
            m = cache.match_prefix(ids).cuda_handle
            cache.lock_handle(m)
            matched = m.get_matched_indices()
            assert (m.cached_len, matched.tolist()) == (want["match_len"], want["matched"]), i
            loc = torch.cat([matched, torch.tensor(op["fresh"][m.cached_len:len(op["ids"])],
                                                   dtype=torch.int32)])
            ins = cache.insert_prefix(ids, loc)
            cache.lock_handle(m, unlock=True)
            cache.lock_handle(ins.handle)
            handles[i] = ins.handle
            got = (ins.cached_len, ins.handle.cached_len, ins.handle.get_matched_indices().tolist())
            assert got == (want["cached_len"], want["insert_len"], want["inserted"]), i
        elif op["kind"] == "finish":
            cache.lock_handle(handles.pop(op["ref"]), unlock=True)
        elif op["kind"] == "evict":
            assert cache.evict(op["size"]).tolist() == want["evicted"], i
        else:
            h = cache.match_prefix(torch.tensor(op["ids"], dtype=torch.int32)).cuda_handle
            assert (h.cached_len, h.get_matched_indices().tolist()) == (want["match_len"],
                                                                        want["matched"]), i
        assert list(cache.size_info) == want["size_info"], i
        cache.check_integrity()


def test_radix_edge_cases() -> None:
    c = RadixPrefixCache("cpu", page_size=2)
    empty = torch.empty(0, dtype=torch.int32)
    # nothing cached, an odd-length key (the partial last page is never inserted)
    assert c.match_prefix(empty).cuda_handle.cached_len == 0
    r = c.insert_prefix(torch.tensor([1, 2, 3], dtype=torch.int32),
                        torch.tensor([10, 11, 12], dtype=torch.int32))
    assert (r.cached_len, r.handle.cached_len) == (0, 2)
    assert r.handle.get_matched_indices().tolist() == [10, 11]
    assert tuple(c.size_info) == (2, 0) and c.size_info.total_size == 2
    # a partial match splits the node at the page boundary, keeping the handle valid
    r2 = c.insert_prefix(torch.tensor([1, 2, 5, 6], dtype=torch.int32),
                         torch.tensor([20, 21, 22, 23], dtype=torch.int32))
    assert r2.cached_len == 2 and r2.handle.get_matched_indices().tolist() == [10, 11, 22, 23]
    c.lock_handle(r2.handle)
    assert tuple(c.size_info) == (0, 4)
    # unlocking twice is refused and changes nothing
    c.lock_handle(r2.handle, unlock=True)
    with pytest.raises(ValueError):
        c.lock_handle(r2.handle, unlock=True)
    assert tuple(c.size_info) == (4, 0)
    # asking for more than is evictable raises and evicts nothing
    with pytest.raises(RuntimeError):
        c.evict(5)
    assert tuple(c.size_info) == (4, 0)
    assert c.evict(0).numel() == 0
    # eviction frees whole leaves (possibly more than asked), oldest first
    assert c.evict(1).tolist() == [22, 23]
    # a handle to an evicted node is refused instead of read
    with pytest.raises(ValueError):
        r2.handle.get_matched_indices()
    assert sorted(c.evict(2).tolist()) == [10, 11]
    assert tuple(c.size_info) == (0, 0)
    c.check_integrity()
    with pytest.raises(NotImplementedError):
        c.reset()


def test_fast_compare_key_known_answers() -> None:
    for dt in (torch.int32, torch.int64):
        a = torch.tensor([1, 2, 3, 4], dtype=dt)
        assert fast_compare_key(a, torch.tensor([1, 2, 9], dtype=dt)) == 2
        assert fast_compare_key(a, a.clone()) == 4
        assert fast_compare_key(a, torch.tensor([1, 2], dtype=dt)) == 2
        assert fast_compare_key(a, torch.tensor([], dtype=dt)) == 0
    with pytest.raises(RuntimeError):
        fast_compare_key(torch.tensor([1]), torch.tensor([1], dtype=torch.int32))
    with pytest.raises(RuntimeError):
        fast_compare_key(torch.ones(2, 2, dtype=torch.int32), torch.ones(2, dtype=torch.int32))


def test_no_prefix_cache() -> None:
    c = create_prefix_cache("cpu", disable_radix_cache=True)
    assert isinstance(c, NoPrefixCache)
    ids = torch.arange(8, dtype=torch.int32)
    assert c.match_prefix(ids).cuda_handle.cached_len == 0
    r = c.insert_prefix(ids, ids)
    assert r.cached_len == 0 and r.handle.get_matched_indices().numel() == 0
    assert tuple(c.size_info) == (0, 0) and c.evict(0).numel() == 0
    with pytest.raises(NotImplementedError):
        c.evict(1)
    assert isinstance(create_prefix_cache("cpu", page_size=4), RadixPrefixCache)
