"""The host-side builder of shared-prefix groups (``prefix_cache.find_shared_prefixes``)
against the specification in ``oracle/prefix_share.py`` (same groups, same prefixes),
plus its cut of large groups into blocks of at most ``max_rows`` rows."""

from __future__ import annotations

import numpy as np

from __graft_entry__ import load_package
from oracle.prefix_share import shared_prefix_groups

load_package()
from loop_sglang_b200.prefix_cache import find_shared_prefixes  # noqa: E402


def _sets(ptr, rows, pre):
    return {(tuple(sorted(rows[ptr[i]:ptr[i + 1]].tolist())), int(pre[i]))
            for i in range(len(pre))}


def _random_tables(seed: int, page: int):
    rng = np.random.default_rng(seed)
    nxt = 1
    tables, lens = [], []
    prefixes = []
    for _ in range(rng.integers(1, 5)):
        n = int(rng.integers(1, 6))
        prefixes.append(list(range(nxt, nxt + n)))
        nxt += n
    for _ in range(int(rng.integers(2, 40))):
        if rng.random() < 0.7:
            pre = prefixes[int(rng.integers(len(prefixes)))]
            keep = int(rng.integers(1, len(pre) + 1))  # some rows diverge inside the prefix
            pages = pre[:keep]
        else:
            pages = []
        own = int(rng.integers(0, 5))
        pages = pages + list(range(nxt, nxt + own))
        nxt += own
        if not pages:
            pages = [nxt]
            nxt += 1
        n = (len(pages) - 1) * page + int(rng.integers(1, page + 1))
        tables.append(pages)
        lens.append(n)
    width = max(len(p) for p in tables)
    table = np.zeros((len(tables), width), np.int32)
    for r, p in enumerate(tables):
        table[r, :len(p)] = p
    return table, np.asarray(lens, np.int32)


def test_builder_matches_specification() -> None:
    for seed in range(40):
        page = [1, 4, 16][seed % 3]
        table, lens = _random_tables(seed, page)
        spec = shared_prefix_groups(table, lens, page)
        got = find_shared_prefixes(table, lens, page, "cpu", max_rows=10**6)
        if got is None:
            assert len(spec["group_prefix"]) == 0
            continue
        assert _sets(spec["group_ptr"], spec["group_rows"], spec["group_prefix"]) == _sets(
            got.group_ptr.numpy(), got.group_rows.numpy(), got.group_prefix.numpy())
        assert np.array_equal(spec["row_prefix"], got.row_prefix.numpy())
        assert got.max_group_prefix == int(spec["group_prefix"].max())


def test_large_groups_are_cut() -> None:
    page = 4
    table = np.zeros((130, 3), np.int32)
    table[:, 0] = 7
    table[:, 1] = 8
    table[:, 2] = np.arange(130) + 100
    lens = np.full(130, 10, np.int32)
    got = find_shared_prefixes(table, lens, page, "cpu", max_rows=64)
    sizes = np.diff(got.group_ptr.numpy())
    assert sizes.tolist() == [64, 64, 2] and got.max_group_rows == 64
    assert (got.group_prefix.numpy() == 8).all()
    # a lone remainder row keeps its prefix unshared
    got = find_shared_prefixes(table[:129], lens[:129], page, "cpu", max_rows=64)
    assert np.diff(got.group_ptr.numpy()).tolist() == [64, 64]
    assert int((got.row_prefix.numpy() == 0).sum()) == 1
