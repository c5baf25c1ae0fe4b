"""Prefix-sharing attention, specified on the CPU: rows grouped by shared leading pages,
attention merged from a per-group prefix part and a per-row suffix part, equal to plain
paged attention (``oracle/ops.paged_attention``, pinned to the reference's attention
backend through the golden fixtures)."""

from __future__ import annotations

import torch

from oracle import ops as O
from oracle.prefix_share import attention_partial, merge_partials, shared_prefix_groups


def _case(seed: int, page: int = 4, hq: int = 4, hkv: int = 2, d: int = 16):
    """Eleven decode rows: three groups sharing 3, 5 and 2 pages (interleaved), two rows
    with private pages only, one group whose rows diverge after their first page."""
    g = torch.Generator().manual_seed(seed)
    n_pages = 200
    kc = torch.randn(n_pages, page, hkv, d, generator=g).to(torch.bfloat16)
    vc = torch.randn(n_pages, page, hkv, d, generator=g).to(torch.bfloat16)
    nxt = [1]

    def take(n):
        out = list(range(nxt[0], nxt[0] + n))
        nxt[0] += n
        return out

    prefixes = [take(3), take(5), take(2)]
    spec = [(0, 20), (1, 31), (2, 13), (0, 17), (1, 24), (2, 9), (None, 14), (None, 6),
            (0, 13), ("split", 15), ("split", 10)]
    split_first = take(1)
    rows, lens = [], []
    for grp, n in spec:
        pages_needed = (n + page - 1) // page
        if grp is None:
            pages = take(pages_needed)
        elif grp == "split":
            pages = split_first + take(pages_needed - 1)
        else:
            pre = prefixes[grp]
            pages = pre[:pages_needed] + take(max(0, pages_needed - len(pre)))
        rows.append(pages)
        lens.append(n)
    width = max(len(p) for p in rows)
    table = torch.zeros(len(rows), width, dtype=torch.int32)
    for r, p in enumerate(rows):
        table[r, :len(p)] = torch.tensor(p, dtype=torch.int32)
    q = torch.randn(len(rows), hq, d, generator=g).to(torch.bfloat16)
    return q, kc, vc, table, torch.tensor(lens, dtype=torch.int32), page


def test_groups_follow_shared_pages() -> None:
    q, kc, vc, table, seq, page = _case(0)
    g = shared_prefix_groups(table.numpy(), seq.numpy(), page)
    groups = [sorted(g["group_rows"][g["group_ptr"][i]:g["group_ptr"][i + 1]].tolist())
              for i in range(len(g["group_prefix"]))]
    by_rows = dict(zip(map(tuple, groups), g["group_prefix"].tolist()))
    # group 0: rows 0, 3, 8 share 3 pages, but row 8 (13 keys) keeps its last key private
    assert by_rows[(0, 3, 8)] == 12
    assert by_rows[(1, 4)] == 20  # 5 shared pages, both rows longer than 20 keys
    assert by_rows[(2, 5)] == 8   # 2 shared pages, row 5 has 9 keys
    assert by_rows[(9, 10)] == 4  # rows that diverge after one page share that page
    assert g["row_prefix"][6] == 0 and g["row_prefix"][7] == 0
    assert len(groups) == 4


def test_merged_parts_equal_plain_attention() -> None:
    for seed in range(3):
        q, kc, vc, table, seq, page = _case(seed)
        scale = 16 ** -0.5
        cu = torch.arange(len(seq) + 1, dtype=torch.int32)
        ref = O.paged_attention(q, kc, vc, table, seq, cu, scale).float()
        g = shared_prefix_groups(table.numpy(), seq.numpy(), page)
        for r in range(len(seq)):
            pre = int(g["row_prefix"][r])
            parts = [attention_partial(q[r], kc, vc, table[r], 0, pre, scale),
                     attention_partial(q[r], kc, vc, table[r], pre, int(seq[r]), scale)]
            got = merge_partials(parts)
            torch.testing.assert_close(got, ref[r], rtol=2e-2, atol=2e-2)
        # every member of a group reads the same prefix pages: one read serves the group
        for i in range(len(g["group_prefix"])):
            members = g["group_rows"][g["group_ptr"][i]:g["group_ptr"][i + 1]]
            n = int(g["group_prefix"][i]) // page
            lead = table[int(members[0]), :n]
            assert all(torch.equal(table[int(m), :n], lead) for m in members)


def test_empty_prefix_part_is_neutral() -> None:
    q, kc, vc, table, seq, page = _case(5)
    scale = 16 ** -0.5
    whole = attention_partial(q[6], kc, vc, table[6], 0, int(seq[6]), scale)
    empty = attention_partial(q[6], kc, vc, table[6], 0, 0, scale)
    torch.testing.assert_close(merge_partials([empty, whole]), merge_partials([whole]))
