"""Shared-prefix decode attention (``lsb_paged_attention_shared_prefix``) against the oracle
and against plain paged attention on the same inputs.

Groups of decode rows point at one copy of their leading pages, as the radix prefix cache
lays them out; each group's prefix is read once for all of its rows (tensor-core pass into
split partials) and merged with each row's own keys by the decode kernel. The result must
equal ``oracle.ops.paged_attention`` within the bf16 tolerance, for groups of 2 to 70 rows
(more than one 64-row block), prefixes of one page to several prefix splits, rows in no
group, and repeated calls on one workspace (its arrival counters back at zero).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from __graft_entry__ import load_package
from oracle import ops as O
from oracle.prefix_share import shared_prefix_groups

load_package()
from loop_sglang_b200 import ops  # noqa: E402
from loop_sglang_b200.prefix_cache import find_shared_prefixes  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOL = dict(rtol=2e-2, atol=2e-2)


def _case(seed, hq, hkv, d, page, groups, loners, suffix):
    """``groups``: (members, prefix pages) per group; ``loners`` rows in no group; every
    row gets 1..suffix keys of its own after its group's prefix."""
    g = torch.Generator().manual_seed(seed)
    rows_pages, lens = [], []
    nxt = [1]

    def take(n):
        out = list(range(nxt[0], nxt[0] + n))
        nxt[0] += n
        return out

    for members, pre_pages in groups:
        pre = take(pre_pages)
        for _ in range(members):
            own = int(torch.randint(1, suffix + 1, (1,), generator=g))
            n = pre_pages * page + own
            rows_pages.append(pre + take((n + page - 1) // page - pre_pages))
            lens.append(n)
    for _ in range(loners):
        n = int(torch.randint(1, suffix + 1, (1,), generator=g))
        rows_pages.append(take((n + page - 1) // page))
        lens.append(n)
    perm = torch.randperm(len(rows_pages), generator=g).tolist()  # members interleaved
    rows_pages = [rows_pages[i] for i in perm]
    lens = [lens[i] for i in perm]
    width = max(len(p) for p in rows_pages)
    table = torch.zeros(len(rows_pages), width, dtype=torch.int32)
    for r, p in enumerate(rows_pages):
        table[r, :len(p)] = torch.tensor(p, dtype=torch.int32)
    num_pages = nxt[0] + 1
    kc = torch.randn(num_pages, page, hkv, d, generator=g).to(torch.bfloat16)
    vc = torch.randn(num_pages, page, hkv, d, generator=g).to(torch.bfloat16)
    q = torch.randn(len(lens), hq, d, generator=g).to(torch.bfloat16)
    return q, kc, vc, table, torch.tensor(lens, dtype=torch.int32)


@pytest.mark.parametrize("hq,hkv,d,page,groups,loners,suffix", [
    (16, 16, 128, 16, [(10, 128), (10, 128), (9, 3), (2, 1)], 5, 300),  # configs[3] heads
    (8, 8, 128, 16, [(70, 20), (3, 64)], 2, 200),    # a TP=2 rank; a 70-row group
    (16, 4, 64, 8, [(5, 40), (2, 2)], 3, 900),        # grouped-query KV, long own keys
    (32, 8, 96, 16, [(4, 33)], 0, 40),                # two heads per consumer warp
])
def test_shared_prefix_matches_oracle(hq, hkv, d, page, groups, loners, suffix) -> None:
    q, kc, vc, table, seq = _case(hq + d + page, hq, hkv, d, page, groups, loners, suffix)
    rows = seq.numel()
    cu = torch.arange(rows + 1, dtype=torch.int32)
    scale = d ** -0.5
    ref = O.paged_attention(q, kc, vc, table, seq, cu, scale)
    grp = find_shared_prefixes(table.numpy(), seq.numpy(), page, DEV, max_rows=128)
    assert grp is not None and grp.num_groups == len(groups)
    kd = kc.to(DEV).view(-1, hkv * d)
    vd = vc.to(DEV).view(-1, hkv * d)
    args = (q.to(DEV), kd, vd, table.to(DEV), seq.to(DEV), cu.to(DEV), page,
            int(table.shape[1] * page), scale, hkv)
    plain = ops.paged_attention(*args)
    for _ in range(2):  # the second call reuses the workspace: counters back at zero
        got = ops.paged_attention_shared_prefix(*args, groups=grp)
        torch.testing.assert_close(got.float().cpu(), ref.float(), **TOL)
        # the same keys, only the prefix's P is rounded to bf16 before PV
        torch.testing.assert_close(got.float(), plain.float(), rtol=1e-2, atol=1e-2)
    again = ops.paged_attention(*args)  # plain attention on the same workspace afterwards
    assert torch.equal(again, plain)
    assert ops.device_error_word(reset=True) == 0


def test_builder_groups_equal_the_specification() -> None:
    """On the GPU case layouts the builder's groups are the oracle specification's."""
    q, kc, vc, table, seq = _case(3, 4, 4, 32, 16, [(6, 5), (3, 1), (2, 7)], 4, 50)
    spec = shared_prefix_groups(table.numpy(), seq.numpy(), 16)
    grp = find_shared_prefixes(table.numpy(), seq.numpy(), 16, "cpu")
    as_sets = lambda ptr, rows, pre: {  # noqa: E731
        (tuple(sorted(rows[ptr[i]:ptr[i + 1]].tolist())), int(pre[i])) for i in range(len(pre))}
    assert as_sets(spec["group_ptr"], spec["group_rows"], spec["group_prefix"]) == as_sets(
        grp.group_ptr.numpy(), grp.group_rows.numpy(), grp.group_prefix.numpy())
    assert np.array_equal(spec["row_prefix"], grp.row_prefix.numpy())
