"""Attention over shared prefix pages, split into a per-group prefix part and a per-row
suffix part (TEST INFRASTRUCTURE ONLY).

The specification a prefix-sharing attention pass has to meet: decode rows whose page
tables start with the same pages (the radix prefix cache gives a group of requests one
copy of a matched prefix, kvcache/radix_cache.py:92-99, 133-147) can attend over those
pages once per group. Each row's attention is then the merge of two partial results --
the group's prefix keys and the row's own remaining keys -- by their softmax statistics
(running max and sum), which must equal ``ops.paged_attention`` over the whole context.

* ``shared_prefix_groups`` finds the groups: rows with the same first page, and the whole
  pages that all of them share and hold entirely inside their contexts.
* ``attention_partial`` is one part: the unnormalised output, max and sum over a key range.
* ``merge_partials`` combines parts as the split-KV merge of the attention kernels does.
"""

from __future__ import annotations

import numpy as np
import torch


def shared_prefix_groups(page_table: np.ndarray, seq_lens: np.ndarray, page_size: int,
                         min_pages: int = 1) -> dict[str, np.ndarray]:
    """Groups of decode rows sharing leading pages.

    ``page_table[r, j]`` is row r's j-th page, ``seq_lens[r]`` its context length (keys).
    Returns CSR arrays: ``group_ptr`` [G+1] into ``group_rows``, ``group_prefix`` [G] (shared
    keys, whole pages, at most every member's context minus its last key so each row keeps
    a suffix), and ``row_prefix`` [rows] (the keys a row takes from its group, 0 if none).
    Rows are grouped by their first page, then a group's prefix is the longest run of pages
    common to all of its members; groups with fewer than ``min_pages`` shared pages or fewer
    than two rows are dropped.
    """
    rows = page_table.shape[0]
    row_prefix = np.zeros(rows, np.int64)
    by_first: dict[int, list[int]] = {}
    for r in range(rows):
        if seq_lens[r] > page_size:  # at least one whole page plus a key of its own
            by_first.setdefault(int(page_table[r, 0]), []).append(r)
    ptr, members, prefix = [0], [], []
    for first in sorted(by_first):
        rs = by_first[first]
        if len(rs) < 2:
            continue
        limit = min((int(seq_lens[r]) - 1) // page_size for r in rs)
        base = page_table[rs[0], :limit]
        common = limit
        for r in rs[1:]:
            diff = np.flatnonzero(page_table[r, :limit] != base)
            if diff.size:
                common = min(common, int(diff[0]))
        if common < min_pages:
            continue
        members.extend(rs)
        ptr.append(len(members))
        prefix.append(common * page_size)
        row_prefix[rs] = common * page_size
    return {"group_ptr": np.asarray(ptr, np.int64), "group_rows": np.asarray(members, np.int64),
            "group_prefix": np.asarray(prefix, np.int64), "row_prefix": row_prefix}


def attention_partial(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      pages: torch.Tensor, k_begin: int, k_end: int, scale: float):
    """One decode row's attention over keys [k_begin, k_end) of its page list: the
    unnormalised output ``[Hq, D]`` (fp32), the running max and the sum ``[Hq]``, with the
    max taken on ``scale * q.k`` (natural exponent)."""
    hq, d = q.shape
    page = k_cache.shape[1]
    hkv = k_cache.shape[2]
    if k_end <= k_begin:
        return (torch.zeros(hq, d), torch.full((hq,), float("-inf")), torch.zeros(hq))
    npages = (k_end + page - 1) // page
    keys = k_cache[pages[:npages].long()].reshape(npages * page, hkv, d)[k_begin:k_end].float()
    vals = v_cache[pages[:npages].long()].reshape(npages * page, hkv, d)[k_begin:k_end].float()
    keys = keys.repeat_interleave(hq // hkv, dim=1)
    vals = vals.repeat_interleave(hq // hkv, dim=1)
    scores = torch.einsum("hd,khd->hk", q.float(), keys) * scale
    m = scores.max(dim=1).values
    p = torch.exp(scores - m[:, None])
    return torch.einsum("hk,khd->hd", p, vals), m, p.sum(dim=1)


def merge_partials(parts) -> torch.Tensor:
    """Normalised output ``[Hq, D]`` of partial results over disjoint key ranges."""
    m = torch.stack([p[1] for p in parts]).max(dim=0).values
    num = torch.zeros_like(parts[0][0])
    den = torch.zeros_like(parts[0][2])
    for o, mi, li in parts:
        c = torch.where(torch.isfinite(mi), torch.exp(mi - m), torch.zeros_like(mi))
        num += o * c[:, None]
        den += li * c
    return num / den[:, None]
