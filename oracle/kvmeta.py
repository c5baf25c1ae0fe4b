"""Integer bookkeeping of the looped-decoder hot path, restated on the CPU with numpy.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Covers the bit-exact parts of the path: KV slot indices per looped-KV policy,
attention metadata built from the token-granular page table, per-token batch
inputs (positions / out_loc), and the last-exited version maps (reserve, alias,
free, resolve). The reference implements the last four as Triton kernels with
atomics; where the reference's result depends on the order in which programs
run, this restatement fixes the order to ascending program id, which is the
order the Triton interpreter uses and the order the CUDA kernels of this
project reproduce with prefix sums.
"""

from __future__ import annotations

from dataclasses import dataclass
from math import gcd

import numpy as np

# ----------------------------------------------------------------------------
# KV slot index math (python/loopsgl/models/looped/base.py:59-91)
# ----------------------------------------------------------------------------

POLICIES = ("depth_indexed", "shared", "last_exited")


def num_kv_layers(policy: str, loop_steps: int, prelude: int, core: int, coda: int) -> int:
    """``BaseLoopedModel.num_kv_layers`` (base.py:59-71)."""
    if policy not in POLICIES:
        raise ValueError(f"unknown looped-KV policy {policy!r}")
    slots = loop_steps if policy == "depth_indexed" else 1
    return prelude + slots * core + coda


def prelude_cache_layer_index(layer_id: int) -> int:
    """base.py:73-74."""
    return layer_id


def core_cache_layer_index(policy: str, prelude: int, core: int, layer_id: int, loop_step) -> int:
    """base.py:76-88: depth-indexed adds ``loop_step * core``; it needs a scalar step."""
    if policy == "depth_indexed":
        if not isinstance(loop_step, (int, np.integer)) or isinstance(loop_step, bool):
            raise ValueError("Depth-indexed KV requires a scalar loop step")
        return prelude + int(loop_step) * core + layer_id
    return prelude + layer_id


def coda_cache_layer_index(policy: str, loop_steps: int, prelude: int, core: int, coda: int,
                           layer_id: int) -> int:
    """base.py:90-91."""
    return num_kv_layers(policy, loop_steps, prelude, core, coda) - coda + layer_id


# ----------------------------------------------------------------------------
# Attention metadata (python/loopsgl/attention/metadata.py:59-216)
# ----------------------------------------------------------------------------


def set_metadata(
    seq_lens: np.ndarray,
    extend_lens: np.ndarray,
    req_to_token: np.ndarray,
    req_pool_indices: np.ndarray,
    max_seq_pages: int,
    page_size: int,
    is_decode: bool,
    seq_len_delta: int = 0,
    page_table: np.ndarray | None = None,
):
    """``_fused_metadata_kernel_general`` (metadata.py:59-113).

    Returns ``(cache_seqlens, cu_seqlens_k, cu_seqlens_q, page_table)``; only the
    first ``min(ceil(seq/page), max_seq_pages)`` columns of each page-table row
    are written (``req_to_token[row, col*page] // page``), the rest keep their
    previous contents.
    """
    bs = len(seq_lens)
    seq = seq_lens.astype(np.int64) + seq_len_delta
    query = np.ones(bs, np.int64) if is_decode else extend_lens.astype(np.int64)
    cache_seqlens = seq.astype(np.int32)
    cu_k = np.zeros(bs + 1, np.int32)
    cu_q = np.zeros(bs + 1, np.int32)
    cu_k[1:] = np.cumsum(seq)
    cu_q[1:] = np.cumsum(query)
    if page_table is None:
        page_table = np.zeros((bs, max_seq_pages), np.int32)
    for b in range(bs):
        live = min(-(-int(seq[b]) // page_size), max_seq_pages)
        row = int(req_pool_indices[b])
        cols = np.arange(live)
        page_table[b, :live] = req_to_token[row, cols * page_size] // page_size
    return cache_seqlens, cu_k, cu_q, page_table


def prepare_batch_inputs(
    seq_lens: np.ndarray,
    extend_lens: np.ndarray,
    req_pool_indices: np.ndarray,
    req_to_token: np.ndarray,
    is_decode: bool,
):
    """``_prepare_batch_inputs`` (kernel/batch.py:72-103).

    Query token ``j`` of request ``r`` sits at ``seq_lens[r] - extend_lens[r] + j``;
    its KV location is ``req_to_token[req_pool_indices[r], pos]``. Returns
    ``(positions, req_mapping, out_loc)`` flattened over requests.
    """
    n = int(np.sum(extend_lens))
    positions = np.zeros(n, np.int32)
    mapping = np.zeros(n, np.int32)
    out_loc = np.zeros(n, np.int32)
    offset = 0
    for r in range(len(seq_lens)):
        q = int(extend_lens[r])
        start = r if is_decode else offset
        row = int(req_pool_indices[r])
        pos = int(seq_lens[r]) - q + np.arange(q)
        positions[start:start + q] = pos
        mapping[start:start + q] = row
        out_loc[start:start + q] = req_to_token[row, pos]
        offset += q
    return positions, mapping, out_loc


def assign_req_to_token_pool(
    req_pool_indices: np.ndarray,
    req_to_token: np.ndarray,
    start_offset: np.ndarray,
    end_offset: np.ndarray,
    out_cache_loc: np.ndarray,
) -> None:
    """``assign_req_to_token_pool`` (kernel/batch.py:17-46): copy each request's slice
    of ``out_cache_loc`` into ``req_to_token[row, start:end]``."""
    consumed = 0
    for r in range(len(req_pool_indices)):
        s, e = int(start_offset[r]), int(end_offset[r])
        row = int(req_pool_indices[r])
        req_to_token[row, s:e] = out_cache_loc[consumed:consumed + (e - s)]
        consumed += e - s


# ----------------------------------------------------------------------------
# Last-exited version maps (python/loopsgl/kvcache/last_exited.py:15-159,
# attention/metadata.py:220-291)
# ----------------------------------------------------------------------------


@dataclass
class LastExitedLayout:
    """Slot grouping of ``LastExitedKVCache.__init__`` (last_exited.py:111-159)."""

    num_layers: int
    core_start: int
    core_end: int
    loop_steps: int

    @property
    def num_core_layers(self) -> int:
        return self.core_end - self.core_start

    @property
    def layers_per_slot(self) -> int:
        return gcd(self.num_core_layers, self.num_layers - self.num_core_layers)

    @property
    def core_groups(self) -> int:
        return self.num_core_layers // self.layers_per_slot

    @property
    def fixed_groups(self) -> int:
        return (self.num_layers - self.num_core_layers) // self.layers_per_slot

    @property
    def slots_per_token(self) -> int:
        return self.fixed_groups + self.loop_steps * self.core_groups

    def num_kv_slots(self, num_pages: int) -> int:
        """``(num_pages - 1) * (num_layers // layers_per_slot) + 1`` (last_exited.py:129)."""
        return (num_pages - 1) * (self.num_layers // self.layers_per_slot) + 1

    def group_and_lane(self, layer: int) -> tuple[int, int]:
        """Per-layer ``(group, lane)`` (last_exited.py:151-159)."""
        if self.core_start <= layer < self.core_end:
            ordinal = layer - self.core_start
        elif layer < self.core_start:
            ordinal = layer
        else:
            ordinal = layer - self.num_core_layers
        return divmod(ordinal, self.layers_per_slot)


class LastExitedVersions:
    """Slot map, completed depths and the shared free-slot stack of ``LastExitedKVCache``."""

    def __init__(self, layout: LastExitedLayout, num_pages: int) -> None:
        self.layout = layout
        self.num_pages = num_pages
        self.num_kv_slots = layout.num_kv_slots(num_pages)
        self.slot_map = np.zeros((layout.slots_per_token, num_pages), np.int32)
        self.completed_depth = np.zeros(num_pages, np.int32)
        self.free_slots = np.arange(1, self.num_kv_slots, dtype=np.int32)
        self.free_count = self.num_kv_slots - 1

    @property
    def version_map(self) -> np.ndarray:
        """``slot_map[fixed:]`` viewed ``[steps, core_groups, pages]`` (last_exited.py:135-137)."""
        lay = self.layout
        return self.slot_map[lay.fixed_groups:].reshape(lay.loop_steps, lay.core_groups,
                                                        self.num_pages)

    @property
    def fixed_map(self) -> np.ndarray:
        """``slot_map[:fixed]`` with a leading depth axis (last_exited.py:134)."""
        return self.slot_map[: self.layout.fixed_groups][None]

    def reserve(self, handles: np.ndarray, restore_depths: np.ndarray | None = None) -> None:
        """``_reserve_versions`` (last_exited.py:15-47), tokens in ascending order.

        Each token pops ``fixed + depth*core`` rows off the top of the free stack;
        depths it did not compute alias the last computed version of each core group.
        """
        lay = self.layout
        fixed, core, steps = lay.fixed_groups, lay.core_groups, lay.loop_steps
        total = fixed + steps * core
        for t, handle in enumerate(handles):
            depth = int(restore_depths[t]) if restore_depths is not None else steps
            count = fixed + depth * core
            self.free_count -= count
            start = self.free_count
            for slot in range(total):
                if slot < fixed:
                    source = slot
                else:
                    source = fixed + min((slot - fixed) // core, depth - 1) * core + (slot - fixed) % core
                self.slot_map[slot, handle] = self.free_slots[start + source]
            self.completed_depth[handle] = depth

    def release(self, handles: np.ndarray, exits: np.ndarray | None = None) -> None:
        """``_release_versions`` (last_exited.py:50-84), tokens in ascending order.

        With ``exits`` (alias): versions at depths >= exit go back to the stack and
        those map entries alias the final computed version. Without: every version
        of the token is freed.
        """
        lay = self.layout
        fixed, core, steps = lay.fixed_groups, lay.core_groups, lay.loop_steps
        alias = exits is not None
        for t, handle in enumerate(handles):
            old_depth = int(self.completed_depth[handle])
            depth = int(exits[t]) if alias else 0
            end = fixed + old_depth * core
            begin = fixed + depth * core if alias else 0
            rows = self.slot_map[:end, handle].copy()
            start = self.free_count
            self.free_count += end - begin
            for slot in range(begin, end):
                self.free_slots[start + slot - begin] = rows[slot]
            if alias:
                finals = {}
                for slot in range(begin, fixed + steps * core):
                    final = fixed + (depth - 1) * core + (slot - fixed) % core
                    finals[slot] = self.slot_map[final, handle]
                for slot, value in finals.items():
                    self.slot_map[slot, handle] = value
            self.completed_depth[handle] = depth


def resolve_last_exited(
    logical_table: np.ndarray,
    version_map: np.ndarray,
    seq_lens: np.ndarray,
    cu_seqlens_q: np.ndarray,
    logical_out: np.ndarray,
    depths,
    physical_table: np.ndarray | None = None,
    physical_out: np.ndarray | None = None,
):
    """``_last_exited_metadata_kernel`` (metadata.py:220-257).

    ``version_map[depth, group, handle]`` -> physical slot. Row ``r`` resolves its
    first ``seq_lens[r]`` context handles and its own query rows of ``logical_out``
    at depth ``depths`` (scalar) or ``depths[r]``. Returns
    ``(physical_table[groups, rows, cols], physical_out[groups, n])``; entries
    outside the written ranges keep their previous contents.
    """
    groups = version_map.shape[1]
    rows, cols = logical_table.shape
    if physical_table is None:
        physical_table = np.zeros((groups, rows, cols), np.int32)
    if physical_out is None:
        physical_out = np.zeros((groups, len(logical_out)), np.int32)
    for g in range(groups):
        for r in range(rows):
            depth = int(depths) if np.isscalar(depths) else int(depths[r])
            n = min(int(seq_lens[r]), cols)
            handles = logical_table[r, :n]
            physical_table[g, r, :n] = version_map[depth, g, handles]
            s, e = int(cu_seqlens_q[r]), int(cu_seqlens_q[r + 1])
            physical_out[g, s:e] = version_map[depth, g, logical_out[s:e]]
    return physical_table, physical_out
