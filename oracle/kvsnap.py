"""KV snapshots for retraction, restated on the CPU (TEST INFRASTRUCTURE ONLY).

Checks ``lsb_kv_backup`` / ``lsb_kv_restore`` and the pools' ``get_cpu_copy`` /
``load_cpu_copy``. Pinned against the reference's own pools run on the CPU
(``tests/golden/kv_snapshot.npz``, made by ``tests/golden/make_golden.py``).

* Paged pool ``[2, L, pages, page, Hkv, D]``: the snapshot is ``[2, L, n, Hkv, D]``
  in the pool's dtype, row j of layer l = the pool row at token location
  ``indices[j]`` (kvcache/mha_pool.py:71-85); restore writes them back at new
  locations (:87-105).
* Last-exited pool ``[2, lanes, slots, Hkv, D]``: the snapshot is raw bytes,
  ``[2, E, n, Hkv, D]`` values (E = layers + core * (steps - 1): each core layer
  once per loop depth, through ``version_map[depth, group, handle]``; fixed layers
  through ``fixed_map[0, group, handle]``) followed by one int32 completed depth per
  token (kvcache/last_exited.py:317-346); restore validates those depths and writes
  every expanded layer back through the (already reserved) maps (:255-267, 348-376).
"""

from __future__ import annotations

import numpy as np
import torch

from .kvmeta import LastExitedLayout


def paged_backup(buf: torch.Tensor, indices) -> torch.Tensor:
    """``MHAKVCache.get_cpu_copy`` (mha_pool.py:71-85)."""
    idx = torch.as_tensor(np.asarray(indices, np.int64))
    two, layers = buf.shape[:2]
    rows = buf.reshape(two, layers, -1, *buf.shape[-2:])
    return rows[:, :, idx].clone()


def paged_restore(buf: torch.Tensor, backup: torch.Tensor, indices) -> None:
    """``MHAKVCache.load_cpu_copy`` (mha_pool.py:87-105)."""
    idx = torch.as_tensor(np.asarray(indices, np.int64))
    two, layers = buf.shape[:2]
    expected = (two, layers, len(idx), *buf.shape[-2:])
    if backup.dtype != buf.dtype or tuple(backup.shape) != expected:
        raise ValueError("CPU KV backup does not match the destination pool and token count.")
    rows = buf.view(two, layers, -1, *buf.shape[-2:])
    rows[:, :, idx] = backup


def expanded_layers(layout: LastExitedLayout) -> list[tuple[int, int]]:
    """``(layer, depth)`` of each expanded layer, in snapshot order (last_exited.py:329-344)."""
    out = []
    for layer in range(layout.num_layers):
        steps = layout.loop_steps if layout.core_start <= layer < layout.core_end else 1
        out += [(layer, d) for d in range(steps)]
    return out


def _row_map(layout: LastExitedLayout, slot_map: np.ndarray, layer: int, depth: int,
             handles: np.ndarray) -> np.ndarray:
    group, _ = layout.group_and_lane(layer)
    if layout.core_start <= layer < layout.core_end:
        row = layout.fixed_groups + depth * layout.core_groups + group
    else:
        row = group
    return slot_map[row, handles].astype(np.int64)


def slot_snapshot_bytes(layout: LastExitedLayout, n: int, row_bytes: int) -> int:
    """``LastExitedKVCache.cpu_copy_size`` (last_exited.py:317-318)."""
    return 2 * len(expanded_layers(layout)) * n * row_bytes + 4 * n


def slot_backup(buf: torch.Tensor, layout: LastExitedLayout, slot_map: np.ndarray,
                completed_depth: np.ndarray, indices) -> np.ndarray:
    """``LastExitedKVCache.get_cpu_copy`` (last_exited.py:320-346) -> uint8 bytes."""
    handles = np.asarray(indices, np.int64)
    parts = []
    for kv in range(2):
        for layer, depth in expanded_layers(layout):
            _, lane = layout.group_and_lane(layer)
            rows = _row_map(layout, slot_map, layer, depth, handles)
            parts.append(buf[kv, lane][torch.as_tensor(rows)].contiguous().view(torch.uint8)
                         .reshape(-1).numpy())
    parts.append(completed_depth[handles].astype(np.int32).view(np.uint8))
    return np.concatenate(parts) if parts else np.zeros(0, np.uint8)


def slot_restore_depths(backup: np.ndarray, layout: LastExitedLayout, n: int,
                        row_bytes: int) -> np.ndarray:
    """``LastExitedKVCache.restore_depths`` (last_exited.py:255-267)."""
    if backup.dtype != np.uint8 or backup.size != slot_snapshot_bytes(layout, n, row_bytes):
        raise ValueError("Invalid last-exited CPU KV backup.")
    depths = backup[backup.size - 4 * n:].view(np.int32) if n else np.zeros(0, np.int32)
    if (depths < 1).any() or (depths > layout.loop_steps).any():
        raise ValueError("CPU KV backup contains invalid completed depths.")
    return depths


def slot_restore(buf: torch.Tensor, layout: LastExitedLayout, slot_map: np.ndarray,
                 backup: np.ndarray, indices) -> None:
    """``LastExitedKVCache.load_cpu_copy`` (last_exited.py:348-376), after the versions
    were reserved with the snapshot's depths."""
    handles = np.asarray(indices, np.int64)
    n = len(handles)
    row_shape = tuple(buf.shape[-2:])
    row_bytes = int(np.prod(row_shape)) * buf.element_size()
    slot_restore_depths(backup, layout, n, row_bytes)
    exp = expanded_layers(layout)
    values = torch.from_numpy(backup[: backup.size - 4 * n].copy()).view(buf.dtype)
    values = values.view(2, len(exp), n, *row_shape)
    for kv in range(2):
        for e, (layer, depth) in enumerate(exp):
            _, lane = layout.group_and_lane(layer)
            rows = _row_map(layout, slot_map, layer, depth, handles)
            buf[kv, lane][torch.as_tensor(rows)] = values[kv, e]
