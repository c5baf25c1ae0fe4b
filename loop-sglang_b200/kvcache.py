"""Device KV pools of the three looped-KV policies.

``MHAKVCache`` keeps the reference's paged layout ``[2, L, pages, page, Hkv, D]``
(python/loopsgl/kvcache/mha_pool.py:16-66), used by the depth-indexed and shared
policies; ``LastExitedKVCache`` keeps ``[2, layers_per_slot, slots, Hkv, D]`` with
its slot map, completed depths and free-slot stack on the device
(kvcache/last_exited.py:87-311), with reserve / alias / free and address
resolution run by this project's CUDA kernels.
"""

from __future__ import annotations

from math import gcd

import torch

from . import ops


class MHAKVCache:
    """Paged pool; page 0 is the padding page and is never written."""

    def __init__(self, num_kv_heads: int, num_layers: int, head_dim: int, num_pages: int,
                 page_size: int, device: torch.device, dtype: torch.dtype = torch.bfloat16,
                 zero: bool = True) -> None:
        alloc = torch.zeros if zero else torch.empty
        self._kv_buffer = alloc(2, num_layers, num_pages, page_size, num_kv_heads, head_dim,
                                dtype=dtype, device=device)
        self._kv_buffer[:, :, 0].zero_()
        self.num_kv_heads, self.head_dim = num_kv_heads, head_dim
        self.page_size = page_size
        self._num_layers = num_layers
        self._row = num_kv_heads * head_dim

    # reference accessors (mha_pool.py:36-41)
    def k_cache(self, index: int) -> torch.Tensor:
        return self._kv_buffer[0, index]

    def v_cache(self, index: int) -> torch.Tensor:
        return self._kv_buffer[1, index]

    def slots(self, index: int) -> tuple[torch.Tensor, torch.Tensor]:
        """``[slots, Hkv*D]`` views of one layer (slot = page*page_size + offset)."""
        return (self._kv_buffer[0, index].view(-1, self._row),
                self._kv_buffer[1, index].view(-1, self._row))

    def store_kv(self, k, v, out_loc, layer_id: int) -> None:
        """mha_pool.py:54-66."""
        kc, vc = self.slots(layer_id)
        ops.store_kv(kc, vc, out_loc, k, v)

    # retraction snapshots (mha_pool.py:68-105) --------------------------------
    @property
    def _row_bytes(self) -> int:
        return self._row * self._kv_buffer.element_size()

    def cpu_copy_size(self, num_tokens: int) -> int:
        return ops.kv_snapshot_bytes(num_tokens, self._row_bytes, self._num_layers)

    def get_cpu_copy(self, indices: torch.Tensor) -> torch.Tensor:
        """Every KV layer's rows of ``indices``, in token order: ``[2, L, n, Hkv, D]`` in
        pinned host memory (one gather kernel + one strided copy per staging chunk)."""
        idx = indices.to(device=self.device, dtype=torch.int32).contiguous()
        out = torch.empty(2, self._num_layers, idx.numel(), self.num_kv_heads, self.head_dim,
                          dtype=self.dtype, pin_memory=True)
        b = self._kv_buffer
        ops.kv_backup(out, b, self._num_layers, b.shape[2] * b.shape[3], self._row_bytes, idx,
                      self._num_layers)
        return out

    def load_cpu_copy(self, cpu_tensors: torch.Tensor, indices: torch.Tensor) -> None:
        """Restore exact KV values into new token locations."""
        expected = (2, self._num_layers, indices.numel(), self.num_kv_heads, self.head_dim)
        if (cpu_tensors.is_cuda or cpu_tensors.dtype != self.dtype
                or tuple(cpu_tensors.shape) != expected):
            raise ValueError("CPU KV backup does not match the destination pool and token count.")
        idx = indices.to(device=self.device, dtype=torch.int32).contiguous()
        b = self._kv_buffer
        ops.kv_restore(b, cpu_tensors.contiguous(), self._num_layers, b.shape[2] * b.shape[3],
                       self._row_bytes, idx, self._num_layers)

    @property
    def num_layers(self) -> int:
        return self._num_layers

    @property
    def device(self) -> torch.device:
        return self._kv_buffer.device

    @property
    def dtype(self) -> torch.dtype:
        return self._kv_buffer.dtype


class LastExitedKVCache:
    """Versioned slot pool of the last-exited policy; page size 1, logical handles are
    token locations, physical slots come from ``slot_map``."""

    def __init__(self, num_kv_heads: int, num_layers: int, head_dim: int, num_pages: int,
                 core_start: int, core_end: int, loop_steps: int, device: torch.device,
                 dtype: torch.dtype = torch.bfloat16, zero: bool = True) -> None:
        if not 0 <= core_start < core_end <= num_layers or loop_steps < 1:
            raise ValueError("Invalid recurrent KV layer range or loop depth.")
        if num_pages < 1:
            raise ValueError("KV pools must include at least the padding row.")
        self.core_start, self.core_end, self.loop_steps = core_start, core_end, loop_steps
        self._num_layers = num_layers
        num_core = core_end - core_start
        num_fixed = num_layers - num_core
        self.layers_per_slot = gcd(num_core, num_fixed)
        self.core_groups = num_core // self.layers_per_slot
        self.fixed_groups = num_fixed // self.layers_per_slot
        self.slots_per_token = self.fixed_groups + loop_steps * self.core_groups
        self.num_kv_slots = (num_pages - 1) * (num_layers // self.layers_per_slot) + 1
        self.available_slots = self.num_kv_slots - 1
        self.page_size = 1
        self.slot_map = torch.zeros(self.slots_per_token, num_pages, dtype=torch.int32,
                                    device=device)
        self.fixed_map = self.slot_map[: self.fixed_groups].unsqueeze(0)
        self.version_map = self.slot_map[self.fixed_groups:].view(loop_steps, self.core_groups,
                                                                  num_pages)
        self.completed_depth = torch.zeros(num_pages, dtype=torch.int32, device=device)
        self._free_slots = torch.arange(1, self.num_kv_slots, dtype=torch.int32, device=device)
        self._free_count = torch.tensor([self.available_slots], dtype=torch.int32, device=device)
        alloc = torch.zeros if zero else torch.empty
        self._kv_buffer = alloc(2, self.layers_per_slot, self.num_kv_slots, num_kv_heads,
                                head_dim, dtype=dtype, device=device)
        self._kv_buffer[:, :, 0].zero_()
        self._row = num_kv_heads * head_dim
        self.num_kv_heads, self.head_dim = num_kv_heads, head_dim
        self.layer_groups: list[int] = []
        self.layer_lanes: list[int] = []
        for layer in range(num_layers):
            if core_start <= layer < core_end:
                ordinal = layer - core_start
            elif layer < core_start:
                ordinal = layer
            else:
                ordinal = layer - num_core
            group, lane = divmod(ordinal, self.layers_per_slot)
            self.layer_groups.append(group)
            self.layer_lanes.append(lane)

    def is_core_layer(self, index: int) -> bool:
        return self.core_start <= index < self.core_end

    def k_cache(self, index: int) -> torch.Tensor:
        return self._kv_buffer[0, self.layer_lanes[index]].unsqueeze(1)

    def v_cache(self, index: int) -> torch.Tensor:
        return self._kv_buffer[1, self.layer_lanes[index]].unsqueeze(1)

    def slots(self, index: int) -> tuple[torch.Tensor, torch.Tensor]:
        lane = self.layer_lanes[index]
        return (self._kv_buffer[0, lane].view(-1, self._row),
                self._kv_buffer[1, lane].view(-1, self._row))

    def store_kv(self, k, v, out_loc, layer_id: int) -> None:
        """last_exited.py:298-311 (out_loc already physical)."""
        kc, vc = self.slots(layer_id)
        ops.store_kv(kc, vc, out_loc, k, v)

    # version maps (last_exited.py:181-248) -----------------------------------
    def reserve_versions(self, handles: torch.Tensor) -> None:
        needed = handles.numel() * self.slots_per_token
        if needed > self.available_slots:
            raise RuntimeError(
                f"KV pool exhausted: {needed} slots requested, {self.available_slots} available.")
        if handles.numel():
            ops.last_exited_reserve(self.slot_map, self.completed_depth, self._free_slots,
                                    self._free_count, handles, self.loop_steps,
                                    self.fixed_groups, self.core_groups)
            self.available_slots -= needed

    def alias_versions(self, handles: torch.Tensor, depths: torch.Tensor,
                       released_versions: int) -> None:
        if handles.numel() != depths.numel() or not (
                0 <= released_versions <= handles.numel() * (self.loop_steps - 1)):
            raise ValueError("Invalid exit metadata.")
        if handles.numel():
            ops.last_exited_release(self.slot_map, self.completed_depth, self._free_slots,
                                    self._free_count, handles, self.loop_steps,
                                    self.fixed_groups, self.core_groups, exits=depths)
            self.available_slots += released_versions * self.core_groups

    def free_versions(self, handles: torch.Tensor, released_slots: int) -> None:
        if not 0 <= released_slots <= handles.numel() * self.slots_per_token:
            raise ValueError("Invalid freed KV slot count.")
        if handles.numel():
            ops.last_exited_release(self.slot_map, self.completed_depth, self._free_slots,
                                    self._free_count, handles, self.loop_steps,
                                    self.fixed_groups, self.core_groups)
            self.available_slots += released_slots

    # retraction snapshots (last_exited.py:160-178, 255-290, 313-376) ---------
    @staticmethod
    def memory_per_page(num_layers: int, num_core_layers: int, loop_steps: int,
                        row_bytes: int) -> int:
        """Storage and allocator metadata bytes per nominal one-token page."""
        lps = gcd(num_core_layers, num_layers - num_core_layers)
        core_groups = num_core_layers // lps
        fixed_groups = (num_layers - num_core_layers) // lps
        mappings = fixed_groups + loop_steps * core_groups
        return 2 * num_layers * row_bytes + (mappings + 1 + fixed_groups + core_groups) * 4

    @property
    def _row_bytes(self) -> int:
        return self._row * self._kv_buffer.element_size()

    @property
    def _expanded_layers(self) -> int:
        return self._num_layers + (self.core_end - self.core_start) * (self.loop_steps - 1)

    def cpu_copy_size(self, num_tokens: int) -> int:
        return ops.kv_snapshot_bytes(num_tokens, self._row_bytes, self._num_layers,
                                     self.core_start, self.core_end, self.loop_steps, True)

    def get_cpu_copy(self, indices: torch.Tensor) -> torch.Tensor:
        """Exact KV bytes of every layer at every loop depth of ``indices``, then one int32
        completed depth per token, as a uint8 tensor in pinned host memory."""
        idx = indices.to(device=self.device, dtype=torch.int32).contiguous()
        out = torch.empty(self.cpu_copy_size(idx.numel()), dtype=torch.uint8, pin_memory=True)
        ops.kv_backup(out, self._kv_buffer, self.layers_per_slot, self.num_kv_slots,
                      self._row_bytes, idx, self._num_layers, slot_map=self.slot_map,
                      completed_depth=self.completed_depth, core_start=self.core_start,
                      core_end=self.core_end, steps=self.loop_steps)
        return out

    def restore_depths(self, backup: torch.Tensor, num_tokens: int) -> torch.Tensor:
        if (backup.dtype != torch.uint8 or backup.is_cuda
                or backup.numel() != self.cpu_copy_size(num_tokens)):
            raise ValueError("Invalid last-exited CPU KV backup.")
        depths = (backup[-num_tokens * 4:].view(torch.int32) if num_tokens
                  else torch.empty(0, dtype=torch.int32))
        if bool((depths < 1).any()) or bool((depths > self.loop_steps).any()):
            raise ValueError("CPU KV backup contains invalid completed depths.")
        return depths

    def restore_slots(self, backup: torch.Tensor, num_tokens: int) -> int:
        """Fixed-layer and recurrent slots a snapshot needs when restored."""
        depths = self.restore_depths(backup, num_tokens)
        return num_tokens * self.fixed_groups + int(depths.sum()) * self.core_groups

    def reserve_restore_versions(self, handles: torch.Tensor, backup: torch.Tensor) -> int:
        """Reserve exactly the versions the snapshot holds (its completed depths; deeper
        depths alias the last computed one). Returns the versions not reserved."""
        depths = self.restore_depths(backup, handles.numel())
        needed = handles.numel() * self.fixed_groups + int(depths.sum()) * self.core_groups
        if needed > self.available_slots:
            raise RuntimeError("Recurrent KV pool lacks space for the exact CPU snapshot.")
        if handles.numel():
            ops.last_exited_reserve(self.slot_map, self.completed_depth, self._free_slots,
                                    self._free_count, handles, self.loop_steps,
                                    self.fixed_groups, self.core_groups,
                                    restore_depths=depths.to(self.device).contiguous())
            self.available_slots -= needed
        return handles.numel() * self.loop_steps - int(depths.sum())

    def load_cpu_copy(self, cpu_tensors: torch.Tensor, indices: torch.Tensor) -> None:
        """Restore a snapshot after its versions have been reserved."""
        self.restore_depths(cpu_tensors, indices.numel())
        idx = indices.to(device=self.device, dtype=torch.int32).contiguous()
        ops.kv_restore(self._kv_buffer, cpu_tensors.contiguous(), self.layers_per_slot,
                       self.num_kv_slots, self._row_bytes, idx, self._num_layers,
                       slot_map=self.slot_map, core_start=self.core_start, core_end=self.core_end,
                       steps=self.loop_steps)

    @property
    def num_layers(self) -> int:
        return self._num_layers

    @property
    def device(self) -> torch.device:
        return self._kv_buffer.device

    @property
    def dtype(self) -> torch.dtype:
        return self._kv_buffer.dtype
