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

    @property
    def num_layers(self) -> int:
        return self._num_layers

    @property
    def device(self) -> torch.device:
        return self._kv_buffer.device

    @property
    def dtype(self) -> torch.dtype:
        return self._kv_buffer.dtype
