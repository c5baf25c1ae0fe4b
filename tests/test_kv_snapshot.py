"""KV snapshots for retraction: the reference's byte format, both pools.

``tests/golden/kv_snapshot.npz`` holds the reference's own ``get_cpu_copy`` /
``load_cpu_copy`` results (``MHAKVCache`` and ``LastExitedKVCache`` on the CPU, fp32,
the last-exited snapshot taken over tokens that exited at different depths). The
CPU tests pin the oracle restatement (``oracle/kvsnap.py``) to them; the GPU tests
run this project's pools (gather / scatter kernels + strided copies through
``lsb_kv_backup`` / ``lsb_kv_restore``) against the same fixture bit-exactly, then
through full-size round trips with several staging chunks against the oracle.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from oracle import kvsnap  # noqa: E402
from oracle.kvmeta import LastExitedLayout, LastExitedVersions  # noqa: E402

FIX = np.load(ROOT / "tests" / "golden" / "kv_snapshot.npz")
LAYOUT = LastExitedLayout(num_layers=6, core_start=1, core_end=5, loop_steps=3)


# ------------------------------------------------------------------ CPU: oracle pin --

def test_oracle_paged_snapshot_matches_reference() -> None:
    pool = torch.from_numpy(FIX["mha_pool"].copy())
    snap = kvsnap.paged_backup(pool, FIX["mha_src"])
    assert np.array_equal(snap.numpy(), FIX["mha_snapshot"])
    fresh = torch.zeros_like(pool)
    kvsnap.paged_restore(fresh, snap, FIX["mha_dst"])
    assert np.array_equal(fresh.numpy(), FIX["mha_restored"])
    with pytest.raises(ValueError):
        kvsnap.paged_restore(fresh, snap[:, :, :-1], FIX["mha_dst"])


def test_oracle_slot_snapshot_matches_reference() -> None:
    pool = torch.from_numpy(FIX["le_pool"].copy())
    snap = kvsnap.slot_backup(pool, LAYOUT, FIX["le_slot_map"], FIX["le_completed"], FIX["le_src"])
    assert snap.dtype == np.uint8 and np.array_equal(snap, FIX["le_snapshot"])
    row_bytes = 2 * 8 * 4
    n = len(FIX["le_src"])
    assert snap.size == kvsnap.slot_snapshot_bytes(LAYOUT, n, row_bytes)
    depths = kvsnap.slot_restore_depths(snap, LAYOUT, n, row_bytes)
    versions = LastExitedVersions(LAYOUT, 20)
    versions.reserve(FIX["le_dst"], restore_depths=depths)
    assert np.array_equal(versions.slot_map, FIX["le_restored_slot_map"])
    assert np.array_equal(versions.completed_depth, FIX["le_restored_completed"])
    assert versions.free_count == int(FIX["le_restored_free_count"][0])
    assert len(depths) * LAYOUT.loop_steps - int(depths.sum()) == int(FIX["le_released"])
    fresh = torch.zeros_like(pool)
    kvsnap.slot_restore(fresh, LAYOUT, versions.slot_map, snap, FIX["le_dst"])
    assert np.array_equal(fresh.numpy(), FIX["le_restored"])
    bad = snap.copy()
    bad[-4:] = np.array([9], np.int32).view(np.uint8)  # a depth beyond the loop
    with pytest.raises(ValueError):
        kvsnap.slot_restore_depths(bad, LAYOUT, n, row_bytes)


def test_snapshot_size_formula() -> None:
    sys.path.insert(0, str(ROOT))
    from __graft_entry__ import load_package

    load_package()
    from loop_sglang_b200 import ops

    # Ouro-1.4B: 24 layers, all recurrent, 4 steps, 16 KV heads x 128 bf16 rows
    assert ops.kv_snapshot_bytes(10, 4096, 24, 0, 24, 4, True) == 2 * 96 * 10 * 4096 + 40
    assert ops.kv_snapshot_bytes(10, 4096, 96) == 2 * 96 * 10 * 4096
    assert ops.kv_snapshot_bytes(0, 64, 6, 1, 5, 3, True) == 0
    assert kvsnap.slot_snapshot_bytes(LAYOUT, 5, 64) == ops.kv_snapshot_bytes(5, 64, 6, 1, 5, 3, True)
    with pytest.raises(ValueError):
        ops.kv_snapshot_bytes(1, 64, 6, 5, 1, 3, True)


# ------------------------------------------------------------------ GPU: CUDA path --

def _pkg():
    from __graft_entry__ import load_package

    load_package()
    from loop_sglang_b200 import kvcache, ops

    return kvcache, ops


@pytest.mark.gpu
def test_paged_snapshot_matches_reference_gpu() -> None:
    kvcache, ops = _pkg()
    dev = torch.device("cuda")
    pool = kvcache.MHAKVCache(2, 3, 8, 6, 4, dev, dtype=torch.float32)
    pool._kv_buffer.copy_(torch.from_numpy(FIX["mha_pool"]))
    src = torch.from_numpy(FIX["mha_src"]).to(dev)
    assert pool.cpu_copy_size(len(src)) == FIX["mha_snapshot"].nbytes
    snap = pool.get_cpu_copy(src)
    assert snap.is_pinned() and np.array_equal(snap.numpy(), FIX["mha_snapshot"])
    fresh = kvcache.MHAKVCache(2, 3, 8, 6, 4, dev, dtype=torch.float32)
    fresh.load_cpu_copy(snap, torch.from_numpy(FIX["mha_dst"]).to(dev))
    assert np.array_equal(fresh._kv_buffer.cpu().numpy(), FIX["mha_restored"])
    with pytest.raises(ValueError):
        fresh.load_cpu_copy(snap[:, :, :-1].contiguous(), torch.from_numpy(FIX["mha_dst"]).to(dev))
    assert ops.device_error_word(reset=True) == 0


@pytest.mark.gpu
def test_slot_snapshot_matches_reference_gpu() -> None:
    kvcache, ops = _pkg()
    dev = torch.device("cuda")

    def pool():
        return kvcache.LastExitedKVCache(2, 6, 8, 20, 1, 5, 3, dev, dtype=torch.float32)

    le = pool()
    le._kv_buffer.copy_(torch.from_numpy(FIX["le_pool"]))
    le.slot_map.copy_(torch.from_numpy(FIX["le_slot_map"]))
    le.completed_depth.copy_(torch.from_numpy(FIX["le_completed"]))
    src = torch.from_numpy(FIX["le_src"]).to(dev)
    snap = le.get_cpu_copy(src)
    assert snap.dtype == torch.uint8 and np.array_equal(snap.numpy(), FIX["le_snapshot"])
    fresh = pool()
    dst = torch.from_numpy(FIX["le_dst"]).to(dev)
    assert fresh.restore_slots(snap, len(dst)) == len(dst) * 1 + int(
        kvsnap.slot_restore_depths(snap.numpy(), LAYOUT, len(dst), 64).sum()) * 2
    assert fresh.reserve_restore_versions(dst, snap) == int(FIX["le_released"])
    fresh.load_cpu_copy(snap, dst)
    assert np.array_equal(fresh.slot_map.cpu().numpy(), FIX["le_restored_slot_map"])
    assert np.array_equal(fresh.completed_depth.cpu().numpy(), FIX["le_restored_completed"])
    assert np.array_equal(fresh._free_count.cpu().numpy(), FIX["le_restored_free_count"])
    assert np.array_equal(fresh._kv_buffer.cpu().numpy(), FIX["le_restored"])
    assert ops.device_error_word(reset=True) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("staging", [None, 3 * 2 * 96 * 4096 + 100])
def test_slot_snapshot_round_trip_ouro_rows(staging, monkeypatch) -> None:
    """Ouro-1.4B rows (24 recurrent layers, 4 loop steps, 16 KV heads x 128 bf16):
    snapshot 300 tokens that exited at mixed depths, restore them at other handles of
    a second pool; the bytes equal the oracle's and every restored version reads back
    the original rows. With a small staging buffer the copies run in 3-token chunks."""
    kvcache, ops = _pkg()
    if staging is not None:
        monkeypatch.setattr(ops, "KV_STAGING_BYTES", staging)
    dev = torch.device("cuda")
    layout = LastExitedLayout(num_layers=24, core_start=0, core_end=24, loop_steps=4)
    n, pages = 300, 1300  # 4 versions per token: 1200 of the 1299 slots
    g = torch.Generator().manual_seed(3)
    a = kvcache.LastExitedKVCache(16, 24, 128, pages, 0, 24, 4, dev)
    handles = torch.randperm(pages - 1, generator=g)[:n].add(1).to(torch.int32).to(dev)
    a.reserve_versions(handles)
    gd = torch.Generator(device=dev).manual_seed(3)
    a._kv_buffer.copy_(torch.randn(a._kv_buffer.shape, generator=gd, device=dev))
    a._kv_buffer[:, :, 0].zero_()
    exits = torch.randint(1, 5, (n,), generator=g, dtype=torch.int32).to(dev)
    a.alias_versions(handles, exits, int((4 - exits).sum()))
    snap = a.get_cpu_copy(handles)
    want = kvsnap.slot_backup(a._kv_buffer.cpu(), layout, a.slot_map.cpu().numpy(),
                              a.completed_depth.cpu().numpy(), handles.cpu().numpy())
    assert np.array_equal(snap.numpy(), want)
    b = kvcache.LastExitedKVCache(16, 24, 128, pages, 0, 24, 4, dev)
    dst = torch.randperm(pages - 1, generator=g)[:n].add(1).to(torch.int32).to(dev)
    b.reserve_restore_versions(dst, snap)
    b.load_cpu_copy(snap, dst)
    again = b.get_cpu_copy(dst)
    assert np.array_equal(again.numpy(), snap.numpy())
    assert np.array_equal(b.completed_depth[dst.long()].cpu().numpy(), exits.cpu().numpy())
    assert ops.device_error_word(reset=True) == 0


@pytest.mark.gpu
def test_paged_snapshot_round_trip_full_pool(monkeypatch) -> None:
    """A paged pool of 96 layers (Ouro-1.4B depth-indexed KV, 16-token pages): 300
    scattered tokens out and back into other locations, in 3 staging chunks."""
    kvcache, ops = _pkg()
    monkeypatch.setattr(ops, "KV_STAGING_BYTES", 100 * 2 * 96 * 4096)
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(4)
    pool = kvcache.MHAKVCache(16, 96, 128, 40, 16, dev)
    gd = torch.Generator(device=dev).manual_seed(4)
    pool._kv_buffer.copy_(torch.randn(pool._kv_buffer.shape, generator=gd, device=dev))
    pool._kv_buffer[:, :, 0].zero_()
    perm = torch.randperm(39 * 16, generator=g).add(16).to(torch.int32)
    src, dst = perm[:300].to(dev), perm[300:600].to(dev)
    snap = pool.get_cpu_copy(src)
    assert torch.equal(snap, kvsnap.paged_backup(pool._kv_buffer.cpu(), src.cpu().numpy()))
    pool.load_cpu_copy(snap, dst)
    assert torch.equal(pool.get_cpu_copy(dst), snap)
    assert ops.device_error_word(reset=True) == 0


@pytest.mark.gpu
def test_snapshot_out_of_range_handle_flagged() -> None:
    """A handle outside the slot map is skipped (zeros) and flagged, not read."""
    kvcache, ops = _pkg()
    dev = torch.device("cuda")
    le = kvcache.LastExitedKVCache(2, 6, 8, 20, 1, 5, 3, dev, dtype=torch.float32)
    ops.device_error_word(reset=True)
    snap = le.get_cpu_copy(torch.tensor([3, 25], dtype=torch.int32, device=dev))
    assert ops.device_error_word(reset=True) & 2  # LSB_DEVERR_SLOT
    assert snap.numel() == le.cpu_copy_size(2)
