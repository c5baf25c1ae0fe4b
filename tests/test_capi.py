"""The C-ABI library loads without a GPU and exports every entry point the header declares.

No compute call is made here (there is no device); argument validation that fails
before any CUDA call is checked, since it is pure host logic.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from __graft_entry__ import ROOT, load_package

HEADER = ROOT / "include" / "loopsgl_b200.h"


def declared() -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(lsb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points() -> None:
    names = declared()
    assert "lsb_gemm" in names and "lsb_paged_attention" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol() -> None:
    pkg = load_package()
    lib = pkg._lib.lib()
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"
    bound = set(pkg._lib.SIGNATURES)
    assert set(declared()) <= bound, f"no ctypes signature for {set(declared()) - bound}"
    assert lib.lsb_abi_version() >= 1


def test_argument_validation_without_device() -> None:
    """Shape checks reject bad calls before touching CUDA and leave a message."""
    pkg = load_package()
    lib = pkg._lib.lib()
    rc = lib.lsb_gemm(ctypes.c_void_p(16), 128, ctypes.c_void_p(16), 100, ctypes.c_void_p(16),
                      100, None, 4, 128, 100, 0, None, 0, None)
    assert rc == pkg._lib.LSB_ERR_INVALID
    assert b"K" in lib.lsb_last_error()
    rc = lib.lsb_rmsnorm(ctypes.c_void_p(16), 12, ctypes.c_void_p(16), 12, ctypes.c_void_p(16), 2,
                         12, ctypes.c_float(1e-6), None)
    assert rc == pkg._lib.LSB_ERR_INVALID
    # out, out_stride, q, q_stride, k, v, slot_stride, num_slots, table, pt_stride, seqlens,
    # cu_q, num_reqs, rows, hq, hkv, head_dim (80: unsupported), page, max_seq, scale, ws...
    p = ctypes.c_void_p(16)
    rc = lib.lsb_paged_attention(p, 8, p, 8, p, p, 8, 1, p, 1, p, p, 1, 1, 1, 1, 80, 16, 16,
                                 ctypes.c_float(1.0), None, 0, None)
    assert rc == pkg._lib.LSB_ERR_INVALID
    with pytest.raises(ValueError):
        pkg._lib.check(pkg._lib.LSB_ERR_INVALID, "x")


def test_workspace_size_queries_are_host_only() -> None:
    lib = load_package()._lib.lib()
    # split-K partials are reduced in distributed shared memory: no workspace
    assert lib.lsb_gemm_workspace_size(144, 6144, 2048) == 0
    assert lib.lsb_paged_attention_workspace_size(144, 16, 128, 2304) > 0


def test_launch_count_ignores_rejected_calls() -> None:
    """The library counts only launches that happened: calls rejected by validation (no
    device needed) leave the count where it was."""
    pkg = load_package()
    lib = pkg._lib.lib()
    before = pkg._lib.launch_count()
    p = ctypes.c_void_p(16)
    for _ in range(3):
        rc = lib.lsb_paged_attention(p, 8, p, 8, p, p, 8, 1, p, 1, p, p, 1, 1, 1, 1, 80, 16, 16,
                                     ctypes.c_float(1.0), None, 0, None)
        assert rc == pkg._lib.LSB_ERR_INVALID
    assert pkg._lib.launch_count() == before



def test_attention_plan_is_host_only() -> None:
    """The decode attention plan (kernel, item size, stages, producer issue mode) is pure
    host logic: 16 KV heads of 128 stream 8 keys per 64 KB stage from one producer lane;
    a TP=8 rank's 2 heads stream 64 keys (four 16-token pages) one page run per lane, but
    not on 64-token pages; Huginn's 55 x 96 heads and scattered 1 KB rows take the per-CTA
    kernel."""
    from loop_sglang_b200 import ops

    load_package()
    p = ops.attention_plan(143, 16, 16, 128, 16, 1448)
    assert p["kernel"] == "streaming" and p["keys_per_stage"] == 8 and p["stages"] == 3
    assert not p["lane_per_page"] and p["keys_per_item"] * p["splits"] >= 1448
    p = ops.attention_plan(256, 2, 2, 128, 16, 2112)
    assert p["kernel"] == "streaming" and p["keys_per_stage"] == 64 and p["lane_per_page"]
    assert p["keys_per_item"] >= 512  # at least 512 KB of K+V per item with few heads
    assert not ops.attention_plan(256, 2, 2, 128, 64, 2112)["lane_per_page"]
    assert ops.attention_plan(64, 55, 55, 96, 16, 1033)["kernel"] == "per_cta"
    assert ops.attention_plan(512, 4, 4, 128, 1, 900)["kernel"] == "per_cta"
    assert ops.attention_plan(512, 16, 16, 128, 1, 900)["kernel"] == "streaming"
    with pytest.raises(ValueError):
        ops.attention_plan(4, 16, 16, 80, 16, 64)
