"""The oracle reproduces the golden vectors produced by the reference's own code.

Integer outputs (page tables, batch inputs, last-exited version maps, exit
signals) must match exactly; fp32 model outputs to 1e-5 (the reference run and
the oracle differ only in summation order).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import kvmeta, ops
from replay import CB_CASES, CDB_CASES, load, replay_cb, replay_cdb


def test_metadata_golden() -> None:
    fx = load("metadata")
    table = np.zeros_like(fx["assign_table"])
    kvmeta.assign_req_to_token_pool(fx["assign_rpi"], table, fx["assign_start"],
                                    fx["assign_end"], fx["assign_out"])
    np.testing.assert_array_equal(table, fx["assign_table"])
    page = 4
    for tag, is_decode in (("decode", True), ("extend", False)):
        maxp = (int(fx["seq"].max()) + page - 1) // page
        pt = np.full_like(fx[f"{tag}_pt"], -1)
        cache, cuk, cuq, pt = kvmeta.set_metadata(fx["seq"], fx["ext"], fx["r2t"], fx["rpi"], maxp,
                                                  page, is_decode, page_table=pt)
        np.testing.assert_array_equal(cache, fx[f"{tag}_cache"])
        np.testing.assert_array_equal(cuk, fx[f"{tag}_cuk"])
        np.testing.assert_array_equal(cuq, fx[f"{tag}_cuq"])
        np.testing.assert_array_equal(pt, fx[f"{tag}_pt"])
        ext = np.ones(3, np.int32) if is_decode else fx["ext"]
        pos, mapping, out_loc = kvmeta.prepare_batch_inputs(fx["seq"], ext, fx["rpi"], fx["r2t"],
                                                             is_decode)
        np.testing.assert_array_equal(pos, fx[f"{tag}_positions"])
        np.testing.assert_array_equal(mapping, fx[f"{tag}_mapping"])
        np.testing.assert_array_equal(out_loc, fx[f"{tag}_outloc"])


def test_store_golden() -> None:
    fx = load("store")
    kc = torch.full((17, 2, 8), -7.0)
    vc = torch.full((17, 2, 8), -7.0)
    ops.store_kv(kc, vc, torch.from_numpy(fx["idx"]), torch.from_numpy(fx["k"]),
                 torch.from_numpy(fx["v"]))
    np.testing.assert_array_equal(kc.numpy(), fx["k_cache"])
    np.testing.assert_array_equal(vc.numpy(), fx["v_cache"])


@pytest.mark.parametrize("name", ["last_exited_huginn_layout", "last_exited_ouro_layout"])
def test_last_exited_golden(name: str) -> None:
    fx = load(name)
    num_layers, core_start, core_end, steps, num_pages = (int(v) for v in fx["layout"])
    lay = kvmeta.LastExitedLayout(num_layers, core_start, core_end, steps)
    ver = kvmeta.LastExitedVersions(lay, num_pages)

    def check(tag: str) -> None:
        np.testing.assert_array_equal(ver.slot_map, fx[f"{tag}_slot_map"])
        np.testing.assert_array_equal(ver.completed_depth, fx[f"{tag}_completed"])
        np.testing.assert_array_equal(ver.free_slots, fx[f"{tag}_free"])
        assert ver.free_count == int(fx[f"{tag}_count"][0])

    ver.reserve(np.array([3, 5, 1, 7]))
    check("op0")
    ver.release(fx["op1_handles"], fx["op1_exits"])
    check("op1")
    ver.reserve(fx["op2_handles"])
    check("op2")
    ver.release(fx["op3_handles"])
    check("op3")
    ver.reserve(fx["op4_handles"], fx["op4_depths"])
    check("op4")
    for tag in ("vec", "scalar"):
        depths = fx[f"resolve_{tag}_depths"]
        depths = int(depths) if depths.ndim == 0 else depths
        groups = lay.core_groups
        table = np.full((groups, 3, 4), -1, np.int32)
        out = np.full((groups, 4), -1, np.int32)
        kvmeta.resolve_last_exited(fx["resolve_logical"], ver.version_map, fx["resolve_seq"],
                                   fx["resolve_cu"], fx["resolve_lout"], depths, table, out)
        np.testing.assert_array_equal(table, fx[f"resolve_{tag}_table"])
        np.testing.assert_array_equal(out, fx[f"resolve_{tag}_out"])
    if "resolve_fixed_table" in fx:
        table = np.full((lay.fixed_groups, 3, 4), -1, np.int32)
        out = np.full((lay.fixed_groups, 4), -1, np.int32)
        kvmeta.resolve_last_exited(fx["resolve_logical"], ver.fixed_map, fx["resolve_seq"],
                                   fx["resolve_cu"], fx["resolve_lout"], 0, table, out)
        np.testing.assert_array_equal(table, fx["resolve_fixed_table"])
        np.testing.assert_array_equal(out, fx["resolve_fixed_out"])


@pytest.mark.parametrize("name", sorted(CB_CASES))
def test_cb_model_golden(name: str) -> None:
    fx, out, pool = replay_cb(name)
    for prefix, logits in out.items():
        np.testing.assert_allclose(logits.numpy(), fx[f"{prefix}_logits"], rtol=1e-5, atol=1e-5)
    kv = pool.buf.double().sum(dim=tuple(range(2, pool.buf.ndim))).numpy()
    np.testing.assert_allclose(kv, fx["kv_checksum"], rtol=1e-6, atol=1e-4)
    if "slot_map" in fx:
        np.testing.assert_array_equal(pool.versions.slot_map, fx["slot_map"])


@pytest.mark.parametrize("name", sorted(CDB_CASES))
def test_cdb_golden(name: str) -> None:
    fx, res = replay_cdb(name)
    np.testing.assert_allclose(res["prefill_logits"].numpy(), fx["prefill_logits"], rtol=1e-5,
                               atol=1e-5)
    np.testing.assert_allclose(res["prelude_hidden"].numpy(), fx["prelude_hidden"], rtol=1e-5,
                               atol=1e-6)
    k = 0
    while f"core{k}_rows" in fx:
        np.testing.assert_array_equal(res[f"core{k}_gates"].numpy(), fx[f"core{k}_gates"])
        np.testing.assert_allclose(res[f"core{k}_hidden"].numpy(), fx[f"core{k}_hidden"],
                                   rtol=1e-4, atol=1e-5)
        np.testing.assert_allclose(res[f"core{k}_exit"].numpy(), fx[f"core{k}_exit"], rtol=1e-5,
                                   atol=1e-6)
        if f"core{k}_core_page_table" in fx:
            n = fx[f"core{k}_core_page_table"].shape
            got = res[f"core{k}_core_page_table"].numpy()
            seq = fx[f"core{k}_cache_seqlens"]
            for r in range(n[1]):
                np.testing.assert_array_equal(got[:, r, : seq[r]],
                                              fx[f"core{k}_core_page_table"][:, r, : seq[r]])
            np.testing.assert_array_equal(res[f"core{k}_core_out_loc"].numpy(),
                                          fx[f"core{k}_core_out_loc"])
        k += 1
    assert k == 4
    np.testing.assert_allclose(res["coda_logits"].numpy(), fx["coda_logits"], rtol=1e-5,
                               atol=1e-5)
    kv = res["kv_buf"].double().sum(dim=tuple(range(2, res["kv_buf"].ndim))).numpy()
    np.testing.assert_allclose(kv, fx["kv_checksum"], rtol=1e-6, atol=1e-4)
