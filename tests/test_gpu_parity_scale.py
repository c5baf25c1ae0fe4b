"""Parity at BASELINE scale: configs[0] end to end, and the Ouro-1.4B architecture at full
size, through the CUDA path.

* configs[0] (the tiny Ouro model the reference runs on the CPU: 4 x 128-token prompts,
  32 greedy decode steps, depth-indexed KV in 16-token pages) in bf16, teacher-forced with
  the reference's own recorded inputs (``tests/golden/c1_ouro_tiny.npz``): logits within
  rel 2e-2 of the oracle in bf16 at every step; every greedy token equal to the bf16
  oracle's unless the two top logits are within that tolerance (a near tie, counted
  apart); greedy agreement with the reference's fp32 run at least that of the bf16
  oracle itself (the part bf16 arithmetic alone costs) less two tokens.
* Ouro-1.4B CB (configs[1] shapes): a real prefill of 4 requests with prompts of
  256-1024 tokens, then 4 greedy decode steps; LM-head rows and logits within 2e-2 of the
  bf16 oracle (``tests/golden/ouro14b_fullsize.npz``, made by
  ``tests/golden/make_fullsize.py``), tokens equal up to near ties.
* Ouro-1.4B CDB (configs[2] shapes, last-exited KV): the device-routed engine after a
  real prefill, exit depths prescribed from the 15/25/30/30% mix: tokens (near-tie
  aware) and the hidden row of every output against the lock-step oracle; exit depths,
  version maps, completed depths and the free-slot stack bit-exact.
"""

from __future__ import annotations

import gc

import numpy as np
import pytest
import torch

import scale_scenarios as S
from cdb_lockstep import gpu_run, make_scenario, token_matches
from oracle.model import LoopedConfig, LoopedModel, PagedKVPool, make_weights, with_fp32_matrices
from replay import device_batch, gpu_model, load

pytestmark = pytest.mark.gpu

REL = 2e-2
C1 = LoopedConfig(arch="ouro", hidden=512, heads=8, kv_heads=8, head_dim=64, intermediate=1408,
                  vocab=32000, num_core_layers=4, loop_steps=4, rope_theta=10000.0,
                  max_position=512)


def rel_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    ref = ref.float()
    return float((got.float() - ref).abs().max() / ref.abs().max().clamp_min(1e-6))


def verdict_full(got: torch.Tensor, ref: torch.Tensor) -> list[str]:
    """Per row: 'agree', 'near_tie' or 'mismatch' of the greedy token against full logits."""
    g, r = got.float().argmax(-1), ref.float().argmax(-1)
    scale = ref.float().abs().max(-1).values
    out = []
    for i in range(got.shape[0]):
        if int(g[i]) == int(r[i]):
            out.append("agree")
        elif ref[i, g[i]] >= ref[i, r[i]] - REL * scale[i]:
            out.append("near_tie")
        else:
            out.append("mismatch")
    return out


def _free() -> None:
    gc.collect()
    torch.cuda.empty_cache()


def test_configs0_greedy_agreement() -> None:
    fx = load("c1_ouro_tiny")
    seed = int(fx["seed"])
    page = int(fx["page_size"])
    model = gpu_model(C1, make_weights(C1, seed, dtype=torch.float32), "depth_indexed")
    kv = model.make_kv_cache(64, page)
    oracle = LoopedModel(C1, with_fp32_matrices(make_weights(C1, seed, dtype=torch.bfloat16)),
                         "depth_indexed")
    pool = PagedKVPool(oracle.num_kv_layers, 64, page, C1.kv_heads, C1.head_dim, torch.bfloat16)
    from replay import batch_from

    tokens = fx["tokens"]
    steps = [("prefill", True)] + [(f"step{k}", False) for k in range(len(tokens) - 1)]
    counts = {"agree": 0, "near_tie": 0, "mismatch": 0}
    gpu_fp32, oracle_fp32, worst = 0, 0, 0.0
    for i, (prefix, prefill) in enumerate(steps):
        ids = fx[f"{prefix}_ids"]
        got = model.forward(device_batch(fx, prefix, ids, prefill, page), kv).float().cpu()
        ref = oracle.forward(batch_from(fx, prefix, ids, prefill), pool).float()
        worst = max(worst, rel_err(got, ref))
        for v in verdict_full(got, ref):
            counts[v] += 1
        gpu_fp32 += int((got.argmax(-1).numpy() == tokens[i]).sum())
        oracle_fp32 += int((ref.argmax(-1).numpy() == tokens[i]).sum())
    total = tokens.size
    summary = (f"configs[0]: {total} greedy tokens; vs bf16 oracle {counts}; "
               f"vs the reference's fp32 run: CUDA {gpu_fp32}, bf16 oracle {oracle_fp32}; "
               f"max logit rel err {worst:.4f}")
    print(summary)
    assert worst < REL, summary
    assert counts["mismatch"] == 0, summary
    assert counts["agree"] >= 0.97 * total, summary
    assert gpu_fp32 >= oracle_fp32 - 2, summary


@pytest.fixture(scope="module")
def fullsize() -> dict:
    return load("ouro14b_fullsize")


def test_ouro14b_cb_prefill_decode_matches_oracle(fullsize) -> None:
    from loop_sglang_b200 import ops
    from loop_sglang_b200.model import DeviceBatch

    fx = fullsize
    model = gpu_model(S.OURO_14B, S.weights(), "depth_indexed")
    table, num_pages = S.cb_pages()
    kv = model.make_kv_cache(num_pages, S.PAGE)
    dev = model.device
    counts = {"agree": 0, "near_tie": 0, "mismatch": 0}
    fp32_agree, worst_logits, worst_hidden = 0, 0.0, 0.0
    for i, step in enumerate(range(-1, S.CB_DECODE)):
        ids = torch.from_numpy(fx["cb_decode_ids"][step]) if step >= 0 else None
        b = S.cb_batch(step, ids, table)
        db = DeviceBatch(b.input_ids.to(dev), b.positions.to(dev), b.out_loc.to(dev),
                         b.page_table.to(dev).contiguous(), b.cache_seqlens.to(dev),
                         b.cu_seqlens_q.to(dev), b.is_prefill,
                         max_seqlen=int(table.shape[1]) * S.PAGE)
        h, inj = model.forward_prelude(db, kv)
        for s in range(S.OURO_14B.loop_steps):
            h = model.core_step(h, s, inj, db, kv)
        rows = model._lm_rows(model.forward_coda(h, db, kv), db)
        logits = ops.gemm(rows, model.lm_head_w).float().cpu()
        want_h = S.from_bf16_bits(fx["cb_bf16_hidden"][i])
        worst_hidden = max(worst_hidden, rel_err(rows.cpu(), want_h))
        rel, verdicts = S.logits_match(
            logits, torch.from_numpy(fx["cb_bf16_probe"][i]), torch.from_numpy(fx["cb_bf16_top_v"][i]),
            torch.from_numpy(fx["cb_bf16_top_i"][i]), torch.from_numpy(fx["cb_bf16_scale"][i]))
        worst_logits = max(worst_logits, rel)
        for v in verdicts:
            counts[v] += 1
        fp32_agree += int((logits.argmax(-1).numpy() == fx["cb_fp32_top_i"][i][:, 0]).sum())
    summary = (f"Ouro-1.4B CB: prefill + {S.CB_DECODE} decode steps x {len(S.CB_PROMPTS)} rows; "
               f"vs bf16 oracle {counts}; vs fp32 oracle {fp32_agree}; rel err logits "
               f"{worst_logits:.4f}, hidden {worst_hidden:.4f}")
    print(summary)
    assert worst_logits < REL and worst_hidden < REL, summary
    assert counts["mismatch"] == 0, summary
    assert ops.device_error_word(reset=True) == 0
    del model, kv
    _free()


def test_ouro14b_cdb_engine_matches_oracle(fullsize) -> None:
    from loop_sglang_b200 import ops

    fx = fullsize
    sc = make_scenario(S.OURO_14B_GATED, S.SEED, S.CDB_PROMPTS, S.CDB_K, S.CDB_MAX_LEN,
                       S.CDB_DEPTH_P)
    model = gpu_model(S.OURO_14B_GATED, S.weights(), "last_exited")
    got_hidden: dict[tuple[int, int], torch.Tensor] = {}

    def record(eng) -> None:
        exited = eng.exited.cpu().bool()
        count = eng.out_count.cpu()
        for r in torch.nonzero(exited).flatten().tolist():
            k = int(count[r]) - 1
            if k < sc.k:
                got_hidden[(r, k)] = eng.hidden_rows[r].cpu()

    eng, kv = gpu_run(model, sc, on_step=record)
    toks, deps = eng.out_tokens.cpu(), eng.out_depths.cpu()
    b, k_out = len(sc.prompts), sc.k
    counts = {"agree": 0, "near_tie": 0, "mismatch": 0}
    worst = 0.0
    for r in range(b):
        assert deps[r, :k_out].tolist() == fx["cdb_depths"][r].tolist() == sc.replay[r].tolist()
        for k in range(k_out):
            topk = (torch.from_numpy(fx["cdb_top_v"][r, k]), torch.from_numpy(fx["cdb_top_i"][r, k]),
                    float(fx["cdb_scale"][r, k]))
            counts[token_matches(int(toks[r, k]), int(fx["cdb_preds"][r, k]), topk)] += 1
            want = S.from_bf16_bits(fx["cdb_hidden"][r, k])
            worst = max(worst, rel_err(got_hidden[(r, k)], want))
    summary = f"Ouro-1.4B CDB: {b} rows x {k_out} outputs vs the oracle {counts}; hidden {worst:.4f}"
    print(summary)
    assert counts["mismatch"] == 0, summary
    assert worst < REL, summary
    assert np.array_equal(kv.slot_map.cpu().numpy(), fx["cdb_slot_map"])
    assert np.array_equal(kv.completed_depth.cpu().numpy(), fx["cdb_completed_depth"])
    n = int(fx["cdb_free_count"])
    assert int(kv._free_count.item()) == n
    assert np.array_equal(kv._free_slots.cpu().numpy()[:n], fx["cdb_free_slots"])
    assert ops.device_error_word(reset=True) == 0
    del model, kv, eng
    _free()
