"""Record the oracle's outputs for the full-size (Ouro-1.4B) parity scenarios.

Usage (CPU, a few minutes)::

    python tests/golden/make_fullsize.py

Runs ``oracle/`` only (itself pinned to the reference by ``make_golden.py``'s fixtures,
including the reference's fp32 run of BASELINE configs[0]) on the scenarios of
``tests/scale_scenarios.py`` and writes ``tests/golden/ouro14b_fullsize.npz``:

* CB: for the prefill and 4 greedy decode steps, the oracle in bf16 (the reference's
  rounding points) -- logits on every 24th vocabulary column, the top 8 logits and
  the LM-head input rows -- and the same for the oracle in fp32 on the same
  (bf16-valued) weights and inputs: how far bf16 arithmetic itself lands from exact
  arithmetic after 96 layer passes, the floor any bf16 implementation is held to.
* CDB: the lock-step restatement of the device-routed engine (``tests/cdb_lockstep.py``)
  in bf16: every output's token, top 8 logits and hidden row, its exit depth, and the
  final version map, completed depths and free-slot stack of the last-exited pool; and
  the hidden rows of the same run in fp32.

The GPU test rebuilds the same weights and inputs from the seeds, so only outputs
are stored.
"""

from __future__ import annotations

import sys
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, str(HERE.parent))

import scale_scenarios as S  # noqa: E402
from cdb_lockstep import make_scenario, oracle_run  # noqa: E402
from oracle.model import LoopedModel, PagedKVPool, with_fp32_matrices  # noqa: E402

OUT = HERE / "ouro14b_fullsize.npz"


def run_cb(dtype: torch.dtype, decode_ids: torch.Tensor | None):
    """Prefill + CB_DECODE decode steps; returns per-step (hidden rows, logits) and the ids
    fed to the decode steps (the run's own greedy tokens unless ``decode_ids`` is given)."""
    w = S.weights()
    w = {k: v.float() for k, v in w.items()} if dtype == torch.float32 else with_fp32_matrices(w)
    model = LoopedModel(S.OURO_14B, w, "depth_indexed")
    table, num_pages = S.cb_pages()
    c = S.OURO_14B
    pool = PagedKVPool(model.num_kv_layers, num_pages, S.PAGE, c.kv_heads, c.head_dim, dtype)
    hiddens, logits_all, fed = [], [], []
    ids = None
    for step in range(-1, S.CB_DECODE):
        if step >= 0:
            ids = decode_ids[step] if decode_ids is not None else ids
            fed.append(ids.clone())
        b = S.cb_batch(step, ids, table)
        h, inj = model.forward_prelude(b, pool)
        for s in range(c.loop_steps):
            h = model.core_step(h, s, inj, b, pool)
        h = model.forward_coda(h, b, pool)
        rows = h[b.last_indices()] if b.is_prefill else h
        lg = model.lm_head(rows, None).float()
        hiddens.append(rows.clone())
        logits_all.append(lg)
        ids = lg.argmax(-1).to(torch.int32)
        print(f"  cb {dtype} step {step}: done", flush=True)
    return hiddens, logits_all, torch.stack(fed) if fed else None


def main() -> None:
    torch.set_num_threads(max(1, torch.get_num_threads()))
    t0 = time.time()
    S.weights()
    print(f"weights {time.time() - t0:.0f}s", flush=True)
    out: dict[str, np.ndarray] = {"seed": np.int64(S.SEED)}
    if "--cdb-only" in sys.argv:  # keep the recorded CB part, redo the CDB part
        with np.load(OUT) as f:
            out.update({k: f[k] for k in f.files if not k.startswith("cdb_")})
    else:
        run_cb_part(out, t0)
    run_cdb_part(out, t0)
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


def run_cb_part(out: dict, t0: float) -> None:
    cols = S.probe_columns(S.OURO_14B.vocab)
    hid, lg, fed = run_cb(torch.bfloat16, None)
    out["cb_decode_ids"] = fed.numpy()
    out["cb_bf16_hidden"] = np.stack([S.bf16_bits(h) for h in hid])
    out["cb_bf16_probe"] = torch.stack([x[:, cols] for x in lg]).numpy()
    top = [x.topk(S.TOPK, dim=-1) for x in lg]
    out["cb_bf16_top_v"] = torch.stack([t.values for t in top]).numpy()
    out["cb_bf16_top_i"] = torch.stack([t.indices for t in top]).to(torch.int32).numpy()
    out["cb_bf16_scale"] = torch.stack([x.abs().max(-1).values for x in lg]).numpy()
    print(f"cb bf16 {time.time() - t0:.0f}s", flush=True)

    hid32, lg32, _ = run_cb(torch.float32, fed)
    out["cb_fp32_hidden"] = torch.stack(hid32).numpy()
    out["cb_fp32_probe"] = torch.stack([x[:, cols] for x in lg32]).numpy()
    top = [x.topk(S.TOPK, dim=-1) for x in lg32]
    out["cb_fp32_top_v"] = torch.stack([t.values for t in top]).numpy()
    out["cb_fp32_top_i"] = torch.stack([t.indices for t in top]).to(torch.int32).numpy()
    out["cb_fp32_scale"] = torch.stack([x.abs().max(-1).values for x in lg32]).numpy()
    print(f"cb fp32 {time.time() - t0:.0f}s", flush=True)


def run_cdb_part(out: dict, t0: float) -> None:
    sc = make_scenario(S.OURO_14B_GATED, S.SEED, S.CDB_PROMPTS, S.CDB_K, S.CDB_MAX_LEN,
                       S.CDB_DEPTH_P)
    ref = oracle_run(S.OURO_14B_GATED, S.weights(), sc)
    b, k = len(sc.prompts), sc.k
    out["cdb_preds"] = np.array(ref["preds"], dtype=np.int32)
    out["cdb_depths"] = np.array(ref["depths"], dtype=np.int32)
    out["cdb_top_v"] = np.stack([[ref["topk"][r][j][0].numpy() for j in range(k)]
                                 for r in range(b)])
    out["cdb_top_i"] = np.stack([[ref["topk"][r][j][1].numpy() for j in range(k)]
                                 for r in range(b)])
    out["cdb_scale"] = np.array([[ref["topk"][r][j][2] for j in range(k)] for r in range(b)],
                                dtype=np.float32)
    out["cdb_hidden"] = np.stack([S.bf16_bits(torch.stack(ref["hidden"][r])) for r in range(b)])
    ref32 = oracle_run(S.OURO_14B_GATED, S.weights(), sc, dtype=torch.float32)
    out["cdb_fp32_hidden"] = np.stack([torch.stack(ref32["hidden"][r]).numpy() for r in range(b)])
    v = ref["pool"].versions
    out["cdb_slot_map"] = np.asarray(v.slot_map, dtype=np.int32)
    out["cdb_completed_depth"] = np.asarray(v.completed_depth, dtype=np.int32)
    out["cdb_free_count"] = np.int64(v.free_count)
    out["cdb_free_slots"] = np.asarray(v.free_slots[: v.free_count], dtype=np.int32)
    print(f"cdb {time.time() - t0:.0f}s", flush=True)


if __name__ == "__main__":
    main()
