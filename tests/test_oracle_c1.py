"""BASELINE configs[0] (the tiny Ouro model the reference runs on the CPU) through the
oracle, against the reference's own fp32 run recorded in ``tests/golden/c1_ouro_tiny.npz``.

4 requests with 128-token prompts, one prefill and 32 full-depth greedy decode steps over
depth-indexed KV in 16-token pages. Every step is replayed with the reference's recorded
batch metadata and input ids (teacher forcing, so a near-tie cannot cascade): the greedy
token must match wherever the reference's top-2 margin leaves room for fp32 reordering, and
the logits of the prefill and of the last step must match to fp32 precision.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))

from oracle.model import LoopedConfig, LoopedModel, PagedKVPool, make_weights  # noqa: E402
from replay import batch_from, load  # noqa: E402

C1 = LoopedConfig(arch="ouro", hidden=512, heads=8, kv_heads=8, head_dim=64, intermediate=1408,
                  vocab=32000, num_core_layers=4, loop_steps=4, rope_theta=10000.0,
                  max_position=512)


def test_c1_oracle_matches_reference_run() -> None:
    torch.set_num_threads(4)
    fx = load("c1_ouro_tiny")
    model = LoopedModel(C1, make_weights(C1, int(fx["seed"]), dtype=torch.float32),
                        "depth_indexed")
    pool = PagedKVPool(model.num_kv_layers, 64, int(fx["page_size"]), C1.kv_heads, C1.head_dim,
                       torch.float32)
    tokens, margins = fx["tokens"], fx["margins"]
    steps = [("prefill", True)] + [(f"step{k}", False) for k in range(len(tokens) - 1)]
    checked = 0
    for i, (prefix, prefill) in enumerate(steps):
        logits = model.forward(batch_from(fx, prefix, fx[f"{prefix}_ids"], prefill), pool).float()
        if prefix == "prefill":
            torch.testing.assert_close(logits, torch.from_numpy(fx["prefill_logits"]),
                                       rtol=1e-4, atol=1e-5)
        if i == len(steps) - 1:
            torch.testing.assert_close(logits, torch.from_numpy(fx["last_logits"]),
                                       rtol=1e-4, atol=1e-5)
        got = logits.argmax(-1).numpy()
        clear = margins[i] > 1e-4
        assert np.array_equal(got[clear], tokens[i][clear]), (prefix, got, tokens[i])
        checked += int(clear.sum())
    assert checked >= 0.95 * tokens.size  # near-ties are rare at this scale
