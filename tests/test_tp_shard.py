"""Tensor-parallel weight sharding against the reference's own loader.

``tests/golden/tp_shard.npz`` holds a small unmerged checkpoint and, for every rank of
worlds 2 and 4, the tensors the reference's ``load_weight`` (models/weight.py:79-127,
shard rules :38-56) yields for it: q/k/v and gate/up merged, k/v replicated where there
are fewer KV heads than ranks, vocabulary ranges of ceil(V/t) rows. ``shard_weights``
must produce the same tensors bit for bit; its LM head carries zero rows beyond the
vocabulary so every rank's logits gather alike.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from __graft_entry__ import load_package  # noqa: E402

load_package()
from loop_sglang_b200.model import LoopedConfig, shard_weights  # noqa: E402

FIX = np.load(ROOT / "tests" / "golden" / "tp_shard.npz")
P = "model.layers.0"


def _config() -> LoopedConfig:
    return LoopedConfig(arch="ouro", hidden=int(FIX["hidden"]), heads=int(FIX["heads"]),
                        kv_heads=int(FIX["kv_heads"]), head_dim=int(FIX["head_dim"]),
                        intermediate=int(FIX["intermediate"]), vocab=int(FIX["vocab"]),
                        num_core_layers=1, attention_bias=True)


def _merged_inputs() -> dict[str, torch.Tensor]:
    raw = {k.split("::", 1)[1]: torch.from_numpy(FIX[k]) for k in FIX.files if k.startswith("in::")}
    out = {}
    for kind in ("weight", "bias"):
        out[f"{P}.self_attn.qkv_proj.{kind}"] = torch.cat(
            [raw.pop(f"{P}.self_attn.{x}_proj.{kind}") for x in "qkv"])
    out[f"{P}.mlp.gate_up_proj.weight"] = torch.cat(
        [raw.pop(f"{P}.mlp.gate_proj.weight"), raw.pop(f"{P}.mlp.up_proj.weight")])
    out.update(raw)
    return out


@pytest.mark.parametrize("world", [2, 4])
def test_shard_weights_match_reference_loader(world: int) -> None:
    cfg = _config()
    full = _merged_inputs()
    vocab_local = -(-cfg.vocab // world)
    for rank in range(world):
        got = shard_weights(cfg, full, rank, world)
        prefix = f"w{world}r{rank}::"
        want = {k[len(prefix):]: FIX[k] for k in FIX.files if k.startswith(prefix)}
        assert set(got) == set(want), (rank, set(got) ^ set(want))
        for name, ref in want.items():
            g = got[name].numpy()
            if name == "lm_head.weight":
                assert g.shape == (vocab_local, cfg.hidden)
                assert not g[len(ref):].any(), "LM head padding must be zero"
                g = g[: len(ref)]
            assert g.shape == ref.shape and np.array_equal(g, ref), (world, rank, name)


def test_shard_weights_single_rank_is_identity() -> None:
    full = _merged_inputs()
    got = shard_weights(_config(), full, 0, 1)
    assert set(got) == set(full) and all(got[k] is full[k] for k in full)
