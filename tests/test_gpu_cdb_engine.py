"""Device-routed continuous-depth batching against a lock-step oracle restatement.

Three requests of different prompt lengths are prefilled (last-exited KV), then the
CDB engine runs core steps until every row has produced K outputs. Inputs are
teacher-forced and exit depths prescribed (the reference's replay depths), so the
oracle takes the same route: per step every row runs one loop step at its own
depth (``oracle.cdb.core_phase``), exiting rows are sampled, their KV versions
aliased at the exit depth and the successors' versions reserved, in row order.
Checked: every predicted token (greedy, near-tie aware), every exit depth, and the
version maps, completed depths and free-slot stack bit-exactly; a gated run (no
replay) checks the gate decisions the device takes on its own.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from cdb_lockstep import gpu_run, make_scenario, oracle_run, token_matches
from oracle.model import make_weights
from replay import OURO_TINY_GATED, gpu_model

pytestmark = pytest.mark.gpu

PROMPTS = [5, 9, 3]
K = 6  # outputs compared per row
MAX_LEN = 40


def _setup(seed: int):
    cfg = OURO_TINY_GATED
    weights = make_weights(cfg, seed, dtype=torch.float32, gate_bias=0.3)
    return cfg, weights, make_scenario(cfg, seed, PROMPTS, K, MAX_LEN)


def check_versions(kv, pool) -> None:
    """Version maps, completed depths and the free-slot stack, bit for bit."""
    v = pool.versions
    assert np.array_equal(kv.slot_map.cpu().numpy(), v.slot_map)
    assert np.array_equal(kv.completed_depth.cpu().numpy(), v.completed_depth)
    assert int(kv._free_count.item()) == v.free_count
    n = v.free_count
    assert np.array_equal(kv._free_slots.cpu().numpy()[:n], v.free_slots[:n])


@pytest.mark.parametrize("graph", [False, True])
def test_cdb_engine_replay_matches_oracle(graph: bool) -> None:
    cfg, weights, sc = _setup(21)
    ref = oracle_run(cfg, weights, sc)
    eng, kv = gpu_run(gpu_model(cfg, weights, "last_exited"), sc, graph=graph)
    count = eng.out_count.cpu()
    toks, deps = eng.out_tokens.cpu(), eng.out_depths.cpu()
    for r in range(len(sc.prompts)):
        assert int(count[r]) >= K and len(ref["preds"][r]) == K, (r, int(count[r]))
        assert deps[r, :K].tolist() == ref["depths"][r] == sc.replay[r].tolist(), r
        for k in range(K):
            verdict = token_matches(int(toks[r, k]), ref["preds"][r][k], ref["topk"][r][k])
            assert verdict != "mismatch", (r, k, int(toks[r, k]), ref["preds"][r][k])
    check_versions(kv, ref["pool"])
    from loop_sglang_b200 import ops  # imported by gpu_model above

    assert ops.device_error_word(reset=True) == 0


def test_cdb_engine_gates_match_oracle() -> None:
    """Without prescribed depths the device routes on its own gate: the first step's
    signals (and exit probabilities) match the oracle's where the decision is clear."""
    cfg, weights, sc = _setup(33)
    ref = oracle_run(cfg, weights, sc, use_replay=False, steps=1)
    eng, _ = gpu_run(gpu_model(cfg, weights, "last_exited"), sc, use_replay=False, steps=1)
    want_sig, want_p, _ = ref["gates"][0]
    got_p = eng.state["exit"][eng.slots].float().cpu()
    exited = eng.exited.bool().cpu()
    # an exited row's exit state was reset by the successor's admission
    keep = ~exited
    assert torch.allclose(got_p[keep], want_p[keep], atol=2e-2)
    sure = (want_p - cfg.exit_threshold).abs() > 1e-3
    assert torch.equal(exited[sure], want_sig[sure] | torch.zeros_like(want_sig[sure]))
