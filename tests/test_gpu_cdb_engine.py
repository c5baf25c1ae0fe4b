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

from oracle import cdb as ocdb
from oracle import ops as O
from oracle.model import Batch, LoopedModel, SlotKVPool, make_weights
from replay import OURO_TINY_GATED, gpu_model

pytestmark = pytest.mark.gpu

PROMPTS = [5, 9, 3]
K = 6  # outputs compared per row
MAX_LEN = 40


def _setup(seed: int):
    cfg = OURO_TINY_GATED
    weights = make_weights(cfg, seed, dtype=torch.float32, gate_bias=0.3)
    g = torch.Generator().manual_seed(seed + 1)
    b = len(PROMPTS)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g, dtype=torch.int32) for n in PROMPTS]
    first = torch.randint(0, cfg.vocab, (b,), generator=g, dtype=torch.int32)
    forced = torch.randint(0, cfg.vocab, (b, K), generator=g, dtype=torch.int32)
    replay = torch.randint(1, cfg.loop_steps + 1, (b, K), generator=g, dtype=torch.int32)
    handles = (1 + torch.arange(b).view(-1, 1) * MAX_LEN + torch.arange(MAX_LEN)).to(torch.int32)
    return cfg, weights, prompts, first, forced, replay, handles


def _prefill_batch(prompts, handles):
    ids = torch.cat(prompts)
    pos = torch.cat([torch.arange(len(p), dtype=torch.int32) for p in prompts])
    loc = torch.cat([handles[r, : len(p)] for r, p in enumerate(prompts)])
    seq = torch.tensor([len(p) for p in prompts], dtype=torch.int32)
    cu = torch.zeros(len(prompts) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(seq, 0)
    return ids, pos, loc, seq, cu


def _oracle_run(cfg, weights, prompts, first, forced, replay, handles, steps, use_replay=True):
    """Lock-step restatement of the engine on the oracle (bf16)."""
    w = {k: v.to(torch.bfloat16) for k, v in weights.items()}
    model = LoopedModel(cfg, w, "last_exited")
    b = len(prompts)
    num_pages = b * MAX_LEN + 1
    pool = SlotKVPool(model.slot_layout(), num_pages, cfg.kv_heads, cfg.head_dim, torch.bfloat16)
    ids, pos, loc, seq, cu = _prefill_batch(prompts, handles)
    pool.versions.reserve(loc.numpy())
    model.forward(Batch(ids, pos, loc, handles.clone(), seq, cu, True), pool)
    seq = seq + 1
    cur_ids = first.clone()
    depth = torch.zeros(b, dtype=torch.int32)
    slots = torch.arange(1, b + 1)
    state = {"hidden": torch.zeros(b + 1, cfg.hidden, dtype=torch.bfloat16),
             "exit": torch.zeros(b + 1, dtype=torch.float32)}
    cur = handles[torch.arange(b), seq.long() - 1]
    pool.versions.reserve(cur.numpy())
    state["hidden"][slots] = O.embedding(cur_ids, w["model.embed_tokens.weight"])
    preds = [[] for _ in range(b)]
    logits_at = [[] for _ in range(b)]
    depths_out = [[] for _ in range(b)]
    gates_all = []
    for _ in range(steps):
        batch = Batch(cur_ids.clone(), (seq - 1).clone(), handles[torch.arange(b), seq.long() - 1],
                      handles.clone(), seq.clone(), torch.arange(b + 1, dtype=torch.int32), False)
        gates = ocdb.core_phase(model, state, slots, depth.clone(), batch, pool)
        gates_all.append((gates.clone(), state["exit"][slots].clone(), depth.clone()))
        logits = model.lm_head(state["hidden"][slots], None).float()
        sampled = logits.argmax(-1).to(torch.int32)
        alias_h, alias_d, reserve_h, exited = [], [], [], []
        for r in range(b):
            d1 = int(depth[r]) + 1
            k = len(preds[r])
            fire = (k < K and d1 >= int(replay[r, k])) if use_replay else bool(gates[r])
            if d1 >= cfg.loop_steps or fire:
                if k < K:
                    preds[r].append(int(sampled[r]))
                    logits_at[r].append(logits[r])
                    depths_out[r].append(d1)
                alias_h.append(int(handles[r, seq[r] - 1]))
                alias_d.append(d1)
                cur_ids[r] = forced[r, k] if k < K else sampled[r]
                reserve_h.append(int(handles[r, seq[r]]))
                seq[r] += 1
                depth[r] = 0
                exited.append(r)
            else:
                depth[r] = d1
        if alias_h:
            pool.versions.release(np.array(alias_h), np.array(alias_d))
            pool.versions.reserve(np.array(reserve_h))
            emb = O.embedding(cur_ids, w["model.embed_tokens.weight"])
            for r in exited:
                state["hidden"][r + 1] = emb[r]
                state["exit"][r + 1] = 0.0
    return preds, logits_at, depths_out, pool, gates_all


def _gpu_run(cfg, weights, prompts, first, forced, replay, handles, steps, use_replay=True,
             graph=False):
    dev = torch.device("cuda")
    model = gpu_model(cfg, weights, "last_exited")  # imports the package
    from loop_sglang_b200.engine import CDBDecodeEngine
    from loop_sglang_b200.model import DeviceBatch

    b = len(prompts)
    kv = model.make_kv_cache(b * MAX_LEN + 1, 1)
    ids, pos, loc, seq, cu = _prefill_batch(prompts, handles)
    batch = DeviceBatch(ids.to(dev), pos.to(dev), loc.to(dev), handles.to(dev).contiguous(),
                        seq.to(dev), cu.to(dev), True, max_seqlen=MAX_LEN)
    kv.reserve_versions(batch.out_loc)
    model.forward(batch, kv)
    eng = CDBDecodeEngine(model, kv, b, MAX_LEN, K,
                          replay_depths=replay.to(dev).contiguous() if use_replay else None,
                          forced_ids=forced.to(dev).contiguous())
    eng.start(handles.to(dev), (seq + 1).to(dev), first.to(dev))
    if graph:
        eng.capture()  # one eager step, then the captured one
        for _ in range(steps - 2):
            eng.replay()
        eng.replay()
    else:
        for _ in range(steps):
            eng.step()
    torch.cuda.synchronize()
    return eng, kv


@pytest.mark.parametrize("graph", [False, True])
def test_cdb_engine_replay_matches_oracle(graph: bool) -> None:
    cfg, weights, prompts, first, forced, replay, handles = _setup(21)
    steps = int(replay.sum(1).max()) + 2
    preds, logits_at, depths_out, pool, _ = _oracle_run(cfg, weights, prompts, first, forced,
                                                        replay, handles, steps)
    eng, kv = _gpu_run(cfg, weights, prompts, first, forced, replay, handles, steps, graph=graph)
    count = eng.out_count.cpu()
    toks, deps = eng.out_tokens.cpu(), eng.out_depths.cpu()
    for r in range(len(prompts)):
        assert int(count[r]) >= K and len(preds[r]) == K, (r, int(count[r]), len(preds[r]))
        assert deps[r, :K].tolist() == depths_out[r] == replay[r].tolist(), r
        for k in range(K):
            got, want = int(toks[r, k]), preds[r][k]
            if got != want:  # accept a near tie of the oracle's own logits
                lg = logits_at[r][k]
                assert lg[got] >= lg.max() - 2e-2 * lg.abs().max(), (r, k, got, want)
    v = pool.versions
    assert np.array_equal(kv.slot_map.cpu().numpy(), v.slot_map)
    assert np.array_equal(kv.completed_depth.cpu().numpy(), v.completed_depth)
    assert int(kv._free_count.item()) == v.free_count
    n = v.free_count
    assert np.array_equal(kv._free_slots.cpu().numpy()[:n], v.free_slots[:n])
    from loop_sglang_b200 import ops  # imported by gpu_model above

    assert ops.device_error_word(reset=True) == 0


def test_cdb_engine_gates_match_oracle() -> None:
    """Without prescribed depths the device routes on its own gate: the first step's
    signals (and exit probabilities) match the oracle's where the decision is clear."""
    cfg, weights, prompts, first, forced, replay, handles = _setup(33)
    _, _, _, _, gates = _oracle_run(cfg, weights, prompts, first, forced, replay, handles, 1,
                                    use_replay=False)
    eng, _ = _gpu_run(cfg, weights, prompts, first, forced, replay, handles, 1, use_replay=False)
    want_sig, want_p, _ = gates[0]
    got_p = eng.state["exit"][eng.slots].float().cpu()
    exited = eng.exited.bool().cpu()
    # an exited row's exit state was reset by the successor's admission
    keep = ~exited
    assert torch.allclose(got_p[keep], want_p[keep], atol=2e-2)
    sure = (want_p - cfg.exit_threshold).abs() > 1e-3
    assert torch.equal(exited[sure], want_sig[sure] | torch.zeros_like(want_sig[sure]))
