"""Device-routed continuous-depth batching and its lock-step oracle restatement.

Shared by the tiny CDB engine tests, the full-size (Ouro-1.4B) parity test and the
fixture generator ``tests/golden/make_fullsize.py``.

A run: the requests' prompts are prefilled at full depth into a last-exited KV pool,
then every step is one core step of every row at its own depth (the reference's
``CDBModelRunner._execute_phase("core")``, cdb_model_runner.py:94-109); rows that
reach their prescribed replay depth (cdb_scheduler.py:207-213, direct timing) or
full depth exit: their token is sampled greedily, their KV versions are aliased at
the exit depth and the successor's versions reserved, in row order
(cache.py:224-248, kvcache/last_exited.py:15-84), and the successor's prelude is
written into the row's state slot. Successor inputs are teacher-forced
(``forced``) so the oracle and the device take the same route.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from oracle import cdb as ocdb
from oracle import ops as O
from oracle.model import Batch, LoopedModel, SlotKVPool, with_fp32_matrices

TOPK = 8  # logits kept per output to judge near-ties without the whole vocabulary


@dataclass
class Scenario:
    prompts: list[torch.Tensor]  # int32 ids per request
    first: torch.Tensor  # [B] the first decoded token's id
    forced: torch.Tensor  # [B, K] ids fed after each output (teacher forcing)
    replay: torch.Tensor  # [B, K] prescribed exit depth of each output
    handles: torch.Tensor  # [B, max_len] token locations (one-token pages)
    max_len: int
    k: int  # outputs compared per row
    slots_per_token: int  # KV versions a full-depth token holds (Ouro: one per loop step)

    @property
    def steps(self) -> int:
        """Core steps until every row has produced ``k`` outputs (+2 spare)."""
        return int(self.replay.sum(1).max()) + 2

    @property
    def num_pages(self) -> int:
        """Handles of the last-exited pool; its version slots are as many, so it must hold
        every prompt token's and every decoded token's full-depth versions."""
        tokens = sum(len(p) for p in self.prompts) + len(self.prompts) * (self.steps + 1)
        return max(len(self.prompts) * self.max_len + 1, self.slots_per_token * tokens + 1)


def make_scenario(cfg, seed: int, prompt_lens: list[int], k: int, max_len: int,
                  depth_probs: tuple[float, ...] | None = None) -> Scenario:
    g = torch.Generator().manual_seed(seed + 1)
    b = len(prompt_lens)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g, dtype=torch.int32)
               for n in prompt_lens]
    first = torch.randint(0, cfg.vocab, (b,), generator=g, dtype=torch.int32)
    forced = torch.randint(0, cfg.vocab, (b, k), generator=g, dtype=torch.int32)
    if depth_probs is None:
        replay = torch.randint(1, cfg.loop_steps + 1, (b, k), generator=g, dtype=torch.int32)
    else:
        rng = np.random.default_rng(seed + 2)
        replay = torch.from_numpy(rng.choice(np.arange(1, cfg.loop_steps + 1), size=(b, k),
                                             p=depth_probs).astype(np.int32))
    handles = (1 + torch.arange(b).view(-1, 1) * max_len + torch.arange(max_len)).to(torch.int32)
    return Scenario(prompts, first, forced, replay, handles, max_len, k, cfg.loop_steps)


def prefill_batch(sc: Scenario):
    ids = torch.cat(sc.prompts)
    pos = torch.cat([torch.arange(len(p), dtype=torch.int32) for p in sc.prompts])
    loc = torch.cat([sc.handles[r, : len(p)] for r, p in enumerate(sc.prompts)])
    seq = torch.tensor([len(p) for p in sc.prompts], dtype=torch.int32)
    cu = torch.zeros(len(sc.prompts) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(seq, 0)
    return ids, pos, loc, seq, cu


def oracle_run(cfg, weights, sc: Scenario, use_replay: bool = True, steps: int | None = None,
               dtype: torch.dtype = torch.bfloat16):
    """Lock-step restatement of ``CDBDecodeEngine`` on the oracle (bf16 rounding points; fp32
    arithmetic throughout with ``dtype=torch.float32``, on the same bf16-valued weights).

    Returns a dict: ``preds`` [B][K] tokens, ``topk`` [B][K] (values, ids, max |logit|)
    of the logits at each output, ``hidden`` [B][K] the exiting rows' hidden, ``depths``
    [B][K], ``pool`` (the oracle pool), ``gates`` per step (signals, exit state, depth).
    """
    w = {k: v.to(torch.bfloat16).to(dtype) for k, v in weights.items()}
    model = LoopedModel(cfg, with_fp32_matrices(w), "last_exited")
    b = len(sc.prompts)
    steps = sc.steps if steps is None else steps
    assert model.slot_layout().slots_per_token == sc.slots_per_token
    pool = SlotKVPool(model.slot_layout(), sc.num_pages, cfg.kv_heads, cfg.head_dim, dtype)
    ids, pos, loc, seq, cu = prefill_batch(sc)
    pool.versions.reserve(loc.numpy())
    model.forward(Batch(ids, pos, loc, sc.handles.clone(), seq, cu, True), pool)
    seq = seq + 1
    cur_ids = sc.first.clone()
    depth = torch.zeros(b, dtype=torch.int32)
    slots = torch.arange(1, b + 1)
    state = {"hidden": torch.zeros(b + 1, cfg.hidden, dtype=dtype),
             "exit": torch.zeros(b + 1, dtype=torch.float32)}
    cur = sc.handles[torch.arange(b), seq.long() - 1]
    pool.versions.reserve(cur.numpy())
    state["hidden"][slots] = O.embedding(cur_ids, w["model.embed_tokens.weight"])
    out = {"preds": [[] for _ in range(b)], "topk": [[] for _ in range(b)],
           "hidden": [[] for _ in range(b)], "depths": [[] for _ in range(b)], "gates": []}
    k_max = sc.k
    for _ in range(steps):
        batch = Batch(cur_ids.clone(), (seq - 1).clone(),
                      sc.handles[torch.arange(b), seq.long() - 1], sc.handles.clone(),
                      seq.clone(), torch.arange(b + 1, dtype=torch.int32), False)
        gates = ocdb.core_phase(model, state, slots, depth.clone(), batch, pool)
        out["gates"].append((None if gates is None else gates.clone(),
                             state["exit"][slots].clone(), depth.clone()))
        hid = state["hidden"][slots]
        logits = model.lm_head(hid, None).float()
        sampled = logits.argmax(-1).to(torch.int32)
        alias_h, alias_d, reserve_h, exited = [], [], [], []
        for r in range(b):
            d1 = int(depth[r]) + 1
            k = len(out["preds"][r])
            fire = (k < k_max and d1 >= int(sc.replay[r, k])) if use_replay else bool(gates[r])
            if d1 >= cfg.loop_steps or fire:
                if k < k_max:
                    out["preds"][r].append(int(sampled[r]))
                    v, i = logits[r].topk(TOPK)
                    out["topk"][r].append((v.clone(), i.to(torch.int32).clone(),
                                           float(logits[r].abs().max())))
                    out["hidden"][r].append(hid[r].clone())
                    out["depths"][r].append(d1)
                alias_h.append(int(sc.handles[r, seq[r] - 1]))
                alias_d.append(d1)
                cur_ids[r] = sc.forced[r, k] if k < k_max else sampled[r]
                reserve_h.append(int(sc.handles[r, seq[r]]))
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
    out["pool"] = pool
    return out


def gpu_run(model, sc: Scenario, use_replay: bool = True, graph: bool = False,
            steps: int | None = None, on_step=None):
    """The same run through ``CDBDecodeEngine`` (``model`` a last-exited ``LoopedDecoder``).
    Returns the engine and its KV cache; outputs are in ``eng.out_tokens`` /
    ``eng.out_depths``. ``on_step(eng)`` (eager runs only) is called after every step."""
    from loop_sglang_b200.engine import CDBDecodeEngine
    from loop_sglang_b200.model import DeviceBatch

    dev = model.device
    b = len(sc.prompts)
    steps = sc.steps if steps is None else steps
    kv = model.make_kv_cache(sc.num_pages, 1)
    ids, pos, loc, seq, cu = prefill_batch(sc)
    batch = DeviceBatch(ids.to(dev), pos.to(dev), loc.to(dev), sc.handles.to(dev).contiguous(),
                        seq.to(dev), cu.to(dev), True, max_seqlen=sc.max_len)
    kv.reserve_versions(batch.out_loc)
    model.forward(batch, kv)
    eng = CDBDecodeEngine(model, kv, b, sc.max_len, sc.k,
                          replay_depths=sc.replay.to(dev).contiguous() if use_replay else None,
                          forced_ids=sc.forced.to(dev).contiguous())
    eng.start(sc.handles.to(dev), (seq + 1).to(dev), sc.first.to(dev))
    if graph:
        eng.capture()  # one eager step, then the captured one
        for _ in range(steps - 1):
            eng.replay()
    else:
        for _ in range(steps):
            eng.step()
            if on_step is not None:
                torch.cuda.synchronize()
                on_step(eng)
    torch.cuda.synchronize()
    return eng, kv


def token_matches(got: int, want: int, topk, rel_tol: float = 2e-2) -> str:
    """'agree', 'near_tie' (the oracle's logit of ``got`` is within ``rel_tol`` x max |logit|
    of its max: bf16 reduction order may take either) or 'mismatch'."""
    if got == want:
        return "agree"
    vals, idx, scale = topk
    tol = rel_tol * scale
    hit = (idx == got).nonzero()
    if hit.numel() and float(vals[hit[0, 0]]) >= float(vals[0]) - tol:
        return "near_tie"
    return "mismatch"
