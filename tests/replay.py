"""Replay the golden fixtures through the oracle (shared by the CPU and GPU tests).

The fixtures in ``tests/golden/`` were produced by the reference's own code
(``tests/golden/make_golden.py``). Each replay rebuilds the same seeded weights,
the same KV pool and the same per-step metadata, and runs the oracle model on
them; the GPU tests run the CUDA path on the same inputs.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from oracle import cdb
from oracle.model import Batch, LoopedConfig, LoopedModel, PagedKVPool, SlotKVPool, make_weights

GOLDEN = Path(__file__).resolve().parent / "golden"

OURO_TINY = LoopedConfig(arch="ouro", hidden=128, heads=4, kv_heads=4, head_dim=32,
                         intermediate=256, vocab=512, num_core_layers=2, loop_steps=3,
                         rope_theta=10000.0, max_position=256)
OURO_TINY_GATED = LoopedConfig(**{**OURO_TINY.__dict__, "exit_threshold": 0.5})
HUGINN_TINY = LoopedConfig(arch="huginn", hidden=96, heads=3, kv_heads=3, head_dim=32,
                           intermediate=192, vocab=384, num_prelude_layers=1, num_core_layers=2,
                           num_coda_layers=1, loop_steps=3, rope_theta=50000.0, max_position=256,
                           embed_scale=1.5, attention_bias=True, adapter_bias=True,
                           exit_threshold=0.8)

CB_CASES = {
    "ouro_cb_depth_indexed": (OURO_TINY, "depth_indexed"),
    "ouro_cb_shared": (OURO_TINY, "shared"),
    "ouro_cb_last_exited": (OURO_TINY, "last_exited"),
    "huginn_cb_shared": (HUGINN_TINY, "shared"),
}
CDB_CASES = {
    "ouro_cdb_last_exited": (OURO_TINY_GATED, "last_exited"),
    "ouro_cdb_shared": (OURO_TINY_GATED, "shared"),
    "huginn_cdb_last_exited": (HUGINN_TINY, "last_exited"),
}
NUM_PAGES = 256
CDB_NUM_PAGES = 512


def load(name: str) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / f"{name}.npz") as f:
        return {k: f[k] for k in f.files}


def batch_from(fx: dict, prefix: str, ids, is_prefill: bool) -> Batch:
    t = lambda k: torch.from_numpy(np.ascontiguousarray(fx[f"{prefix}_{k}"]))  # noqa: E731
    return Batch(
        input_ids=torch.as_tensor(np.asarray(ids)).to(torch.int32),
        positions=t("positions"),
        out_loc=t("out_loc"),
        page_table=t("page_table"),
        cache_seqlens=t("cache_seqlens"),
        cu_seqlens_q=t("cu_seqlens_q"),
        is_prefill=is_prefill,
    )


def cb_steps(fx: dict) -> list[tuple[str, bool]]:
    steps = [("prefill", True)]
    k = 0
    while f"decode{k}_logits" in fx:
        steps.append((f"decode{k}", False))
        k += 1
    return steps


def make_pool(model: LoopedModel, num_pages: int, page_size: int, dtype):
    c = model.cfg
    if model.policy == "last_exited":
        return SlotKVPool(model.slot_layout(), num_pages, c.kv_heads, c.head_dim, dtype)
    return PagedKVPool(model.num_kv_layers, num_pages, page_size, c.kv_heads, c.head_dim, dtype)


def replay_cb(name: str, dtype=torch.float32,
              tp: int = 1) -> tuple[dict, dict[str, torch.Tensor], object]:
    """Oracle logits for every step of a CB fixture; returns (fixture, logits-by-step, pool).
    ``tp``: the rounding points of that many tensor-parallel ranks."""
    cfg, policy = CB_CASES[name]
    fx = load(name)
    weights = make_weights(cfg, int(fx["seed"]), dtype=dtype, gate_bias=0.0)
    model = LoopedModel(cfg, weights, policy, tp=tp)
    pool = make_pool(model, NUM_PAGES, int(fx["page_size"]), dtype)
    out = {}
    for prefix, is_prefill in cb_steps(fx):
        batch = batch_from(fx, prefix, fx[f"{prefix}_ids"], is_prefill)
        if policy == "last_exited":
            pool.versions.reserve(batch.out_loc.numpy())
        out[prefix] = model.forward(batch, pool).float()
    return fx, out, pool


def replay_cdb(name: str, dtype=torch.float32,
               tp: int = 1) -> tuple[dict, dict[str, torch.Tensor]]:
    """Oracle prefill, prelude, mixed-depth core phases and coda for a CDB fixture
    (``tp``: the rounding points of that many tensor-parallel ranks)."""
    cfg, policy = CDB_CASES[name]
    fx = load(name)
    weights = make_weights(cfg, int(fx["seed"]), dtype=dtype, gate_bias=0.3)
    model = LoopedModel(cfg, weights, policy, tp=tp)
    pool = make_pool(model, CDB_NUM_PAGES, 1, dtype)
    res: dict[str, torch.Tensor] = {}
    pre = batch_from(fx, "prefill", fx["prefill_ids"], True)
    if policy == "last_exited":
        pool.versions.reserve(pre.out_loc.numpy())
    res["prefill_logits"] = model.forward(pre, pool).float()
    dec = batch_from(fx, "decode", fx["tokens"], False)
    if policy == "last_exited":
        pool.versions.reserve(dec.out_loc.numpy())
    rows = len(fx["tokens"])
    cap = rows + 5
    state = {"hidden": torch.zeros(cap, cfg.hidden, dtype=dtype)}
    if cfg.arch == "huginn":
        state["injection"] = torch.zeros(cap, cfg.hidden, dtype=dtype)
        state["exit"] = torch.zeros(cap, cfg.hidden, dtype=dtype)
    else:
        state["exit"] = torch.zeros(cap, dtype=torch.float32)
    slots = torch.arange(1, rows + 1)
    if isinstance(pool, SlotKVPool):
        model.resolve_fixed(dec, pool)
    hidden, inj = model.forward_prelude(dec, pool)
    state["hidden"].index_copy_(0, slots, hidden)
    if inj is not None:
        state["injection"].index_copy_(0, slots, inj)
    state["exit"].index_copy_(0, slots, model.init_exit_state(hidden))
    res["prelude_hidden"] = state["hidden"][slots].float()
    k = 0
    while f"core{k}_rows" in fx:
        srows = torch.from_numpy(fx[f"core{k}_rows"]).long()
        depths = torch.from_numpy(fx[f"core{k}_depths"])
        ids = fx["tokens"][(srows - 1).numpy()]
        batch = batch_from(fx, f"core{k}", ids, False)
        if isinstance(pool, SlotKVPool):
            model.resolve_fixed(batch, pool)
        gates = cdb.core_phase(model, state, srows, depths, batch, pool)
        res[f"core{k}_gates"] = gates
        res[f"core{k}_hidden"] = state["hidden"][srows].float()
        res[f"core{k}_exit"] = state["exit"][srows].float()
        if policy == "last_exited":
            res[f"core{k}_core_page_table"] = batch.core_page_table
            res[f"core{k}_core_out_loc"] = batch.core_out_loc
        k += 1
    if isinstance(pool, SlotKVPool):
        model.resolve_fixed(dec, pool)
    res["coda_logits"] = model.lm_head(model.forward_coda(state["hidden"][slots], dec, pool),
                                       dec).float()
    res["kv_buf"] = pool.buf
    return fx, res


# ---------------------------------------------------------------------------
# The same scenarios through the CUDA path (GPU tests only)
# ---------------------------------------------------------------------------


def gpu_model(cfg: LoopedConfig, weights, policy: str, comm=None):
    """The CUDA-path model; with ``comm`` this rank's tensor-parallel shard of it."""
    from __graft_entry__ import load_package

    load_package()
    from loop_sglang_b200.model import LoopedConfig as GpuConfig
    from loop_sglang_b200.model import LoopedDecoder

    return LoopedDecoder(GpuConfig(**cfg.__dict__), weights, policy, torch.device("cuda"),
                         comm=comm)


def device_batch(fx: dict, prefix: str, ids, is_prefill: bool, page_size: int):
    from loop_sglang_b200.model import DeviceBatch

    b = batch_from(fx, prefix, ids, is_prefill)
    dev = torch.device("cuda")
    return DeviceBatch(b.input_ids.to(dev), b.positions.to(dev), b.out_loc.to(dev),
                       b.page_table.to(dev).contiguous(), b.cache_seqlens.to(dev),
                       b.cu_seqlens_q.to(dev), is_prefill,
                       max_seqlen=int(b.page_table.shape[1]) * page_size)


def gpu_replay_cb(name: str, comm=None) -> tuple[dict, dict[str, torch.Tensor]]:
    """CUDA-path logits for every step of a CB fixture (bf16 weights; sharded over
    ``comm``'s ranks when given)."""
    cfg, policy = CB_CASES[name]
    fx = load(name)
    weights = make_weights(cfg, int(fx["seed"]), dtype=torch.float32, gate_bias=0.0)
    model = gpu_model(cfg, weights, policy, comm)
    page = int(fx["page_size"])
    kv = model.make_kv_cache(NUM_PAGES, page)
    out = {}
    for prefix, is_prefill in cb_steps(fx):
        batch = device_batch(fx, prefix, fx[f"{prefix}_ids"], is_prefill, page)
        if policy == "last_exited":
            kv.reserve_versions(batch.out_loc)
        out[prefix] = model.forward(batch, kv).float().cpu()
    return fx, out


def gpu_replay_cdb(name: str, comm=None) -> tuple[dict, dict[str, torch.Tensor]]:
    """CUDA-path prefill, prelude, mixed-depth fused core phases and coda of a CDB fixture
    (sharded over ``comm``'s ranks when given)."""
    cfg, policy = CDB_CASES[name]
    fx = load(name)
    weights = make_weights(cfg, int(fx["seed"]), dtype=torch.float32, gate_bias=0.3)
    model = gpu_model(cfg, weights, policy, comm)
    dev = torch.device("cuda")
    kv = model.make_kv_cache(CDB_NUM_PAGES, 1)
    res: dict[str, torch.Tensor] = {}
    pre = device_batch(fx, "prefill", fx["prefill_ids"], True, 1)
    if policy == "last_exited":
        kv.reserve_versions(pre.out_loc)
    res["prefill_logits"] = model.forward(pre, kv).float().cpu()
    dec = device_batch(fx, "decode", fx["tokens"], False, 1)
    if policy == "last_exited":
        kv.reserve_versions(dec.out_loc)
    rows = len(fx["tokens"])
    cap = rows + 5
    state = {"hidden": torch.zeros(cap, cfg.hidden, dtype=torch.bfloat16, device=dev)}
    if cfg.arch == "huginn":
        state["injection"] = torch.zeros(cap, cfg.hidden, dtype=torch.bfloat16, device=dev)
        state["exit"] = torch.zeros(cap, cfg.hidden, dtype=torch.bfloat16, device=dev)
    else:
        state["exit"] = torch.zeros(cap, dtype=torch.float32, device=dev)
    slots = torch.arange(1, rows + 1, device=dev)
    if policy == "last_exited":
        model.resolve_fixed(dec, kv)
    hidden, inj = model.forward_prelude(dec, kv)
    state["hidden"][slots] = hidden
    if inj is not None:
        state["injection"][slots] = inj
    state["exit"][slots] = model.init_exit_state(hidden)
    res["prelude_hidden"] = state["hidden"][slots].float().cpu()
    k = 0
    while f"core{k}_rows" in fx:
        srows = torch.from_numpy(fx[f"core{k}_rows"]).long().to(dev)
        depths = torch.from_numpy(fx[f"core{k}_depths"]).to(dev)
        ids = fx["tokens"][(fx[f"core{k}_rows"] - 1)]
        batch = device_batch(fx, f"core{k}", ids, False, 1)
        signal = torch.zeros(srows.numel(), dtype=torch.uint8, device=dev)
        model.core_step_exit(state, srows, depths, batch, kv, signal)
        res[f"core{k}_gates"] = signal.bool().cpu()
        res[f"core{k}_hidden"] = state["hidden"][srows].float().cpu()
        res[f"core{k}_exit"] = state["exit"][srows].float().cpu()
        if policy == "last_exited":
            res[f"core{k}_core_page_table"] = batch.core_page_table.cpu()
            res[f"core{k}_core_out_loc"] = batch.core_out_loc.cpu()
        k += 1
    if policy == "last_exited":
        model.resolve_fixed(dec, kv)
    res["coda_logits"] = model.lm_head(model.forward_coda(state["hidden"][slots], dec, kv),
                                       dec).float().cpu()
    return fx, res
