"""Generate the golden fixtures of ``tests/golden/`` by running the REFERENCE on the CPU.

Usage (in a container that has the Loop-SGLang sources; nothing here runs on the
GPU box, which only reads the committed ``*.npz`` files)::

    python tests/golden/make_golden.py --reference <loop-sglang checkout>/python

What runs is the reference's own code:

* its model classes ``OuroForCausalLM`` / ``HuginnForCausalLM`` (fp32, seeded
  weights from ``oracle.model.make_weights``) through its ``FlashAttentionBackend``
  (metadata, last-exited resolution, KV store), with two CPU substitutions for
  calls that need a GPU: the FlashInfer element-wise ops (norm, RoPE, SiLU*mul)
  and the final paged-attention library call are replaced by the oracle's
  restatements;
* its Triton kernels (page-table metadata, batch inputs, request-table
  assignment, last-exited reserve / alias / free / resolve) through the Triton
  interpreter (``TRITON_INTERPRET=1``), which runs programs in ascending order;
* its ``store_cache`` CPU fallback;
* its streaming weight loader ``load_weight`` (tensor-parallel shard + merge) on a
  small safetensors checkpoint, once per rank of two world sizes;
* its ``RadixPrefixCache`` on a seeded sequence of matches, inserts, locks and
  evictions (page sizes 1 and 4);
* its two KV pools' retraction snapshots (``get_cpu_copy`` / ``load_cpu_copy``);
* BASELINE configs[0] (the tiny Ouro model, 4 x 128-token prompts, 32 greedy tokens).

Each fixture stores inputs and outputs; ``tests/test_oracle_golden.py`` checks
that the oracle reproduces them (integers exactly, fp32 to 1e-5).
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from oracle import ops  # noqa: E402
from oracle.model import LoopedConfig, make_weights  # noqa: E402

# ---------------------------------------------------------------------------
# CPU substitutes for the library calls that need a GPU
# ---------------------------------------------------------------------------


def _fi_rmsnorm(x, w, eps, out=None, **_):
    y = ops.rmsnorm(x, w, eps)
    if out is not None:
        out.copy_(y)
        return out
    return y


def _fi_fused_add_rmsnorm(x, residual, w, eps, **_):
    y, r = ops.fused_add_rmsnorm(x, residual, w, eps)
    x.copy_(y)
    residual.copy_(r)


def _fi_rope(positions, query, key, head_size, cos_sin_cache, is_neox=True):
    assert is_neox
    t = query.shape[0]
    q = query.view(t, -1, head_size)
    k = key.view(t, -1, head_size)
    q.copy_(ops.apply_rope_neox(positions, q, cos_sin_cache))
    k.copy_(ops.apply_rope_neox(positions, k, cos_sin_cache))


def _fi_silu_and_mul(x, out=None, **_):
    y = ops.silu_and_mul(x)
    if out is not None:
        out.copy_(y)
        return out
    return y


def _attention_substitute(q, k_cache, v_cache, page_table, cache_seqlens, cu_seqlens_q,
                          cu_seqlens_k, max_seqlen_q, softmax_scale, version, **_):
    return ops.paged_attention(q, k_cache, v_cache, page_table, cache_seqlens, cu_seqlens_q,
                               softmax_scale)


def install_reference(ref_python: Path):
    sys.path.insert(0, str(ref_python))
    import flashinfer

    flashinfer.rmsnorm = _fi_rmsnorm
    flashinfer.fused_add_rmsnorm = _fi_fused_add_rmsnorm
    flashinfer.apply_rope_with_cos_sin_cache_inplace = _fi_rope
    flashinfer.silu_and_mul = _fi_silu_and_mul
    from loopsgl.distributed import set_tp_info
    from loopsgl.layers.rotary import set_rope_device

    set_tp_info(0, 1)
    set_rope_device(torch.device("cpu"))
    import loopsgl.attention.fa as fa

    fa._fa_sgl_impl = _attention_substitute


# ---------------------------------------------------------------------------
# Model runs through the reference's code
# ---------------------------------------------------------------------------


def reference_model(cfg: LoopedConfig, weights: dict[str, torch.Tensor], policy: str):
    from transformers import PretrainedConfig

    from loopsgl.core import LoopParams
    from loopsgl.models.config import ModelConfig, RotaryConfig
    from loopsgl.models.looped.huginn import HuginnForCausalLM
    from loopsgl.models.looped.ouro import OuroForCausalLM

    hf = PretrainedConfig()
    hf.min_loop_steps = cfg.min_loop_steps
    hf.exit_gate_type = cfg.exit_gate_type
    hf.num_prelude_layers = cfg.num_prelude_layers
    hf.num_core_layers = cfg.num_core_layers
    hf.num_coda_layers = cfg.num_coda_layers
    hf.attention_bias = cfg.attention_bias
    hf.bias = cfg.adapter_bias
    hf.init_values = {"embed_scale": cfg.embed_scale, "std": 0.0}
    hf.state_init = "zero"
    mc = ModelConfig(
        num_layers=cfg.num_core_layers if cfg.arch == "ouro" else cfg.num_layers,
        num_qo_heads=cfg.heads,
        num_kv_heads=cfg.kv_heads,
        head_dim=cfg.head_dim,
        hidden_size=cfg.hidden,
        vocab_size=cfg.vocab,
        intermediate_size=cfg.intermediate,
        rms_norm_eps=cfg.rms_eps,
        rotary_config=RotaryConfig(cfg.head_dim, cfg.head_dim, cfg.max_position, cfg.rope_theta,
                                   None),
        hidden_act="silu",
        tie_word_embeddings=cfg.tie_word_embeddings,
        num_experts=0,
        num_experts_per_tok=0,
        moe_intermediate_size=0,
        norm_topk_prob=False,
        model_type="ouro" if cfg.arch == "ouro" else "huginn_raven",
        architectures=["OuroForCausalLM" if cfg.arch == "ouro" else "HuginnForCausalLM"],
        loop_params=LoopParams(loop_steps=cfg.loop_steps, exit_threshold=cfg.exit_threshold),
        hf_config=hf,
    )
    model = (OuroForCausalLM if cfg.arch == "ouro" else HuginnForCausalLM)(mc)
    model.load_state_dict({k: v.clone() for k, v in weights.items()})
    model.model.loop_cache_policy = policy
    return model, mc


class RefRun:
    """Drive a reference model through prefill / CB decode / CDB phases on the CPU."""

    def __init__(self, cfg, weights, policy, page_size, num_pages, max_reqs, max_len):
        import loopsgl.core as core
        from loopsgl.attention.fa import FlashAttentionBackend
        from loopsgl.kvcache.last_exited import LastExitedKVCache
        from loopsgl.kvcache.mha_pool import MHAKVCache

        self.cfg, self.policy, self.page_size = cfg, policy, page_size
        self.model, self.mc = reference_model(cfg, weights, policy)
        core._GLOBAL_CTX = None
        ctx = core.Context(page_size=page_size)
        nl = self.model.model.num_kv_layers
        if policy == "last_exited":
            m = self.model.model
            ctx.kv_cache = LastExitedKVCache(cfg.kv_heads, nl, cfg.head_dim, num_pages, 1,
                                             torch.float32, torch.device("cpu"),
                                             m.num_prelude_layers,
                                             m.num_prelude_layers + m.num_core_layers,
                                             cfg.loop_steps)
        else:
            ctx.kv_cache = MHAKVCache(cfg.kv_heads, nl, cfg.head_dim, num_pages, page_size,
                                      torch.float32, torch.device("cpu"))
        # the pools allocate with torch.empty; zero them so checksums only see written rows
        ctx.kv_cache._kv_buffer.zero_()
        ctx.page_table = torch.zeros(max_reqs + 1, max_len, dtype=torch.int32)
        core.set_global_ctx(ctx)
        ctx.attn_backend = FlashAttentionBackend(self.mc)
        self.ctx = ctx
        self.next_page = 1
        self.seq_lens = {}

    def allocate(self, row: int, new_len: int) -> torch.Tensor:
        """Extend request ``row`` to ``new_len`` tokens with fresh page-aligned locations."""
        old = self.seq_lens.get(row, 0)
        p = self.page_size
        locs = []
        page = int(self.ctx.page_table[row, old - 1]) // p if old % p else 0
        for pos in range(old, new_len):
            if pos % p == 0:
                page = self.next_page
                self.next_page += 1
            locs.append(page * p + pos % p)
        locs_t = torch.tensor(locs, dtype=torch.int32)
        self.ctx.page_table[row, old:new_len] = locs_t
        if self.policy == "last_exited" and len(locs):
            self.ctx.kv_cache.reserve_versions(locs_t)
        self.seq_lens[row] = new_len
        return locs_t

    def batch(self, rows, extend, phase):
        from loopsgl.core import ForwardBatch
        from loopsgl.kernel.batch import prepare_batch_inputs

        seq = [self.seq_lens[r] for r in rows]
        fb = ForwardBatch(
            size=len(rows), phase=phase,
            req_pool_indices=torch.tensor(rows, dtype=torch.int32),
            seq_lens=torch.tensor(seq, dtype=torch.int32),
            extend_lens=torch.tensor(extend, dtype=torch.int32),
            seq_lens_cpu=tuple(seq), extend_lens_cpu=tuple(extend))
        prepare_batch_inputs(fb, self.ctx.page_table)
        return fb

    def run(self, fb, input_ids):
        fb.input_ids = input_ids
        with self.ctx.forward_batch(fb):
            self.ctx.attn_backend.prepare_metadata(fb)
            logits = self.model.forward()
        return fb, logits

    def phase(self, fb, input_ids, fn):
        fb.input_ids = input_ids
        with self.ctx.forward_batch(fb):
            self.ctx.attn_backend.prepare_metadata(fb)
            return fb, fn()


def snapshot_meta(fb) -> dict:
    md = fb.attn_metadata
    out = {
        "positions": fb.positions.numpy().copy(),
        "out_loc": fb.out_loc.numpy().copy(),
        "page_table": md.page_table.numpy().copy(),
        "cache_seqlens": md.cache_seqlens.numpy().copy(),
        "cu_seqlens_q": md.cu_seqlens_q.numpy().copy(),
    }
    return out


def model_case(name, cfg, policy, seed, prompts, decode_steps, page_size, out_dir):
    weights = make_weights(cfg, seed, dtype=torch.float32, gate_bias=0.0)
    num_pages = 256
    run = RefRun(cfg, weights, policy, page_size, num_pages, max_reqs=8, max_len=64)
    rows = list(range(1, len(prompts) + 1))
    rec: dict[str, np.ndarray] = {"seed": np.array(seed), "page_size": np.array(page_size)}
    # prefill every prompt in one extend batch
    for r, p in zip(rows, prompts):
        run.allocate(r, len(p))
    ids = torch.tensor([t for p in prompts for t in p], dtype=torch.int32)
    fb, logits = run.run(run.batch(rows, [len(p) for p in prompts], "prefill"), ids)
    rec["prefill_ids"] = ids.numpy()
    for k, v in snapshot_meta(fb).items():
        rec[f"prefill_{k}"] = v
    rec["prefill_logits"] = logits.numpy()
    tokens = torch.argmax(logits, dim=-1).to(torch.int32)
    for step in range(decode_steps):
        for r in rows:
            run.allocate(r, run.seq_lens[r] + 1)
        fb, logits = run.run(run.batch(rows, [1] * len(rows), "decode"), tokens)
        rec[f"decode{step}_ids"] = tokens.numpy()
        for k, v in snapshot_meta(fb).items():
            rec[f"decode{step}_{k}"] = v
        rec[f"decode{step}_logits"] = logits.numpy()
        tokens = torch.argmax(logits, dim=-1).to(torch.int32)
    rec["final_tokens"] = tokens.numpy()
    kv = run.ctx.kv_cache._kv_buffer
    rec["kv_checksum"] = kv.double().sum(dim=tuple(range(2, kv.ndim))).numpy()
    if policy == "last_exited":
        rec["slot_map"] = run.ctx.kv_cache.slot_map.numpy().copy()
    np.savez_compressed(out_dir / f"{name}.npz", **rec)
    print(f"wrote {name}: prefill logits {tuple(logits.shape)}")


def cdb_case(name, cfg, policy, seed, prompts, depth_plan, out_dir):
    """Prefill, then CDB phases with mixed per-row depths through the reference's model
    phase methods, mirroring ``CDBModelRunner._execute_phase`` (cdb_model_runner.py:81-109)."""
    weights = make_weights(cfg, seed, dtype=torch.float32, gate_bias=0.3)
    run = RefRun(cfg, weights, policy, 1, 512, max_reqs=8, max_len=64)
    model = run.model.model
    rows = list(range(1, len(prompts) + 1))
    for r, p in zip(rows, prompts):
        run.allocate(r, len(p))
    ids = torch.tensor([t for p in prompts for t in p], dtype=torch.int32)
    fb, logits = run.run(run.batch(rows, [len(p) for p in prompts], "prefill"), ids)
    tokens = torch.argmax(logits, dim=-1).to(torch.int32)
    rec: dict[str, np.ndarray] = {"seed": np.array(seed), "prefill_ids": ids.numpy(),
                                  "prefill_logits": logits.numpy(), "tokens": tokens.numpy()}
    for key, val in snapshot_meta(fb).items():
        rec[f"prefill_{key}"] = val
    for r in rows:
        run.allocate(r, run.seq_lens[r] + 1)
    # state pool rows are the request rows (slot = req_pool_idx)
    cap = len(rows) + 4
    pool = {"hidden": torch.zeros(cap, cfg.hidden)}
    if cfg.arch == "huginn":
        pool["injection"] = torch.zeros(cap, cfg.hidden)
        pool["exit"] = torch.zeros(cap, cfg.hidden)
    else:
        pool["exit"] = torch.zeros(cap, dtype=torch.float32)
    slots = torch.tensor(rows, dtype=torch.int64)

    def prelude():
        hidden, inj = model.forward_prelude(run.ctx.batch.input_ids)
        pool["hidden"].index_copy_(0, slots, hidden)
        if inj is not None:
            pool["injection"].index_copy_(0, slots, inj)
        pool["exit"].index_copy_(0, slots, model.init_exit_state(hidden))

    fb, _ = run.phase(run.batch(rows, [1] * len(rows), "decode"), tokens, prelude)
    rec["prelude_hidden"] = pool["hidden"][slots].numpy().copy()
    for key, val in snapshot_meta(fb).items():
        rec[f"decode_{key}"] = val
    for k, depths in enumerate(depth_plan):
        sel = [i for i, d in enumerate(depths) if d is not None]
        srows = [rows[i] for i in sel]
        sslots = slots[sel]
        d = torch.tensor([depths[i] for i in sel], dtype=torch.int32)

        def core_fn():
            hidden = pool["hidden"].index_select(0, sslots)
            inj = pool["injection"].index_select(0, sslots) if "injection" in pool else None
            exit_state = pool["exit"].index_select(0, sslots)
            hidden = model.core_step(hidden, d, inj)
            gates, exit_state = model.exit_signal(hidden, exit_state, d)
            pool["exit"].index_copy_(0, sslots, exit_state)
            pool["hidden"].index_copy_(0, sslots, hidden)
            return gates

        fb, gates = run.phase(run.batch(srows, [1] * len(srows), "decode"), tokens[sel], core_fn)
        rec[f"core{k}_rows"] = np.array(srows, np.int32)
        rec[f"core{k}_depths"] = d.numpy()
        rec[f"core{k}_gates"] = gates.numpy()
        rec[f"core{k}_hidden"] = pool["hidden"][sslots].numpy().copy()
        rec[f"core{k}_exit"] = pool["exit"][sslots].numpy().copy()
        for key, val in snapshot_meta(fb).items():
            rec[f"core{k}_{key}"] = val
        if policy == "last_exited":
            md = fb.attn_metadata
            rec[f"core{k}_core_page_table"] = md.core_page_table.numpy().copy()
            rec[f"core{k}_core_out_loc"] = md.core_out_loc.numpy().copy()

    def coda():
        return run.model.forward_coda(pool["hidden"].index_select(0, slots))

    _, logits = run.phase(run.batch(rows, [1] * len(rows), "decode"), tokens, coda)
    rec["coda_logits"] = logits.numpy()
    kv = run.ctx.kv_cache._kv_buffer
    rec["kv_checksum"] = kv.double().sum(dim=tuple(range(2, kv.ndim))).numpy()
    np.savez_compressed(out_dir / f"{name}.npz", **rec)
    print(f"wrote {name}")


# ---------------------------------------------------------------------------
# Integer kernels through the Triton interpreter
# ---------------------------------------------------------------------------


def last_exited_case(name, num_layers, core_start, core_end, steps, num_pages, out_dir):
    from loopsgl.kvcache.last_exited import LastExitedKVCache

    pool = LastExitedKVCache(2, num_layers, 4, num_pages, 1, torch.float32, torch.device("cpu"),
                             core_start, core_end, steps)
    rec: dict[str, np.ndarray] = {
        "layout": np.array([num_layers, core_start, core_end, steps, num_pages], np.int32)}
    rng = np.random.default_rng(7)

    def snap(tag):
        rec[f"{tag}_slot_map"] = pool.slot_map.numpy().copy()
        rec[f"{tag}_completed"] = pool.completed_depth.numpy().copy()
        rec[f"{tag}_free"] = pool._free_slots.numpy().copy()
        rec[f"{tag}_count"] = pool._free_count.numpy().copy()

    ops_log = []
    h1 = torch.tensor([3, 5, 1, 7], dtype=torch.int32)
    pool.reserve_versions(h1)
    ops_log.append(("reserve", h1.numpy(), None))
    snap("op0")
    ex = torch.tensor([1, steps], dtype=torch.int32)
    released = int(sum(steps - int(e) for e in ex))
    pool.alias_versions(h1[:2], ex, released)
    rec["op1_handles"], rec["op1_exits"] = h1[:2].numpy(), ex.numpy()
    snap("op1")
    h2 = torch.tensor([2, 9], dtype=torch.int32)
    pool.reserve_versions(h2)
    rec["op2_handles"] = h2.numpy()
    snap("op2")
    fh = torch.tensor([1, 3], dtype=torch.int32)
    freed = int(sum(pool.fixed_groups + int(pool.completed_depth[int(h)]) * pool.core_groups
                    for h in fh))
    pool.free_versions(fh, freed)
    rec["op3_handles"] = fh.numpy()
    snap("op3")
    # restore-style reservation with explicit completed depths
    h4 = torch.tensor([4, 6], dtype=torch.int32)
    depths4 = torch.tensor([2, 1], dtype=torch.int32)
    fixed_bytes = 2 * pool._expanded_layers * len(h4) * pool._row_bytes
    backup = torch.zeros(fixed_bytes + len(h4) * 4, dtype=torch.uint8)
    backup[-len(h4) * 4:].view(torch.int32).copy_(depths4)
    pool.reserve_restore_versions(h4, backup)
    rec["op4_handles"], rec["op4_depths"] = h4.numpy(), depths4.numpy()
    snap("op4")
    # resolve: rows of live handles, per-row depths and a scalar depth
    from loopsgl.attention.metadata import prepare_last_exited_metadata

    live = np.array([5, 7, 2, 9, 4, 6], np.int32)
    table = torch.from_numpy(np.stack([rng.permutation(live)[:4] for _ in range(3)]).astype(
        np.int32))
    seq = torch.tensor([4, 2, 3], dtype=torch.int32)
    cu = torch.tensor([0, 1, 3, 4], dtype=torch.int32)
    lout = torch.tensor([7, 2, 9, 6], dtype=torch.int32)
    groups = pool.core_groups
    for tag, depths in (("vec", torch.tensor([0, steps - 1, 1], dtype=torch.int32)),
                        ("scalar", 1)):
        phys = torch.full((groups, 3, 4), -1, dtype=torch.int32)
        pout = torch.full((groups, 4), -1, dtype=torch.int32)
        prepare_last_exited_metadata(table, phys, pool.version_map, seq, cu, lout, pout, depths)
        rec[f"resolve_{tag}_table"] = phys.numpy()
        rec[f"resolve_{tag}_out"] = pout.numpy()
        rec[f"resolve_{tag}_depths"] = np.array(depths if isinstance(depths, int) else depths.numpy())
    rec["resolve_logical"] = table.numpy()
    rec["resolve_seq"] = seq.numpy()
    rec["resolve_cu"] = cu.numpy()
    rec["resolve_lout"] = lout.numpy()
    if pool.fixed_groups:
        phys = torch.full((pool.fixed_groups, 3, 4), -1, dtype=torch.int32)
        pout = torch.full((pool.fixed_groups, 4), -1, dtype=torch.int32)
        prepare_last_exited_metadata(table, phys, pool.fixed_map, seq, cu, lout, pout, 0)
        rec["resolve_fixed_table"] = phys.numpy()
        rec["resolve_fixed_out"] = pout.numpy()
    np.savez_compressed(out_dir / f"{name}.npz", **rec)
    print(f"wrote {name}")


def metadata_case(out_dir):
    from loopsgl.attention.metadata import extend_set_metadata, normal_decode_set_metadata
    from loopsgl.core import ForwardBatch
    from loopsgl.kernel.batch import assign_req_to_token_pool_func, prepare_batch_inputs

    rng = np.random.default_rng(11)
    rec: dict[str, np.ndarray] = {}
    page = 4
    rows, width = 6, 40
    req_to_token = torch.zeros(rows, width, dtype=torch.int32)
    # assign: three requests get ranges of fresh locations
    rpi = torch.tensor([2, 5, 1], dtype=torch.int32)
    start = torch.tensor([0, 0, 0], dtype=torch.int32)
    end = torch.tensor([13, 7, 21], dtype=torch.int32)
    out_cache = torch.from_numpy(rng.permutation(np.arange(4, 4 + 41)).astype(np.int32))
    assign_req_to_token_pool_func(rpi, req_to_token, start, end, out_cache, 3)
    rec.update(assign_rpi=rpi.numpy(), assign_start=start.numpy(), assign_end=end.numpy(),
               assign_out=out_cache.numpy(), assign_table=req_to_token.numpy().copy())
    # page-aligned table for metadata: location = page*4 + offset
    r2t = torch.zeros(rows, width, dtype=torch.int32)
    pages = rng.permutation(np.arange(1, 80))
    k = 0
    for r in range(rows):
        for c in range(0, width, page):
            r2t[r, c:c + page] = int(pages[k]) * page + torch.arange(page)
            k += 1
    rec["r2t"] = r2t.numpy()
    seq = torch.tensor([13, 7, 21], dtype=torch.int32)
    ext = torch.tensor([5, 7, 2], dtype=torch.int32)
    for tag, is_decode in (("decode", True), ("extend", False)):
        bs = 3
        cache = torch.zeros(bs, dtype=torch.int32)
        cuk = torch.zeros(bs + 1, dtype=torch.int32)
        cuq = torch.zeros(bs + 1, dtype=torch.int32)
        pt = torch.full((bs, 8), -1, dtype=torch.int32)
        maxp = (int(seq.max()) + page - 1) // page
        if is_decode:
            normal_decode_set_metadata(cache, cuk, pt, r2t, rpi, maxp, seq, 0, page, cuq)
        else:
            extend_set_metadata(cache, cuk, cuq, pt, r2t, rpi, maxp, seq, ext, page)
        rec.update({f"{tag}_cache": cache.numpy(), f"{tag}_cuk": cuk.numpy(),
                    f"{tag}_cuq": cuq.numpy(), f"{tag}_pt": pt.numpy()})
        extend = [1, 1, 1] if is_decode else ext.tolist()
        fb = ForwardBatch(size=bs, phase="decode" if is_decode else "prefill",
                          req_pool_indices=rpi, seq_lens=seq,
                          extend_lens=torch.tensor(extend, dtype=torch.int32),
                          seq_lens_cpu=tuple(seq.tolist()), extend_lens_cpu=tuple(extend))
        mapping, positions = prepare_batch_inputs(fb, r2t)
        rec.update({f"{tag}_positions": positions.numpy(), f"{tag}_mapping": mapping.numpy(),
                    f"{tag}_outloc": fb.out_loc.numpy()})
    rec["seq"], rec["ext"], rec["rpi"] = seq.numpy(), ext.numpy(), rpi.numpy()
    np.savez_compressed(out_dir / "metadata.npz", **rec)
    print("wrote metadata")


def store_case(out_dir):
    from loopsgl.kernel.store import store_cache

    g = torch.Generator().manual_seed(5)
    k_cache = torch.full((17, 2, 8), -7.0)
    v_cache = torch.full((17, 2, 8), -7.0)
    k = torch.randn(5, 2, 8, generator=g)
    v = torch.randn(5, 2, 8, generator=g)
    idx = torch.tensor([0, 16, 0, 11, 7], dtype=torch.int64)
    store_cache(k_cache, v_cache, idx, k, v)
    np.savez_compressed(out_dir / "store.npz", k=k.numpy(), v=v.numpy(), idx=idx.numpy(),
                        k_cache=k_cache.numpy(), v_cache=v_cache.numpy())
    print("wrote store")

# ---------------------------------------------------------------------------
# Tensor-parallel weight sharding through the reference's own loader
# ---------------------------------------------------------------------------

TP_CFG = dict(hidden=32, heads=4, kv_heads=2, head_dim=8, intermediate=48, vocab=37)


def tp_shard_case(out_dir):
    """A tiny unmerged checkpoint (q/k/v with biases, gate/up, o/down, norms, embedding,
    LM head; vocabulary 37 so the last rank's range is short) written as safetensors and
    read back by ``loopsgl.models.weight.load_weight`` for every rank of worlds 2 and 4
    (4 > kv heads, so k/v are replicated there). Stores the inputs and every rank's
    sharded, merged tensors."""
    import tempfile
    from types import SimpleNamespace

    import loopsgl.distributed.info as tp_info
    from loopsgl.distributed import set_tp_info
    from loopsgl.models.weight import load_weight
    from safetensors.torch import save_file

    c = TP_CFG
    h, d, f, v = c["hidden"], c["head_dim"], c["intermediate"], c["vocab"]
    g = torch.Generator().manual_seed(11)
    p = "model.layers.0"
    shapes = {
        f"{p}.self_attn.q_proj.weight": (c["heads"] * d, h),
        f"{p}.self_attn.k_proj.weight": (c["kv_heads"] * d, h),
        f"{p}.self_attn.v_proj.weight": (c["kv_heads"] * d, h),
        f"{p}.self_attn.q_proj.bias": (c["heads"] * d,),
        f"{p}.self_attn.k_proj.bias": (c["kv_heads"] * d,),
        f"{p}.self_attn.v_proj.bias": (c["kv_heads"] * d,),
        f"{p}.self_attn.o_proj.weight": (h, c["heads"] * d),
        f"{p}.mlp.gate_proj.weight": (f, h),
        f"{p}.mlp.up_proj.weight": (f, h),
        f"{p}.mlp.down_proj.weight": (h, f),
        f"{p}.input_layernorm.weight": (h,),
        "model.norm.weight": (h,),
        "model.embed_tokens.weight": (v, h),
        "lm_head.weight": (v, h),
    }
    tensors = {k: torch.randn(*s, generator=g) for k, s in shapes.items()}
    rec = {f"in::{k}": t.numpy() for k, t in tensors.items()}
    rec.update({k: np.array(val) for k, val in c.items()})
    mc = SimpleNamespace(num_kv_heads=c["kv_heads"], is_moe=False)
    with tempfile.TemporaryDirectory(dir=out_dir) as tmp:
        save_file(tensors, os.path.join(tmp, "model.safetensors"))
        for world in (2, 4):
            for rank in range(world):
                tp_info._TP_INFO = None
                set_tp_info(rank, world)
                for name, t in load_weight(tmp, torch.device("cpu"), model_config=mc):
                    rec[f"w{world}r{rank}::{name}"] = t.numpy().copy()
    tp_info._TP_INFO = None
    set_tp_info(0, 1)
    np.savez_compressed(out_dir / "tp_shard.npz", **rec)
    print("wrote tp_shard")


# ---------------------------------------------------------------------------
# Radix prefix cache: a seeded operation sequence through the reference's tree
# ---------------------------------------------------------------------------


def radix_ops(page_size: int, seed: int, n_ops: int = 160) -> list[dict]:
    """A scheduler-like sequence: requests made of one of four shared prefixes plus a
    suffix over a small alphabet (so partial matches and splits are common) are matched,
    locked, inserted with fresh page-aligned locations and later released; evictions
    and unlocked probes are interleaved."""
    rng = np.random.default_rng(seed)
    prefixes = [rng.integers(0, 5, int(rng.integers(2, 7)) * page_size).tolist() for _ in range(4)]
    ops: list[dict] = []
    live: list[int] = []  # op numbers of requests whose inserted handle is locked
    next_page = 1
    for _ in range(n_ops):
        r = rng.random()
        if r < 0.5 or not live:
            ids = list(prefixes[int(rng.integers(0, 4))])
            ids += rng.integers(0, 3, int(rng.integers(0, 4 * page_size + 3))).tolist()
            if rng.random() < 0.2:
                ids = rng.integers(0, 5, int(rng.integers(1, 6 * page_size))).tolist()
            pages = -(-len(ids) // page_size)
            fresh = [(next_page + i // page_size) * page_size + i % page_size
                     for i in range(pages * page_size)]
            next_page += pages
            ops.append({"kind": "request", "ids": ids, "fresh": fresh})
            live.append(len(ops) - 1)
        elif r < 0.75:
            ops.append({"kind": "finish", "ref": live.pop(int(rng.integers(0, len(live))))})
        elif r < 0.9:
            ops.append({"kind": "evict", "frac": float(rng.random())})
        else:
            ids = list(prefixes[int(rng.integers(0, 4))])[: int(rng.integers(1, 5 * page_size))]
            ops.append({"kind": "probe", "ids": ids})
    return ops


def radix_case(out_dir):
    """Runs ``radix_ops`` through ``loopsgl.kvcache.radix_cache.RadixPrefixCache`` on the
    CPU (its node timestamps drawn from a counter instead of the wall clock, its key
    comparison from numpy: both order-preserving) and records every result: match and
    insert lengths, matched indices, evicted indices in eviction order, size totals."""
    import json

    import loopsgl.core as core
    import loopsgl.kernel as lk
    import loopsgl.kvcache.radix_cache as rc

    tick = iter(range(1, 1 << 62))
    rc.time = type("Clock", (), {"monotonic_ns": staticmethod(lambda: next(tick))})

    def compare(a, b):
        n = min(len(a), len(b))
        d = np.flatnonzero(a[:n].numpy() != b[:n].numpy())
        return int(d[0]) if d.size else n

    lk.fast_compare_key = compare

    def indices(h):  # the reference's callers read a handle only when it holds a prefix
        return h.get_matched_indices() if h.cached_len else torch.empty(0, dtype=torch.int32)

    cases = []
    for page_size, seed in ((1, 5), (4, 6)):
        old = core._GLOBAL_CTX
        core._GLOBAL_CTX = None
        core.set_global_ctx(core.Context(page_size=page_size))
        cache = rc.RadixPrefixCache(torch.device("cpu"))
        ops = radix_ops(page_size, seed)
        handles = {}
        for i, op in enumerate(ops):
            if op["kind"] == "request":
                ids = torch.tensor(op["ids"], dtype=torch.int32)
                m = cache.match_prefix(ids).cuda_handle
                cache.lock_handle(m)
                matched = indices(m)
                loc = torch.cat([matched, torch.tensor(op["fresh"][m.cached_len:len(op["ids"])],
                                                       dtype=torch.int32)])
                ins = cache.insert_prefix(ids, loc)
                cache.lock_handle(m, unlock=True)  # the order of CacheManager.cache_req
                cache.lock_handle(ins.handle)
                handles[i] = ins.handle
                op["want"] = {"match_len": m.cached_len, "matched": matched.tolist(),
                              "cached_len": ins.cached_len, "insert_len": ins.handle.cached_len,
                              "inserted": indices(ins.handle).tolist()}
            elif op["kind"] == "finish":
                cache.lock_handle(handles.pop(op["ref"]), unlock=True)
                op["want"] = {}
            elif op["kind"] == "evict":
                size = int(op["frac"] * cache.size_info.evictable_size)
                op["size"] = size
                op["want"] = {"evicted": cache.evict(size).tolist()}
            else:
                h = cache.match_prefix(torch.tensor(op["ids"], dtype=torch.int32)).cuda_handle
                op["want"] = {"match_len": h.cached_len, "matched": indices(h).tolist()}
            info = cache.size_info
            op["want"]["size_info"] = [info.evictable_size, info.protected_size]
        cases.append({"page_size": page_size, "seed": seed, "ops": ops})
        core._GLOBAL_CTX = old
    with open(out_dir / "radix.json", "w") as f:
        json.dump({"cases": cases}, f, separators=(",", ":"))
    print("wrote radix")


# ---------------------------------------------------------------------------
# Retraction snapshots of both KV pools through the reference's own pools
# ---------------------------------------------------------------------------


def kv_snapshot_case(out_dir):
    """``MHAKVCache`` and ``LastExitedKVCache`` (fp32, CPU) filled with seeded values:
    the snapshot ``get_cpu_copy`` takes of some tokens, and the pool state after
    ``load_cpu_copy`` restores it at other tokens of a fresh (zeroed) pool -- for the
    last-exited pool after ``reserve_restore_versions`` with the snapshot's depths, and
    with tokens that exited at different depths (aliased versions) in the snapshot."""
    from loopsgl.kvcache.last_exited import LastExitedKVCache
    from loopsgl.kvcache.mha_pool import MHAKVCache

    g = torch.Generator().manual_seed(17)
    rec = {}
    # paged pool: 3 layers, 6 pages of 4, 2 heads x 8
    mha = MHAKVCache(2, 3, 8, 6, 4, torch.float32, torch.device("cpu"))
    mha._kv_buffer.copy_(torch.randn(mha._kv_buffer.shape, generator=g))
    mha._kv_buffer[:, :, 0].zero_()
    src = torch.tensor([5, 6, 7, 12, 13, 21, 4], dtype=torch.int32)
    dst = torch.tensor([8, 9, 10, 16, 17, 18, 23], dtype=torch.int32)
    rec["mha_pool"] = mha._kv_buffer.numpy().copy()
    rec["mha_src"], rec["mha_dst"] = src.numpy(), dst.numpy()
    snap = mha.get_cpu_copy(src)
    rec["mha_snapshot"] = snap.numpy().copy()
    fresh = MHAKVCache(2, 3, 8, 6, 4, torch.float32, torch.device("cpu"))
    fresh._kv_buffer.zero_()
    fresh.load_cpu_copy(snap, dst)
    rec["mha_restored"] = fresh._kv_buffer.numpy().copy()

    # last-exited pool: 6 layers, core [1, 5), 3 loop steps (2 layers per slot)
    def pool():
        p = LastExitedKVCache(2, 6, 8, 20, 1, torch.float32, torch.device("cpu"), 1, 5, 3)
        p._kv_buffer.zero_()
        return p

    le = pool()
    handles = torch.arange(1, 7, dtype=torch.int32)
    le.reserve_versions(handles)
    le._kv_buffer.copy_(torch.randn(le._kv_buffer.shape, generator=g))
    le._kv_buffer[:, :, 0].zero_()
    exits = torch.tensor([1, 3, 2, 3, 1, 2], dtype=torch.int32)
    le.alias_versions(handles, exits, int((3 - exits).sum()))
    rec["le_pool"] = le._kv_buffer.numpy().copy()
    rec["le_slot_map"] = le.slot_map.numpy().copy()
    rec["le_completed"] = le.completed_depth.numpy().copy()
    src = torch.tensor([2, 5, 1, 6, 3], dtype=torch.int32)
    snap = le.get_cpu_copy(src)
    rec["le_src"], rec["le_snapshot"] = src.numpy(), snap.numpy().copy()
    fresh = pool()
    dst = torch.tensor([4, 9, 2, 11, 7], dtype=torch.int32)
    rec["le_dst"] = dst.numpy()
    rec["le_released"] = np.array(fresh.reserve_restore_versions(dst, snap))
    fresh.load_cpu_copy(snap, dst)
    rec["le_restored"] = fresh._kv_buffer.numpy().copy()
    rec["le_restored_slot_map"] = fresh.slot_map.numpy().copy()
    rec["le_restored_completed"] = fresh.completed_depth.numpy().copy()
    rec["le_restored_free_count"] = fresh._free_count.numpy().copy()
    np.savez_compressed(out_dir / "kv_snapshot.npz", **rec)
    print("wrote kv_snapshot")


# ---------------------------------------------------------------------------
# the tiny Ouro model the reference runs on the CPU
# ---------------------------------------------------------------------------

C1 = LoopedConfig(arch="ouro", hidden=512, heads=8, kv_heads=8, head_dim=64, intermediate=1408,
                  vocab=32000, num_core_layers=4, loop_steps=4, rope_theta=10000.0,
                  max_position=512)


def c1_case(out_dir, decode_steps=32, seed=7):
    """configs[0] through the reference model on the CPU in fp32: 4 requests with prompts
    of 128 uniform-random ids, one prefill, then 32 greedy decode steps at full depth over
    depth-indexed KV in 16-token pages. Records every step's batch metadata and input ids,
    the greedy tokens with their top-2 logit margins, and the full logits of the prefill
    and of the last step (the other steps' logits are not kept: 0.5 MB each)."""
    weights = make_weights(C1, seed, dtype=torch.float32, gate_bias=0.0)
    run = RefRun(C1, weights, "depth_indexed", 16, num_pages=64, max_reqs=8, max_len=192)
    prompts = np.random.default_rng(seed).integers(0, C1.vocab, (4, 128)).astype(np.int32)
    rows = [1, 2, 3, 4]
    for r in rows:
        run.allocate(r, prompts.shape[1])
    ids = torch.from_numpy(prompts.reshape(-1).copy())
    fb, logits = run.run(run.batch(rows, [prompts.shape[1]] * 4, "prefill"), ids)
    rec: dict[str, np.ndarray] = {"seed": np.array(seed), "page_size": np.array(16),
                                  "prefill_ids": ids.numpy(), "prefill_logits": logits.numpy()}
    for k, v in snapshot_meta(fb).items():
        rec[f"prefill_{k}"] = v

    def top2(lg):
        v = torch.topk(lg, 2, dim=-1).values
        return torch.argmax(lg, dim=-1).to(torch.int32), (v[:, 0] - v[:, 1]).numpy()

    tokens, margin = top2(logits)
    all_tokens, margins = [tokens.numpy()], [margin]
    for step in range(decode_steps):
        for r in rows:
            run.allocate(r, run.seq_lens[r] + 1)
        fb, logits = run.run(run.batch(rows, [1] * 4, "decode"), tokens)
        rec[f"step{step}_ids"] = tokens.numpy()
        for k, v in snapshot_meta(fb).items():
            rec[f"step{step}_{k}"] = v
        tokens, margin = top2(logits)
        all_tokens.append(tokens.numpy())
        margins.append(margin)
    rec["last_logits"] = logits.numpy()
    rec["tokens"] = np.stack(all_tokens)
    rec["margins"] = np.stack(margins).astype(np.float32)
    np.savez_compressed(out_dir / "c1_ouro_tiny.npz", **rec)
    print(f"wrote c1_ouro_tiny: {decode_steps} decode steps")


OURO_TINY = LoopedConfig(arch="ouro", hidden=128, heads=4, kv_heads=4, head_dim=32,
                         intermediate=256, vocab=512, num_core_layers=2, loop_steps=3,
                         rope_theta=10000.0, max_position=256)
OURO_TINY_GATED = LoopedConfig(**{**OURO_TINY.__dict__, "exit_threshold": 0.5})
HUGINN_TINY = LoopedConfig(arch="huginn", hidden=96, heads=3, kv_heads=3, head_dim=32,
                           intermediate=192, vocab=384, num_prelude_layers=1, num_core_layers=2,
                           num_coda_layers=1, loop_steps=3, rope_theta=50000.0, max_position=256,
                           embed_scale=1.5, attention_bias=True, adapter_bias=True,
                           exit_threshold=0.8)
PROMPTS = [[5, 17, 3, 99, 42], [7] * 3 + [250, 11, 12, 13, 14, 15], [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12]]


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--reference", required=True, type=Path,
                    help="the reference checkout's python/ directory (holds loopsgl/)")
    ap.add_argument("--out", type=Path, default=HERE)
    args = ap.parse_args()
    install_reference(args.reference)
    torch.set_num_threads(4)
    out = args.out
    metadata_case(out)
    store_case(out)
    tp_shard_case(out)
    radix_case(out)
    kv_snapshot_case(out)
    c1_case(out)
    last_exited_case("last_exited_huginn_layout", 8, 2, 6, 3, 12, out)
    last_exited_case("last_exited_ouro_layout", 6, 0, 6, 4, 24, out)
    model_case("ouro_cb_depth_indexed", OURO_TINY, "depth_indexed", 1, PROMPTS, 3, 4, out)
    model_case("ouro_cb_shared", OURO_TINY, "shared", 1, PROMPTS, 3, 4, out)
    model_case("ouro_cb_last_exited", OURO_TINY, "last_exited", 1, PROMPTS, 2, 1, out)
    model_case("huginn_cb_shared", HUGINN_TINY, "shared", 2, PROMPTS, 2, 4, out)
    plan = [[0, 0, 0], [1, 1, None], [2, None, 1], [None, 2, 2]]
    cdb_case("ouro_cdb_last_exited", OURO_TINY_GATED, "last_exited", 3, PROMPTS, plan, out)
    cdb_case("ouro_cdb_shared", OURO_TINY_GATED, "shared", 3, PROMPTS, plan, out)
    cdb_case("huginn_cdb_last_exited", HUGINN_TINY, "last_exited", 4, PROMPTS, plan, out)


if __name__ == "__main__":
    main()
