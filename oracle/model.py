"""Ouro and Huginn looped decoders restated on the CPU over a paged KV pool.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

The layer and step structure follows ``python/loopsgl/models/looped/{base,ouro,huginn}.py``
and ``models/utils.py`` line by line; every operator comes from ``oracle.ops``
and every index from ``oracle.kvmeta``. Weights use the reference's state-dict
names (``models/weight.py`` merges q/k/v into ``qkv_proj`` and gate/up into
``gate_up_proj``), so a weight dict made here loads into the reference model
and into the CUDA path unchanged.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

from . import kvmeta, ops

__all__ = ["LoopedConfig", "make_weights", "Batch", "PagedKVPool", "SlotKVPool", "LoopedModel"]


@dataclass(frozen=True)
class LoopedConfig:
    """Shape of a looped decoder (the subset of ``ModelConfig`` the hot path reads)."""

    arch: str  # "ouro" | "huginn"
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    num_core_layers: int
    num_prelude_layers: int = 0
    num_coda_layers: int = 0
    loop_steps: int = 4
    rope_theta: float = 1e6
    rms_eps: float = 1e-6
    max_position: int = 8192
    exit_threshold: float | None = None
    min_loop_steps: int = 1
    exit_gate_type: str = "early_exit"
    embed_scale: float = 1.0
    attention_bias: bool = False
    adapter_bias: bool = False
    tie_word_embeddings: bool = False

    @property
    def num_layers(self) -> int:
        return self.num_prelude_layers + self.num_core_layers + self.num_coda_layers

    @property
    def qkv_out(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim

    def layer_names(self) -> list[str]:
        """State-dict prefixes of every decoder layer, in execution order."""
        if self.arch == "ouro":
            return [f"model.layers.{i}" for i in range(self.num_core_layers)]
        return (
            [f"model.prelude.{i}" for i in range(self.num_prelude_layers)]
            + [f"model.layers.{i}" for i in range(self.num_core_layers)]
            + [f"model.coda.{i}" for i in range(self.num_coda_layers)]
        )


NORM_NAMES = (
    "input_layernorm",
    "input_layernorm_2",
    "post_attention_layernorm",
    "post_attention_layernorm_2",
)


def make_weights(
    cfg: LoopedConfig,
    seed: int,
    dtype: torch.dtype = torch.bfloat16,
    std: float = 0.02,
    norm_jitter: float = 0.05,
    gate_bias: float = 0.0,
) -> dict[str, torch.Tensor]:
    """Seeded random-init weights under the reference's state-dict keys.

    Matrices ``N(0, std)``; norm weights ``1 + N(0, norm_jitter)``; exit-gate bias
    ``gate_bias``. Generated in fp32 on the CPU from ``torch.Generator(seed)`` in a
    fixed key order, then cast to ``dtype``.
    """
    g = torch.Generator().manual_seed(seed)
    w: dict[str, torch.Tensor] = {}

    def mat(name: str, *shape: int) -> None:
        w[name] = (torch.randn(*shape, generator=g) * std).to(dtype)

    def norm(name: str, n: int) -> None:
        w[name] = (1.0 + torch.randn(n, generator=g) * norm_jitter).to(dtype)

    h, i = cfg.hidden, cfg.intermediate
    mat("model.embed_tokens.weight", cfg.vocab, h)
    for p in cfg.layer_names():
        mat(f"{p}.self_attn.qkv_proj.weight", cfg.qkv_out, h)
        if cfg.attention_bias:
            mat(f"{p}.self_attn.qkv_proj.bias", cfg.qkv_out)
        mat(f"{p}.self_attn.o_proj.weight", h, cfg.heads * cfg.head_dim)
        mat(f"{p}.mlp.gate_up_proj.weight", 2 * i, h)
        mat(f"{p}.mlp.down_proj.weight", h, i)
        for n in NORM_NAMES:
            norm(f"{p}.{n}.weight", h)
    norm("model.norm.weight", h)
    if cfg.arch == "ouro":
        mat("model.early_exit_gate.weight", 1, h)
        w["model.early_exit_gate.bias"] = torch.full((1,), gate_bias).to(dtype)
    else:
        mat("model.adapter.weight", h, 2 * h)
        if cfg.adapter_bias:
            mat("model.adapter.bias", h)
    if not cfg.tie_word_embeddings:
        mat("lm_head.weight", cfg.vocab, h)
    return w


LINEAR_SUFFIXES = ("qkv_proj.weight", "o_proj.weight", "gate_up_proj.weight",
                   "down_proj.weight", "adapter.weight", "lm_head.weight")


def with_fp32_matrices(weights: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """The same weights with every ``ops.linear`` matrix held in fp32.

    bf16 values are exact in fp32 and ``ops.linear`` computes in fp32 and rounds to the
    activation's dtype, so results are bit-identical; only the per-call conversion of the
    matrix is saved (full-size models: several GB per step). Embedding and norm weights
    keep their dtype (they set the dtype of the rows they produce).
    """
    return {k: (v.float() if k.endswith(LINEAR_SUFFIXES) else v) for k, v in weights.items()}


@dataclass
class Batch:
    """The fields of ``ForwardBatch`` + attention metadata the hot path consumes
    (``core.py:217-252``, ``attention/fa.py:26-41``)."""

    input_ids: torch.Tensor  # [T] int32
    positions: torch.Tensor  # [T] int32
    out_loc: torch.Tensor  # [T] int32 token locations (page*page_size + offset)
    page_table: torch.Tensor  # [B, max_pages] int32 page ids (page_size 1: token handles)
    cache_seqlens: torch.Tensor  # [B] int32
    cu_seqlens_q: torch.Tensor  # [B+1] int32
    is_prefill: bool
    # last-exited only: physical tables per layer group, resolved per core step
    core_page_table: torch.Tensor | None = None
    core_out_loc: torch.Tensor | None = None
    fixed_page_table: torch.Tensor | None = None
    fixed_out_loc: torch.Tensor | None = None

    @property
    def size(self) -> int:
        return self.cache_seqlens.numel()

    def last_indices(self) -> torch.Tensor:
        """``get_last_indices`` (``attention/fa.py:40-41``)."""
        return (self.cu_seqlens_q[1:] - 1).long()


class PagedKVPool:
    """``MHAKVCache`` layout ``[2, L, pages, page, Hkv, D]`` (``kvcache/mha_pool.py:16-66``)."""

    def __init__(self, num_layers, num_pages, page_size, kv_heads, head_dim, dtype):
        self.buf = torch.zeros(2, num_layers, num_pages, page_size, kv_heads, head_dim, dtype=dtype)
        self.page_size = page_size

    def k_cache(self, layer: int) -> torch.Tensor:
        return self.buf[0, layer]

    def v_cache(self, layer: int) -> torch.Tensor:
        return self.buf[1, layer]

    def store(self, layer, k, v, out_loc) -> None:
        kc = self.buf[0, layer].view(-1, *self.buf.shape[-2:])
        vc = self.buf[1, layer].view(-1, *self.buf.shape[-2:])
        ops.store_kv(kc, vc, out_loc, k, v)


class SlotKVPool:
    """``LastExitedKVCache`` storage ``[2, layers_per_slot, slots, Hkv, D]`` and version maps
    (``kvcache/last_exited.py:87-311``); page size 1."""

    def __init__(self, layout: kvmeta.LastExitedLayout, num_pages, kv_heads, head_dim, dtype):
        self.layout = layout
        self.versions = kvmeta.LastExitedVersions(layout, num_pages)
        self.buf = torch.zeros(2, layout.layers_per_slot, self.versions.num_kv_slots, kv_heads,
                               head_dim, dtype=dtype)
        self.page_size = 1

    def k_cache(self, layer: int) -> torch.Tensor:
        _, lane = self.layout.group_and_lane(layer)
        return self.buf[0, lane].unsqueeze(1)

    def v_cache(self, layer: int) -> torch.Tensor:
        _, lane = self.layout.group_and_lane(layer)
        return self.buf[1, lane].unsqueeze(1)

    def store(self, layer, k, v, out_loc) -> None:
        _, lane = self.layout.group_and_lane(layer)
        ops.store_kv(self.buf[0, lane], self.buf[1, lane], out_loc, k, v)


@dataclass
class LoopedModel:
    """A looped decoder over a KV pool under one looped-KV policy."""

    cfg: LoopedConfig
    weights: dict[str, torch.Tensor]
    policy: str = "depth_indexed"
    # tensor-parallel ranks whose rounding points the row-parallel linears reproduce
    tp: int = 1
    cos_sin: torch.Tensor = field(init=False)

    def __post_init__(self) -> None:
        self.cos_sin = ops.rope_cos_sin_cache(self.cfg.head_dim, self.cfg.max_position,
                                              self.cfg.rope_theta)
        self.scale = ops.softmax_scale(self.cfg.head_dim)

    # -- KV layer indices (base.py:59-91) ----------------------------------
    @property
    def num_kv_layers(self) -> int:
        c = self.cfg
        return kvmeta.num_kv_layers(self.policy, c.loop_steps, c.num_prelude_layers,
                                    c.num_core_layers, c.num_coda_layers)

    def slot_layout(self) -> kvmeta.LastExitedLayout:
        c = self.cfg
        return kvmeta.LastExitedLayout(self.num_kv_layers, c.num_prelude_layers,
                                       c.num_prelude_layers + c.num_core_layers, c.loop_steps)

    # -- sublayers -------------------------------------------------------------
    def _w(self, name: str) -> torch.Tensor:
        return self.weights[name]

    def _row_parallel(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """``LinearOProj`` / ``LinearRowParallel`` over ``tp`` ranks (layers/linear.py:92-128
        with distributed/impl.py:63-70): rank r's ``F.linear`` over its contiguous slice of
        the input features is rounded to the working dtype, then the ranks' outputs are
        summed -- in rank order in fp32 and rounded once, which is NCCL's result for two
        ranks and the order of this repository's fused all-reduce for any number."""
        if self.tp == 1:
            return ops.linear(x, w)
        k = x.shape[-1] // self.tp
        acc = torch.zeros(x.shape[0], w.shape[0], dtype=torch.float32)
        for r in range(self.tp):
            acc += ops.linear(x[:, r * k:(r + 1) * k], w[:, r * k:(r + 1) * k]).float()
        return acc.to(x.dtype)

    def attention(self, p: str, x: torch.Tensor, cache_layer: int, batch: Batch, pool,
                  depth) -> torch.Tensor:
        """``RopeAttn.forward`` + ``AttentionLayer.forward`` (models/utils.py:119-131,
        layers/attention.py:77-100); Huginn rounds before its QKV bias (huginn.py:44-47)."""
        c = self.cfg
        wq = self._w(f"{p}.self_attn.qkv_proj.weight")
        bq = self.weights.get(f"{p}.self_attn.qkv_proj.bias")
        if c.arch == "huginn":
            qkv = ops.linear_bias_after_rounding(x, wq, bq)
        else:
            qkv = ops.linear(x, wq, bq)
        qd, kd = c.heads * c.head_dim, c.kv_heads * c.head_dim
        q = qkv[:, :qd].reshape(-1, c.heads, c.head_dim)
        k = qkv[:, qd:qd + kd].reshape(-1, c.kv_heads, c.head_dim)
        v = qkv[:, qd + kd:].reshape(-1, c.kv_heads, c.head_dim)
        q = ops.apply_rope_neox(batch.positions, q, self.cos_sin)
        k = ops.apply_rope_neox(batch.positions, k, self.cos_sin)
        out_loc, table = batch.out_loc, batch.page_table
        if isinstance(pool, SlotKVPool):
            group, _ = pool.layout.group_and_lane(cache_layer)
            lay = pool.layout
            core = lay.core_start <= cache_layer < lay.core_end
            if core:
                out_loc, table = batch.core_out_loc[group], batch.core_page_table[group]
            else:
                out_loc, table = batch.fixed_out_loc[group], batch.fixed_page_table[group]
        pool.store(cache_layer, k, v, out_loc)
        o = ops.paged_attention(q, pool.k_cache(cache_layer), pool.v_cache(cache_layer), table,
                                batch.cache_seqlens, batch.cu_seqlens_q, self.scale)
        return self._row_parallel(o.reshape(-1, qd), self._w(f"{p}.self_attn.o_proj.weight"))

    def mlp(self, p: str, x: torch.Tensor) -> torch.Tensor:
        """``GatedMLP.forward`` (models/utils.py:45-50): gate_up rows are ``[gate; up]``."""
        gu = ops.linear(x, self._w(f"{p}.mlp.gate_up_proj.weight"))
        return self._row_parallel(ops.silu_and_mul(gu), self._w(f"{p}.mlp.down_proj.weight"))

    def ouro_layer(self, p, x, residual, cache_layer, batch, pool, depth):
        """``OuroDecoderLayer.forward`` (ouro.py:37-53), the sandwich-norm layer."""
        eps = self.cfg.rms_eps
        x, residual = ops.rms_norm_fused(x, residual, self._w(f"{p}.input_layernorm.weight"), eps)
        x = self.attention(p, x, cache_layer, batch, pool, depth)
        x = ops.rmsnorm(x, self._w(f"{p}.input_layernorm_2.weight"), eps)
        x, residual = ops.fused_add_rmsnorm(x, residual,
                                            self._w(f"{p}.post_attention_layernorm.weight"), eps)
        x = self.mlp(p, x)
        x = ops.rmsnorm(x, self._w(f"{p}.post_attention_layernorm_2.weight"), eps)
        return x, residual

    def huginn_layer(self, p, x, cache_layer, batch, pool, depth):
        """``HuginnDecoderLayer.forward`` (huginn.py:66-83)."""
        eps = self.cfg.rms_eps
        residual = x
        x = ops.rmsnorm(x, self._w(f"{p}.input_layernorm.weight"), eps)
        x = self.attention(p, x, cache_layer, batch, pool, depth)
        x = ops.fused_add_rmsnorm(x, residual, self._w(f"{p}.input_layernorm_2.weight"), eps)[0]
        residual = x
        x = ops.rmsnorm(x, self._w(f"{p}.post_attention_layernorm.weight"), eps)
        x = self.mlp(p, x)
        return ops.fused_add_rmsnorm(x, residual,
                                     self._w(f"{p}.post_attention_layernorm_2.weight"), eps)[0]

    # -- phases (base.py:104-156) ------------------------------------------
    def forward_prelude(self, batch: Batch, pool):
        c = self.cfg
        emb = ops.embedding(batch.input_ids, self._w("model.embed_tokens.weight"))
        if c.arch == "ouro":
            return emb, None  # ouro.py:117
        inj = (emb.float() * c.embed_scale).to(emb.dtype)  # huginn.py:146-160
        for i in range(c.num_prelude_layers):
            inj = self.huginn_layer(f"model.prelude.{i}", inj, kvmeta.prelude_cache_layer_index(i),
                                    batch, pool, None)
        return torch.zeros_like(inj), inj

    def core_step(self, hidden, loop_step, injection, batch: Batch, pool):
        """One loop step over the shared block (ouro.py:119-136, huginn.py:162-178).

        ``loop_step`` is an int (CB) or a per-row int tensor (CDB); under last-exited
        the caller resolves ``batch.core_*`` tables at the rows' depths first.
        """
        c = self.cfg
        step = loop_step if isinstance(loop_step, int) else None
        if c.arch == "ouro":
            x, residual = hidden, None
            for i in range(c.num_core_layers):
                layer = self._core_layer(i, step)
                x, residual = self.ouro_layer(f"model.layers.{i}", x, residual, layer, batch, pool,
                                              loop_step)
            return ops.fused_add_rmsnorm(x, residual, self._w("model.norm.weight"), c.rms_eps)[0]
        x = ops.linear(torch.cat([hidden, injection], dim=-1), self._w("model.adapter.weight"),
                       self.weights.get("model.adapter.bias"))
        for i in range(c.num_core_layers):
            x = self.huginn_layer(f"model.layers.{i}", x, self._core_layer(i, step), batch, pool,
                                  loop_step)
        return x

    def _core_layer(self, i: int, step) -> int:
        c = self.cfg
        return kvmeta.core_cache_layer_index(self.policy, c.num_prelude_layers, c.num_core_layers,
                                             i, step if step is not None else 0)

    def forward_coda(self, hidden, batch: Batch, pool):
        c = self.cfg
        if c.arch == "ouro":
            return hidden  # ouro.py:161-162
        x = ops.rmsnorm(hidden, self._w("model.norm.weight"), c.rms_eps)  # huginn.py:196-201
        for i in range(c.num_coda_layers):
            layer = kvmeta.coda_cache_layer_index(self.policy, c.loop_steps, c.num_prelude_layers,
                                                  c.num_core_layers, c.num_coda_layers, i)
            x = self.huginn_layer(f"model.coda.{i}", x, layer, batch, pool, None)
        return ops.rmsnorm(x, self._w("model.norm.weight"), c.rms_eps)

    def lm_head(self, hidden, batch: Batch | None):
        """``ParallelLMHead.forward`` at TP=1 (layers/embedding.py:89-111)."""
        if batch is not None and batch.is_prefill:
            hidden = hidden[batch.last_indices()]
        w = self._w("model.embed_tokens.weight" if self.cfg.tie_word_embeddings else "lm_head.weight")
        return ops.linear(hidden, w)

    def init_exit_state(self, hidden):
        """ouro.py:138-140 (zeros, fp32) / huginn.py:180-182 (the state itself)."""
        if self.cfg.arch == "ouro":
            return torch.zeros(hidden.shape[0], dtype=torch.float32)
        return hidden

    def exit_signal(self, hidden, exit_state, loop_step):
        c = self.cfg
        if c.arch == "ouro":
            return ops.ouro_exit_signal(hidden, exit_state, loop_step,
                                        self._w("model.early_exit_gate.weight"),
                                        self._w("model.early_exit_gate.bias"), c.exit_threshold,
                                        c.min_loop_steps, c.exit_gate_type == "lookahead")
        return ops.huginn_exit_signal(hidden, exit_state, c.exit_threshold)

    def forward(self, batch: Batch, pool) -> torch.Tensor:
        """Full-depth pass (base.py:148-164): prelude, every loop step, coda, LM head."""
        if isinstance(pool, SlotKVPool):
            self.resolve_fixed(batch, pool)
        h, inj = self.forward_prelude(batch, pool)
        for step in range(self.cfg.loop_steps):
            if isinstance(pool, SlotKVPool):
                self.resolve_core(batch, pool, step)
            h = self.core_step(h, step, inj, batch, pool)
        return self.lm_head(self.forward_coda(h, batch, pool), batch)

    # -- last-exited address resolution (attention/fa.py:95-157) -----------
    def resolve_core(self, batch: Batch, pool: SlotKVPool, depths) -> None:
        vmap = pool.versions.version_map
        d = depths if isinstance(depths, int) else np.asarray(depths)
        table, out = kvmeta.resolve_last_exited(
            batch.page_table.numpy(), vmap, batch.cache_seqlens.numpy(),
            batch.cu_seqlens_q.numpy(), batch.out_loc.numpy(), d)
        batch.core_page_table = torch.from_numpy(table)
        batch.core_out_loc = torch.from_numpy(out)

    def resolve_fixed(self, batch: Batch, pool: SlotKVPool) -> None:
        if pool.layout.fixed_groups == 0:
            return
        table, out = kvmeta.resolve_last_exited(
            batch.page_table.numpy(), pool.versions.fixed_map, batch.cache_seqlens.numpy(),
            batch.cu_seqlens_q.numpy(), batch.out_loc.numpy(), 0)
        batch.fixed_page_table = torch.from_numpy(table)
        batch.fixed_out_loc = torch.from_numpy(out)
