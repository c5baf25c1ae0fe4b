"""Ouro and Huginn looped decoders on the B200 kernels.

Follows the layer and step structure of python/loopsgl/models/looped/{base,ouro,
huginn}.py and models/utils.py, with these fusions:

* Ouro's two back-to-back norms at every layer boundary (``input_layernorm_2``
  then ``post_attention_layernorm``; ``post_attention_layernorm_2`` then the next
  layer's ``input_layernorm``) are one ``sandwich_norm`` launch;
* the step's last sandwich, the final ``norm``, the exit gate and the CDB state
  scatter are one ``ouro_step_exit`` launch (one per loop step);
* RoPE and the KV store are one launch writing straight into the paged pool;
* gate_up + SiLU*mul is one GEMM with a SwiGLU epilogue (weights interleaved once
  at load).

Every launch goes through ``ops`` to ``libloopsgl_b200.so``; the per-step work
has no host synchronisation and can be captured in a CUDA graph.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import ops
from .kvcache import LastExitedKVCache, MHAKVCache

BF16 = torch.bfloat16


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
        if self.arch == "ouro":
            return [f"model.layers.{i}" for i in range(self.num_core_layers)]
        return ([f"model.prelude.{i}" for i in range(self.num_prelude_layers)]
                + [f"model.layers.{i}" for i in range(self.num_core_layers)]
                + [f"model.coda.{i}" for i in range(self.num_coda_layers)])


def num_kv_layers(policy: str, cfg: LoopedConfig) -> int:
    """``BaseLoopedModel.num_kv_layers`` (models/looped/base.py:59-71)."""
    slots = cfg.loop_steps if policy == "depth_indexed" else 1
    return cfg.num_prelude_layers + slots * cfg.num_core_layers + cfg.num_coda_layers


def core_cache_layer_index(policy: str, cfg: LoopedConfig, layer_id: int, loop_step) -> int:
    """base.py:76-88; depth-indexed needs a scalar step."""
    if policy == "depth_indexed":
        if not isinstance(loop_step, int):
            raise ValueError("Depth-indexed KV requires a scalar loop step")
        return cfg.num_prelude_layers + loop_step * cfg.num_core_layers + layer_id
    return cfg.num_prelude_layers + layer_id


def coda_cache_layer_index(policy: str, cfg: LoopedConfig, layer_id: int) -> int:
    """base.py:90-91."""
    return num_kv_layers(policy, cfg) - cfg.num_coda_layers + layer_id


def rope_cos_sin_cache(head_dim: int, max_position: int, base: float,
                       device: torch.device) -> torch.Tensor:
    """fp32 ``cat(cos, sin)`` table built as layers/rotary.py:26-34 does, on ``device``."""
    with torch.device(device):
        inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
        t = torch.arange(max_position, dtype=torch.float)
        freqs = torch.einsum("i,j -> ij", t, inv_freq)
        return torch.cat((freqs.cos(), freqs.sin()), dim=-1).contiguous()


@dataclass
class DeviceBatch:
    """The ``ForwardBatch`` fields + attention metadata the hot path reads (core.py:217-252,
    attention/fa.py:26-41), as int32 device tensors."""

    input_ids: torch.Tensor
    positions: torch.Tensor
    out_loc: torch.Tensor
    page_table: torch.Tensor  # [B, cols] page ids (page size 1: token handles)
    cache_seqlens: torch.Tensor  # [B]
    cu_seqlens_q: torch.Tensor  # [B+1]
    is_prefill: bool
    max_seqlen: int
    core_page_table: torch.Tensor | None = None  # [groups, B, cols] (last-exited)
    core_out_loc: torch.Tensor | None = None  # [groups, T]
    fixed_page_table: torch.Tensor | None = None
    fixed_out_loc: torch.Tensor | None = None
    last_indices: torch.Tensor | None = field(default=None)  # int64 [B] for prefill LM head
    # decode rows whose page tables start with the same pages (prefix_cache.SharedPrefixGroups):
    # attention reads each group's shared prefix once for all of its rows
    prefix_groups: object | None = None

    @property
    def size(self) -> int:
        return self.cache_seqlens.numel()

    @property
    def num_tokens(self) -> int:
        return self.input_ids.numel()


@dataclass
class _Layer:
    qkv: torch.Tensor
    qkv_bias: torch.Tensor | None
    o: torch.Tensor
    gate_up: torch.Tensor  # interleaved for the SwiGLU epilogue
    down: torch.Tensor
    norms: list[torch.Tensor]  # input, input_2, post_attention, post_attention_2


def shard_weights(cfg: LoopedConfig, weights: dict[str, torch.Tensor], rank: int,
                  world: int) -> dict[str, torch.Tensor]:
    """This rank's tensor-parallel shard of a full state dict with merged ``qkv_proj`` and
    ``gate_up_proj``, as the reference's loader splits (models/weight.py:38-56) and merges
    (:106-115) it: q/k/v and gate/up rows chunked per rank (k/v replicated when there are
    fewer KV heads than ranks), o_proj/down_proj columns chunked, the embedding and LM head
    cut into ceil(V/t)-row vocabulary ranges; everything else replicated. The LM head
    shard is zero-padded to ceil(V/t) rows so every rank's logits gather alike."""
    t, r = world, rank
    if t == 1:
        return dict(weights)
    d = cfg.head_dim

    def rows(x: torch.Tensor) -> torch.Tensor:
        return x.chunk(t, dim=0)[r]

    def kv_rows(x: torch.Tensor) -> torch.Tensor:
        if cfg.kv_heads < t:
            h = r * cfg.kv_heads // t
            return x[h * d:(h + 1) * d]
        return rows(x)

    vocab_local = -(-cfg.vocab // t)
    start = r * vocab_local
    vlen = max(0, min(vocab_local, cfg.vocab - start))
    out: dict[str, torch.Tensor] = {}
    for name, x in weights.items():
        if name.endswith("self_attn.qkv_proj.weight") or name.endswith("self_attn.qkv_proj.bias"):
            q, k, v = x.split([cfg.heads * d, cfg.kv_heads * d, cfg.kv_heads * d], dim=0)
            out[name] = torch.cat([rows(q), kv_rows(k), kv_rows(v)], dim=0).contiguous()
        elif name.endswith("mlp.gate_up_proj.weight"):
            g, u = x.chunk(2, dim=0)
            out[name] = torch.cat([rows(g), rows(u)], dim=0).contiguous()
        elif name.endswith("self_attn.o_proj.weight") or name.endswith("mlp.down_proj.weight"):
            out[name] = x.chunk(t, dim=1)[r].contiguous()
        elif name in ("model.embed_tokens.weight", "lm_head.weight"):
            part = x[start:start + vlen]
            if name == "lm_head.weight" and vlen < vocab_local:
                part = torch.cat([part, part.new_zeros(vocab_local - vlen, x.shape[1])])
            out[name] = part.contiguous()
        else:
            out[name] = x
    if cfg.tie_word_embeddings:  # the head is the embedding's vocabulary range
        part = weights["model.embed_tokens.weight"][start:start + vlen]
        if vlen < vocab_local:
            part = torch.cat([part, part.new_zeros(vocab_local - vlen, part.shape[1])])
        out["lm_head.weight"] = part.contiguous()
    return out


class LoopedDecoder:
    """A looped decoder under one looped-KV policy, weights resident in HBM (bf16)."""

    def __init__(self, cfg: LoopedConfig, weights: dict[str, torch.Tensor], policy: str,
                 device: torch.device | str = "cuda", comm=None) -> None:
        """``weights`` is the full (unsharded) state dict. With a ``comm``
        (``comm.B200Communicator``) this rank keeps its tensor-parallel shard, split as
        the reference's loader does (models/weight.py:38-56): q/k/v and gate/up rows,
        o_proj and down_proj columns, vocabulary rows of the embedding and LM head."""
        if policy not in ("depth_indexed", "shared", "last_exited"):
            raise ValueError(f"unknown looped-KV policy {policy!r}")
        self.cfg, self.policy = cfg, policy
        self.device = torch.device(device)
        self.comm = comm
        self.rank, self.world = (comm.rank, comm.world) if comm is not None else (0, 1)
        t, r = self.world, self.rank
        if t > 1 and (cfg.arch != "ouro" or cfg.heads % t or cfg.intermediate % t):
            raise ValueError(f"{cfg.arch} with {cfg.heads} heads does not shard over {t} ranks "
                             "(Huginn runs as data-parallel replicas)")
        self.hq = cfg.heads // t
        self.hkv = max(cfg.kv_heads // t, 1)
        self.inter = cfg.intermediate // t
        self.vocab_local = -(-cfg.vocab // t)
        self.vocab_start = r * self.vocab_local
        self.vocab_len = max(0, min(self.vocab_local, cfg.vocab - self.vocab_start))
        weights = shard_weights(cfg, weights, r, t)

        def bf(name_or_x) -> torch.Tensor:
            x = weights[name_or_x] if isinstance(name_or_x, str) else name_or_x
            return x.to(device=self.device, dtype=BF16).contiguous()

        def opt(name: str) -> torch.Tensor | None:
            return bf(name) if name in weights else None

        self.layers: dict[str, _Layer] = {}
        for p in cfg.layer_names():
            gu = bf(f"{p}.mlp.gate_up_proj.weight")
            self.layers[p] = _Layer(
                qkv=bf(f"{p}.self_attn.qkv_proj.weight"),
                qkv_bias=opt(f"{p}.self_attn.qkv_proj.bias"),
                o=bf(f"{p}.self_attn.o_proj.weight"),
                gate_up=ops.swiglu_interleave(gu),
                down=bf(f"{p}.mlp.down_proj.weight"),
                norms=[bf(f"{p}.{n}.weight") for n in (
                    "input_layernorm", "input_layernorm_2", "post_attention_layernorm",
                    "post_attention_layernorm_2")],
            )
            del gu
        self.embed = bf("model.embed_tokens.weight")
        if cfg.tie_word_embeddings and t == 1:
            self.lm_head_w = self.embed
        else:
            self.lm_head_w = bf("lm_head.weight")
        self.norm = bf(weights["model.norm.weight"])
        self.gate_w = opt("model.early_exit_gate.weight")
        self.gate_b = opt("model.early_exit_gate.bias")
        self.adapter = opt("model.adapter.weight")
        self.adapter_b = opt("model.adapter.bias")
        self.cos_sin = rope_cos_sin_cache(cfg.head_dim, cfg.max_position, cfg.rope_theta,
                                          self.device)
        self.scale = cfg.head_dim ** -0.5
        self.core_names = [f"model.layers.{i}" for i in range(cfg.num_core_layers)]
        self._pairs: dict[int, torch.Tensor] = {}  # greedy-sampling pairs per row count

    def _row_parallel(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """LinearOProj / LinearRowParallel (layers/linear.py:103-107, 124-128): the local
        GEMM and the all-reduce in one kernel over NVLink when sharded."""
        if self.world > 1:
            return self.comm.gemm_allreduce(x, w)
        return ops.gemm(x, w)

    # ------------------------------------------------------------------ KV --
    @property
    def num_kv_layers(self) -> int:
        return num_kv_layers(self.policy, self.cfg)

    def make_kv_cache(self, num_pages: int, page_size: int, zero: bool = True):
        c = self.cfg
        if self.policy == "last_exited":
            return LastExitedKVCache(self.hkv, self.num_kv_layers, c.head_dim, num_pages,
                                     c.num_prelude_layers,
                                     c.num_prelude_layers + c.num_core_layers, c.loop_steps,
                                     self.device, zero=zero)
        return MHAKVCache(self.hkv, self.num_kv_layers, c.head_dim, num_pages, page_size,
                          self.device, zero=zero)

    def resolve_core(self, batch: DeviceBatch, kv: LastExitedKVCache, depths) -> None:
        """``prepare_core_metadata`` (attention/fa.py:95-108) at the rows' depths."""
        groups = kv.core_groups
        if batch.core_page_table is None:
            batch.core_page_table = torch.zeros(groups, *batch.page_table.shape,
                                                dtype=torch.int32, device=self.device)
            batch.core_out_loc = torch.zeros(groups, batch.num_tokens, dtype=torch.int32,
                                             device=self.device)
        ops.last_exited_resolve(batch.page_table, kv.version_map, batch.cache_seqlens,
                                batch.cu_seqlens_q, batch.out_loc, depths, batch.core_page_table,
                                batch.core_out_loc)

    def resolve_fixed(self, batch: DeviceBatch, kv: LastExitedKVCache) -> None:
        """Fixed-layer tables at depth 0 (attention/fa.py:110-157)."""
        if kv.fixed_groups == 0:
            return
        if batch.fixed_page_table is None:
            batch.fixed_page_table = torch.zeros(kv.fixed_groups, *batch.page_table.shape,
                                                 dtype=torch.int32, device=self.device)
            batch.fixed_out_loc = torch.zeros(kv.fixed_groups, batch.num_tokens,
                                              dtype=torch.int32, device=self.device)
        ops.last_exited_resolve(batch.page_table, kv.fixed_map, batch.cache_seqlens,
                                batch.cu_seqlens_q, batch.out_loc, 0, batch.fixed_page_table,
                                batch.fixed_out_loc)

    # ----------------------------------------------------------- sublayers --
    def _attention(self, lw: _Layer, x: torch.Tensor, cache_layer: int, batch: DeviceBatch, kv,
                   huginn: bool) -> torch.Tensor:
        """RopeAttn + AttentionLayer + backend (models/utils.py:119-131,
        layers/attention.py:77-100, attention/fa.py:68-93)."""
        c = self.cfg
        out_loc, table, page = batch.out_loc, batch.page_table, getattr(kv, "page_size", 1)
        if isinstance(kv, LastExitedKVCache):
            group = kv.layer_groups[cache_layer]
            if kv.is_core_layer(cache_layer):
                out_loc, table = batch.core_out_loc[group], batch.core_page_table[group]
            else:
                out_loc, table = batch.fixed_out_loc[group], batch.fixed_page_table[group]
        kc, vc = kv.slots(cache_layer)
        if lw.qkv_bias is None and c.head_dim == 128:
            # one head per weight tile: RoPE and the KV store run in the GEMM's epilogue
            qkv = ops.gemm_rope_store(x, lw.qkv, batch.positions, self.cos_sin, self.hq,
                                      self.hkv, c.head_dim, kc, vc, out_loc)
        else:
            if lw.qkv_bias is None:
                qkv = ops.gemm(x, lw.qkv)
            else:
                epi = ops.LSB_EPI_BIAS_AFTER_ROUND if huginn else ops.LSB_EPI_BIAS
                qkv = ops.gemm(x, lw.qkv, lw.qkv_bias, epi)
            ops.rope_store_kv(qkv, batch.positions, self.cos_sin, self.hq, self.hkv,
                              c.head_dim, kc, vc, out_loc)
        q = qkv[:, : self.hq * c.head_dim].view(-1, self.hq, c.head_dim)
        if batch.prefix_groups is not None and not batch.is_prefill and table is batch.page_table:
            o = ops.paged_attention_shared_prefix(q, kc, vc, table, batch.cache_seqlens,
                                                  batch.cu_seqlens_q, page, batch.max_seqlen,
                                                  self.scale, self.hkv, batch.prefix_groups)
        else:
            o = ops.paged_attention(q, kc, vc, table, batch.cache_seqlens, batch.cu_seqlens_q,
                                    page, batch.max_seqlen, self.scale, self.hkv)
        return self._row_parallel(o.view(-1, self.hq * c.head_dim), lw.o)

    def _mlp(self, lw: _Layer, x: torch.Tensor) -> torch.Tensor:
        """GatedMLP (models/utils.py:45-50) with the SwiGLU epilogue."""
        return self._row_parallel(ops.gemm(x, lw.gate_up, epilogue=ops.LSB_EPI_SWIGLU), lw.down)

    def _ouro_core(self, hidden: torch.Tensor, loop_step, batch: DeviceBatch, kv):
        """All core layers of one Ouro step up to the last MLP output (ouro.py:119-135).

        Returns ``(d, residual)``; the caller applies the step-end kernel. ``hidden``
        becomes the residual stream and is updated in place, as RMSNormFused does.
        """
        c = self.cfg
        eps = c.rms_eps
        step = loop_step if isinstance(loop_step, int) else None
        residual = hidden
        first = self.layers[self.core_names[0]]
        x = ops.rmsnorm(hidden, first.norms[0], eps)
        d = None
        for i, name in enumerate(self.core_names):
            lw = self.layers[name]
            cache_layer = core_cache_layer_index(self.policy, c, i, step if step is not None else 0)
            a = self._attention(lw, x, cache_layer, batch, kv, huginn=False)
            x = ops.sandwich_norm(a, residual, lw.norms[1], lw.norms[2], eps, out=a)
            d = self._mlp(lw, x)
            if i + 1 < len(self.core_names):
                nxt = self.layers[self.core_names[i + 1]]
                x = ops.sandwich_norm(d, residual, lw.norms[3], nxt.norms[0], eps, out=d)
        return d, residual

    def _huginn_layer(self, lw: _Layer, x: torch.Tensor, cache_layer: int, batch, kv):
        """HuginnDecoderLayer.forward (huginn.py:66-83); ``x`` is overwritten."""
        eps = self.cfg.rms_eps
        h = ops.rmsnorm(x, lw.norms[0], eps)
        a = self._attention(lw, h, cache_layer, batch, kv, huginn=True)
        ops.fused_add_rmsnorm(a, x, lw.norms[1], eps)
        h = ops.rmsnorm(a, lw.norms[2], eps)
        d = self._mlp(lw, h)
        ops.fused_add_rmsnorm(d, a, lw.norms[3], eps)
        return d

    # --------------------------------------------------------------- phases --
    def forward_prelude(self, batch: DeviceBatch, kv):
        """base.py:104-107: Ouro embeds (ouro.py:117); Huginn scales and runs the prelude
        layers, with a zero recurrent state (huginn.py:146-160)."""
        c = self.cfg
        if c.arch == "ouro":
            if self.world == 1:
                return ops.embedding(batch.input_ids, self.embed), None
            # VocabParallelEmbedding (layers/embedding.py:34-43): local rows, zeros elsewhere,
            # summed over the ranks
            h = ops.embedding(batch.input_ids, self.embed, vocab_start=self.vocab_start,
                              vocab_len=self.vocab_len)
            return self.comm.all_reduce(h), None
        inj = ops.embedding(batch.input_ids, self.embed, scale=c.embed_scale)
        for i in range(c.num_prelude_layers):
            inj = self._huginn_layer(self.layers[f"model.prelude.{i}"], inj, i, batch, kv)
        return torch.zeros_like(inj), inj

    def embed_tokens(self, ids: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Ouro's prelude (ouro.py:117): the token embedding, vocab-parallel when sharded
        (layers/embedding.py:34-43)."""
        if self.world == 1:
            return ops.embedding(ids, self.embed, out=out)
        h = ops.embedding(ids, self.embed, vocab_start=self.vocab_start,
                          vocab_len=self.vocab_len, out=out)
        return self.comm.all_reduce(h)

    def core_step(self, hidden: torch.Tensor, loop_step, injection, batch: DeviceBatch, kv,
                  out: torch.Tensor | None = None) -> torch.Tensor:
        """One loop step (ouro.py:119-136, huginn.py:162-178); ``hidden`` may be consumed."""
        c = self.cfg
        if c.arch == "ouro":
            d, residual = self._ouro_core(hidden, loop_step, batch, kv)
            last = self.layers[self.core_names[-1]]
            out = torch.empty_like(d) if out is None else out
            ops.ouro_step_exit(d, residual, last.norms[3], self.norm, c.rms_eps, hidden_out=out)
            return out
        step = loop_step if isinstance(loop_step, int) else None
        # adapter(cat[h, injection]) (huginn.py:162-167): the GEMM's K loop reads both halves
        x = ops.gemm_concat(hidden, injection, self.adapter, self.adapter_b)
        for i, name in enumerate(self.core_names):
            layer = core_cache_layer_index(self.policy, c, i, step if step is not None else 0)
            x = self._huginn_layer(self.layers[name], x, layer, batch, kv)
        if out is not None:
            out.copy_(x)
            return out
        return x

    def core_step_exit(self, state: dict[str, torch.Tensor], slots: torch.Tensor,
                       depths: torch.Tensor, batch: DeviceBatch, kv,
                       signal: torch.Tensor) -> torch.Tensor:
        """``CDBModelRunner._execute_phase("core")`` (cdb_model_runner.py:94-109) fused:
        gather by slot, one loop step at the rows' depths, exit gate, scatter back.
        ``state`` holds "hidden" [cap, H] bf16, "exit" ([cap] fp32 Ouro / [cap, H] bf16
        Huginn) and Huginn's "injection"; ``signal`` receives one uint8 per row."""
        c = self.cfg
        hidden = ops.gather_rows(state["hidden"], slots)
        if isinstance(kv, LastExitedKVCache):
            self.resolve_fixed(batch, kv)
            self.resolve_core(batch, kv, depths)
        if c.arch == "ouro":
            d, residual = self._ouro_core(hidden, None, batch, kv)
            last = self.layers[self.core_names[-1]]
            ops.ouro_step_exit(d, residual, last.norms[3], self.norm, c.rms_eps,
                               hidden_out=state["hidden"], gate_w=self.gate_w,
                               gate_b=self.gate_b, exit_state=state["exit"], signal=signal,
                               slot=slots, depth=depths, threshold=c.exit_threshold,
                               min_loop_steps=c.min_loop_steps,
                               lookahead=c.exit_gate_type == "lookahead")
            return signal
        inj = ops.gather_rows(state["injection"], slots)
        h = self.core_step(hidden, None, inj, batch, kv)
        ops.huginn_step_exit(h, state["exit"], state["hidden"], signal, c.exit_threshold,
                             slot=slots)
        return signal

    def forward_coda(self, hidden: torch.Tensor, batch: DeviceBatch, kv) -> torch.Tensor:
        c = self.cfg
        if c.arch == "ouro":
            return hidden
        x = ops.rmsnorm(hidden, self.norm, c.rms_eps)
        for i in range(c.num_coda_layers):
            layer = coda_cache_layer_index(self.policy, c, i)
            x = self._huginn_layer(self.layers[f"model.coda.{i}"], x, layer, batch, kv)
        return ops.rmsnorm(x, self.norm, c.rms_eps)

    def _lm_rows(self, hidden: torch.Tensor, batch: DeviceBatch | None) -> torch.Tensor:
        if batch is not None and batch.is_prefill:
            idx = batch.last_indices
            if idx is None:
                idx = (batch.cu_seqlens_q[1:] - 1).long()
            hidden = ops.gather_rows(hidden, idx)
        return hidden

    def lm_head(self, hidden: torch.Tensor, batch: DeviceBatch | None) -> torch.Tensor:
        """ParallelLMHead (layers/embedding.py:89-111): logits [B, V] (all-gathered and
        put in vocabulary order when sharded)."""
        logits = ops.gemm(self._lm_rows(hidden, batch), self.lm_head_w)
        if self.world == 1:
            return logits
        g = self.comm.all_gather(logits)  # [t*B, V/t] rank by rank
        bs = logits.shape[0]
        g = g.view(self.world, bs, self.vocab_local).permute(1, 0, 2).reshape(bs, -1)
        return g[:, : self.cfg.vocab]

    def greedy(self, hidden: torch.Tensor, batch: DeviceBatch | None,
               out: torch.Tensor | None = None) -> torch.Tensor:
        """LM head + greedy sampling (embedding.py:89-111, sample.py:108-112) into int32
        ``out``, fused: the LM-head GEMM's epilogue keeps only the best logit of every
        128-entry vocabulary tile per row, so the logits are never written; with shards,
        only those (value, index) pairs are all-gathered over NVLink, then one reduction
        picks each row's token (first index on ties, as torch.argmax)."""
        rows = self._lm_rows(hidden, batch)
        m = rows.shape[0]
        pairs = self._pairs.get(m)
        if pairs is None:  # kept per row count: graph replays reuse the same buffer
            pairs = ops.argmax_pairs_buffer(m, self.vocab_local, rows.device)
            self._pairs[m] = pairs
        ops.gemm_argmax(rows, self.lm_head_w, pairs, n_valid=self.vocab_len)
        tiles = -(-self.vocab_len // 128)
        if self.world > 1:
            pairs = self.comm.all_gather(pairs)
        return ops.argmax_pairs(pairs, self.world, m, tiles, self.vocab_local, out=out)

    def forward(self, batch: DeviceBatch, kv) -> torch.Tensor:
        """Full-depth pass (base.py:148-164)."""
        if isinstance(kv, LastExitedKVCache):
            self.resolve_fixed(batch, kv)
        h, inj = self.forward_prelude(batch, kv)
        for step in range(self.cfg.loop_steps):
            if isinstance(kv, LastExitedKVCache):
                self.resolve_core(batch, kv, step)
            h = self.core_step(h, step, inj, batch, kv)
        return self.lm_head(self.forward_coda(h, batch, kv), batch)

    def init_exit_state(self, hidden: torch.Tensor) -> torch.Tensor:
        """ouro.py:138-140 / huginn.py:180-182."""
        if self.cfg.arch == "ouro":
            return torch.zeros(hidden.shape[0], dtype=torch.float32, device=hidden.device)
        return hidden
