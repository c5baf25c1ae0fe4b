"""Drop-ins with the reference's plugin interfaces, running this project's kernels.

Each class keeps the name, method signatures, argument meaning and error behaviour
of the Loop-SGLang interface it replaces, so the reference can register it where
it registers its own:

* ``B200AttnBackend`` -- a ``BaseAttnBackend`` (python/loopsgl/attention/base.py:19-38).
  When ``loopsgl`` is importable it subclasses the reference's own abstract class and
  ``register()`` adds it to ``SUPPORTED_ATTENTION_BACKENDS`` as ``"b200"``
  (attention/__init__.py:19-40). It serves all three looped-KV policies, including
  last-exited on SM100 (the reference's selector rejects that combination,
  attention/selector.py:99-106), over this package's pools or the reference's own.
* ``LinearReplicated`` / ``LinearColParallelMerged`` / ``LinearQKVMerged`` /
  ``LinearOProj`` / ``LinearRowParallel`` -- the TP linear layers
  (layers/linear.py:14-128), ``forward(x) -> y`` on the tcgen05 GEMM; the row-parallel
  ones run the GEMM and the NVLink all-reduce as one kernel when the B200 communicator
  is installed (``comm.install``).
* ``RMSNorm`` / ``RMSNormFused`` -- layers/norm.py:8-38.
* ``RotaryEmbedding`` -- layers/rotary.py:12-55 (neox, fp32 cos/sin table).
* ``silu_and_mul`` -- layers/activation.py:9-12.
* ``store_cache`` -- kernel/store.py:89-152.

The batch object passed to the backend is the reference's ``ForwardBatch``
(core.py:217-252) or anything with the same fields; ``Context`` supplies
``kv_cache``, ``page_table`` (token-granular, page size 1) and ``page_size``
(core.py:255-277).
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass
from typing import List

import torch

from . import ops
from .model import rope_cos_sin_cache

try:  # the reference's own abstract interface, when it is installed
    from loopsgl.attention.base import BaseAttnBackend, BaseAttnMetadata

    HAVE_LOOPSGL = True
except ImportError:
    HAVE_LOOPSGL = False

    class BaseAttnMetadata(ABC):  # type: ignore[no-redef]
        """The abstract metadata of attention/base.py:13-16."""

        @abstractmethod
        def get_last_indices(self, bs: int) -> torch.Tensor: ...

    class BaseAttnBackend(ABC):  # type: ignore[no-redef]
        """The abstract backend of attention/base.py:19-38."""

        @abstractmethod
        def forward(self, q, k, v, layer_id: int, batch) -> torch.Tensor: ...

        @abstractmethod
        def prepare_metadata(self, batch) -> None: ...

        def prepare_core_metadata(self, batch, depths) -> None:
            raise ValueError("This attention backend does not support last-exited KV")

        @abstractmethod
        def init_capture_graph(self, max_seq_len: int, bs_list: List[int]) -> None: ...

        @abstractmethod
        def prepare_for_capture(self, batch) -> None: ...

        @abstractmethod
        def prepare_for_replay(self, batch) -> None: ...


# ----------------------------------------------------------------- attention --

@dataclass
class B200Metadata(BaseAttnMetadata):
    """Attention metadata (the fields of ``FAMetadata``, attention/fa.py:26-41)."""

    cu_seqlens_k: torch.Tensor
    cu_seqlens_q: torch.Tensor
    cache_seqlens: torch.Tensor
    max_seqlen_k: int
    max_seqlen_q: int
    page_table: torch.Tensor
    core_page_table: torch.Tensor | None = None
    core_out_loc: torch.Tensor | None = None
    fixed_page_table: torch.Tensor | None = None
    fixed_out_loc: torch.Tensor | None = None

    def get_last_indices(self, bs: int) -> torch.Tensor:
        return self.cu_seqlens_q[1: 1 + bs] - 1


class _Buffers:
    """Reusable metadata buffers (attention/utils.py:13-51)."""

    def __init__(self, max_bs: int, max_pages: int, device: torch.device) -> None:
        i32 = dict(dtype=torch.int32, device=device)
        self.seq_lens = torch.ones(max_bs, **i32)
        self.cu_seqlens_k = torch.arange(0, max_bs + 1, **i32)
        self.cu_seqlens_q = torch.arange(0, max_bs + 1, **i32)
        self.page_table = torch.zeros(max_bs, max_pages, **i32)


def _slot_views(kvcache, layer_id: int) -> tuple[torch.Tensor, torch.Tensor]:
    """One KV layer as ``[slots, Hkv*D]`` matrices: this package's pools expose them
    directly, the reference's as ``k_cache``/``v_cache`` views (mha_pool.py:48-52,
    last_exited.py:292-296) of contiguous ``[..., Hkv, D]`` rows."""
    if hasattr(kvcache, "slots"):
        return kvcache.slots(layer_id)
    kc, vc = kvcache.k_cache(layer_id), kvcache.v_cache(layer_id)
    return (kc.reshape(-1, kc.shape[-2] * kc.shape[-1]),
            vc.reshape(-1, vc.shape[-2] * vc.shape[-1]))


class B200AttnBackend(BaseAttnBackend):
    """``BaseAttnBackend`` on the sm_100a paged-attention kernel.

    ``B200AttnBackend(config)`` takes the pool and page size from the reference's global
    ``Context`` (as its FlashAttention backend does, attention/fa.py:47-52); ``ctx``
    supplies them directly."""

    def __init__(self, config, ctx=None) -> None:
        if ctx is None:
            from loopsgl.core import get_global_ctx

            ctx = get_global_ctx()
        self.config = config
        self.ctx = ctx
        self.kvcache = ctx.kv_cache
        self.page_size = ctx.page_size
        self.scale = config.head_dim ** -0.5
        self.num_kv_heads = getattr(self.kvcache, "num_kv_heads", None) or \
            getattr(config, "num_kv_heads")
        # last-exited pools carry a slot map (the reference's test, attention/fa.py:74)
        self.last_exited = hasattr(self.kvcache, "slot_map")
        self.core_start = getattr(self.kvcache, "core_start", 0)
        self.core_end = getattr(self.kvcache, "core_end", 0)
        self.eager: _Buffers | None = None
        self.capture: _Buffers | None = None
        self.capture_bs: List[int] = []
        self._group_tables: dict[tuple[str, bool], tuple[torch.Tensor, torch.Tensor]] = {}

    # -- BaseAttnBackend.forward (attention/fa.py:68-93) ---------------------------
    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layer_id: int,
                batch) -> torch.Tensor:
        md = batch.attn_metadata
        out_loc, table = batch.out_loc, md.page_table
        if self.last_exited:
            group = self.kvcache.layer_groups[layer_id]
            core = self.core_start <= layer_id < self.core_end
            locs = md.core_out_loc if core else md.fixed_out_loc
            tables = md.core_page_table if core else md.fixed_page_table
            if locs is None or tables is None:
                raise ValueError("Last-exited KV needs prepare_core_metadata before attention")
            out_loc, table = locs[group], tables[group]
        self.kvcache.store_kv(k, v, out_loc, layer_id)
        kc, vc = _slot_views(self.kvcache, layer_id)
        q3 = q.view(q.shape[0], -1, self.config.head_dim) if q.dim() == 2 else q
        return ops.paged_attention(q3, kc, vc, table, md.cache_seqlens, md.cu_seqlens_q,
                                   self.page_size, table.shape[1] * self.page_size, self.scale,
                                   self.num_kv_heads)

    # -- metadata (attention/utils.py:54-83, fa.py:95-231) -----------------------
    def _fill(self, batch, buf: _Buffers, width: int) -> B200Metadata:
        bs = batch.padded_size
        ops.set_metadata(batch.seq_lens, None if batch.is_decode else batch.extend_lens,
                         self.ctx.page_table, batch.req_pool_indices, width, self.page_size,
                         batch.is_decode, buf.seq_lens[:bs], buf.cu_seqlens_k[: bs + 1],
                         buf.cu_seqlens_q[: bs + 1], buf.page_table[:bs])
        return B200Metadata(cu_seqlens_k=buf.cu_seqlens_k[: bs + 1],
                            cu_seqlens_q=buf.cu_seqlens_q[: bs + 1],
                            cache_seqlens=buf.seq_lens[:bs],
                            max_seqlen_k=width * self.page_size,
                            max_seqlen_q=1 if batch.is_decode else max(batch.extend_lens_cpu),
                            page_table=buf.page_table[:bs, :width])

    def _attach(self, batch, md: B200Metadata, capture: bool) -> None:
        if not self.last_exited:
            return
        kv = self.kvcache
        dev = md.page_table.device
        for kind, groups in (("core", kv.core_groups), ("fixed", kv.fixed_groups)):
            if not groups:
                continue
            shape = (groups, *md.page_table.shape)
            n = batch.out_loc.numel()
            key = (kind, capture)
            have = self._group_tables.get(key)
            if have is None or have[0].shape[1] < shape[1] or have[0].shape[2] < shape[2] \
                    or have[1].shape[1] < n:
                have = (torch.zeros(shape, dtype=torch.int32, device=dev),
                        torch.zeros(groups, max(n, 1), dtype=torch.int32, device=dev))
                self._group_tables[key] = have
            table, out = have[0][:, : shape[1], : shape[2]], have[1][:, :n]
            setattr(md, f"{kind}_page_table", table)
            setattr(md, f"{kind}_out_loc", out)
            if kind == "fixed":
                ops.last_exited_resolve(md.page_table, kv.fixed_map, md.cache_seqlens,
                                        md.cu_seqlens_q, batch.out_loc, 0, table, out)

    def prepare_metadata(self, batch) -> None:
        width = (max(batch.seq_lens_cpu) + self.page_size - 1) // self.page_size
        bs = batch.padded_size
        if self.eager is None or bs > self.eager.seq_lens.numel() \
                or width > self.eager.page_table.shape[1]:
            max_bs = 1 << (max(bs, 1) - 1).bit_length()
            max_pages = 1 << (max(width, 1) - 1).bit_length()
            self.eager = _Buffers(max_bs, max_pages, batch.seq_lens.device)
        md = self._fill(batch, self.eager, width)
        batch.attn_metadata = md
        self._attach(batch, md, capture=False)

    def prepare_core_metadata(self, batch, depths: int | torch.Tensor) -> None:
        """Resolve last-exited addresses at the rows' depths (attention/fa.py:95-108)."""
        if not self.last_exited:
            raise ValueError("This attention backend does not support last-exited KV")
        md = batch.attn_metadata
        if md.core_page_table is None or md.core_out_loc is None:
            raise ValueError("prepare_metadata must run before prepare_core_metadata")
        ops.last_exited_resolve(md.page_table, self.kvcache.version_map, md.cache_seqlens,
                                md.cu_seqlens_q, batch.out_loc, depths, md.core_page_table,
                                md.core_out_loc)

    def init_capture_graph(self, max_seq_len: int, bs_list: List[int]) -> None:
        assert self.capture is None, "Capture already initialized."
        max_pages = (max_seq_len + self.page_size - 1) // self.page_size
        dev = self.ctx.page_table.device
        self.capture = _Buffers(max(bs_list), max_pages, dev)
        self.capture_bs = sorted(bs_list)

    def prepare_for_capture(self, batch) -> None:
        assert batch.size in self.capture_bs and self.capture is not None
        cap, bs = self.capture, batch.size
        md = B200Metadata(cu_seqlens_k=cap.cu_seqlens_k[: bs + 1],
                          cu_seqlens_q=cap.cu_seqlens_q[: bs + 1],
                          cache_seqlens=cap.seq_lens[:bs],
                          max_seqlen_k=cap.page_table.shape[1] * self.page_size, max_seqlen_q=1,
                          page_table=cap.page_table[:bs, :])
        batch.attn_metadata = md
        self._attach(batch, md, capture=True)

    def prepare_for_replay(self, batch) -> None:
        assert self.capture is not None and batch.padded_size in self.capture_bs
        md = self._fill(batch, self.capture, self.capture.page_table.shape[1])
        batch.attn_metadata = md
        self._attach(batch, md, capture=True)


def create_b200_backend(config) -> B200AttnBackend:
    """The ``BackendCreator`` of attention/__init__.py:15-16."""
    return B200AttnBackend(config)


def register(name: str = "b200") -> bool:
    """Add the backend to the reference's ``SUPPORTED_ATTENTION_BACKENDS``
    (attention/__init__.py:19-40) under ``name``. False when ``loopsgl`` is absent;
    registering twice is a no-op."""
    if not HAVE_LOOPSGL:
        return False
    from loopsgl.attention import SUPPORTED_ATTENTION_BACKENDS

    if name not in SUPPORTED_ATTENTION_BACKENDS.supported_names():
        SUPPORTED_ATTENTION_BACKENDS.register(name)(create_b200_backend)
    return True


# ------------------------------------------------------------------- linears --

class _LinearTPImpl:
    """``_LinearTPImpl`` (layers/linear.py:14-33): ``y = x W^T (+ b)``."""

    def __init__(self, full_isize: int, full_osize: int, local_isize: int, local_osize: int,
                 has_bias: bool) -> None:
        self.full_input_size, self.full_output_size = full_isize, full_osize
        self.local_input_size, self.local_output_size = local_isize, local_osize
        self.weight = torch.empty(local_osize, local_isize)
        self.bias = torch.empty(local_osize) if has_bias else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        y = ops.linear(x.reshape(-1, shape[-1]), self.weight, self.bias)
        return y.view(*shape[:-1], y.shape[-1])


def _tp_size() -> int:
    from .comm import tp_size

    return tp_size()


class LinearReplicated(_LinearTPImpl):
    def __init__(self, input_size: int, output_size: int, has_bias: bool) -> None:
        super().__init__(input_size, output_size, input_size, output_size, has_bias)


class LinearColParallelMerged(_LinearTPImpl):
    def __init__(self, input_size: int, output_sizes: List[int], has_bias: bool) -> None:
        size = _tp_size()
        if any(s % size for s in output_sizes):
            raise ValueError(f"output sizes {output_sizes} do not divide by TP {size}")
        super().__init__(input_size, sum(output_sizes), input_size,
                         sum(s // size for s in output_sizes), has_bias)


class LinearQKVMerged(_LinearTPImpl):
    def __init__(self, hidden_size: int, head_dim: int, num_qo_heads: int, num_kv_heads: int,
                 has_bias: bool) -> None:
        size = _tp_size()
        if num_qo_heads % size:
            raise ValueError(f"{num_qo_heads} heads do not divide by TP {size}")
        local_kv = num_kv_heads // size if num_kv_heads % size == 0 else num_kv_heads
        super().__init__(hidden_size, (num_qo_heads + 2 * num_kv_heads) * head_dim, hidden_size,
                         (num_qo_heads // size + 2 * local_kv) * head_dim, has_bias)


class _RowParallel(_LinearTPImpl):
    """Row-parallel: this rank's input columns, the sum over the ranks. With the B200
    communicator installed the GEMM and the all-reduce are one kernel
    (``lsb_gemm_allreduce``); otherwise the local GEMM is all-reduced through the
    reference's communicator stack, as layers/linear.py:103-107 does."""

    def __init__(self, input_size: int, output_size: int, has_bias: bool) -> None:
        size = _tp_size()
        if input_size % size:
            raise ValueError(f"input size {input_size} does not divide by TP {size}")
        self._tp_size = size
        super().__init__(input_size, output_size, input_size // size, output_size, has_bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from .comm import active, reference_all_reduce

        if self._tp_size == 1:
            return super().forward(x)
        comm = active()
        if comm is None:
            return reference_all_reduce(super().forward(x))
        shape = x.shape
        y = comm.gemm_allreduce(x.reshape(-1, shape[-1]), self.weight, self.bias)
        return y.view(*shape[:-1], y.shape[-1])


class LinearOProj(_RowParallel):
    """layers/linear.py:92-107."""


class LinearRowParallel(_RowParallel):
    """layers/linear.py:110-128."""


# --------------------------------------------------------- norms / rotary --

class RMSNorm:
    """layers/norm.py:8-21."""

    def __init__(self, size: int, eps: float) -> None:
        self.eps = eps
        self.weight = torch.empty(size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return ops.rmsnorm(x, self.weight, self.eps)

    def forward_inplace(self, x: torch.Tensor) -> None:
        ops.rmsnorm(x, self.weight, self.eps, out=x)


class RMSNormFused:
    """layers/norm.py:24-38: ``(rmsnorm(x), x)`` or the in-place fused add."""

    def __init__(self, size: int, eps: float) -> None:
        self.eps = eps
        self.weight = torch.empty(size)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        if residual is None:
            return ops.rmsnorm(x, self.weight, self.eps), x
        ops.fused_add_rmsnorm(x, residual, self.weight, self.eps)
        return x, residual


class RotaryEmbedding:
    """layers/rotary.py:12-55 (neox); rotates q and k in place and returns them."""

    def __init__(self, head_size: int, rotary_dim: int, max_position_embeddings: int,
                 base: float, is_neox_style: bool = True, device="cuda") -> None:
        if rotary_dim != head_size or not is_neox_style:
            raise ValueError("only full-dimension neox RoPE is on the hot path")
        self.head_size = head_size
        self._cos_sin_cache = rope_cos_sin_cache(head_size, max_position_embeddings, base,
                                                 torch.device(device))

    def forward(self, positions: torch.Tensor, query: torch.Tensor, key: torch.Tensor):
        d = self.head_size
        for t in (query, key):
            t2 = t.reshape(t.shape[0], -1) if t.dim() != 2 else t
            ops.rope_only(t2, positions, self._cos_sin_cache, t2.shape[1] // d, d)
        return query, key


def silu_and_mul(x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """layers/activation.py:9-12."""
    y = ops.silu_and_mul(x)
    if out is not None:
        out.copy_(y)
        return out
    return y


def store_cache(k_cache: torch.Tensor, v_cache: torch.Tensor, indices: torch.Tensor,
                k: torch.Tensor, v: torch.Tensor, **_) -> None:
    """kernel/store.py:89-152 with the padding slot 0 preserved."""
    kc = k_cache.view(k_cache.shape[0], -1)
    vc = v_cache.view(v_cache.shape[0], -1)
    ops.store_kv(kc, vc, indices.to(torch.int32), k, v)
