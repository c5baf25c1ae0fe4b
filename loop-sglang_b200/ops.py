"""Tensor-level wrappers of the C ABI: validate torch tensors, pass raw pointers and
the current CUDA stream, raise on a non-zero status.

Every function launches one kernel of ``libloopsgl_b200.so`` on
``torch.cuda.current_stream()``; none of them synchronises the host, so they can
be captured into CUDA graphs. Scratch buffers (split-KV and split-K partials)
are cached per device and kernel kind, zeroed at allocation; the kernels leave
their counters zeroed, so one buffer serves every later call.
"""

from __future__ import annotations

import ctypes
import math

import torch

from ._lib import (
    LSB_EPI_BIAS,
    LSB_EPI_BIAS_AFTER_ROUND,
    LSB_EPI_NONE,
    LSB_EPI_SWIGLU,
    call,
    check,
    lib,
)

__all__ = [
    "rmsnorm", "fused_add_rmsnorm", "sandwich_norm", "rope_store_kv", "rope_only", "store_kv",
    "paged_attention",
    "gemm", "gemm_concat", "linear", "swiglu_interleave", "ouro_step_exit", "huginn_step_exit", "embedding",
    "gather_rows", "argmax", "argmax_sharded", "gemm_argmax", "argmax_pairs",
    "argmax_pairs_buffer", "silu_and_mul", "last_exited_resolve", "last_exited_reserve",
    "last_exited_release", "cdb_route", "cdb_admit", "device_error_word", "Workspace", "prepare_batch_inputs",
    "set_metadata",
    "LSB_EPI_NONE", "LSB_EPI_BIAS", "LSB_EPI_BIAS_AFTER_ROUND", "LSB_EPI_SWIGLU",
]

BF16 = torch.bfloat16


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, dtype: torch.dtype, name: str, contiguous: bool = True) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _row_stride(t: torch.Tensor, name: str) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be 2-D with unit column stride")
    return t.stride(0)


class Workspace:
    """Zero-initialised scratch per (device, kind), grown on demand.

    Growing replaces the buffer, so grow (call once at the largest shape) before
    capturing a CUDA graph that uses it.
    """

    _bufs: dict[tuple[int, str], torch.Tensor] = {}

    @classmethod
    def get(cls, kind: str, nbytes: int, device: torch.device) -> torch.Tensor | None:
        if nbytes <= 0:
            return None
        key = (device.index if device.index is not None else torch.cuda.current_device(), kind)
        buf = cls._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
            cls._bufs[key] = buf
        return buf

    @classmethod
    def clear(cls) -> None:
        cls._bufs.clear()


def device_error_word(reset: bool = True) -> int:
    """Sticky LSB_DEVERR_* bits set by kernels that met an out-of-range index."""
    out = torch.zeros(1, dtype=torch.int32)
    call("lsb_device_error_word", out.data_ptr(), int(reset), _stream())
    return int(out[0])


# -------------------------------------------------------------------- norms --

def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """``flashinfer.rmsnorm`` (layers/norm.py:16-17)."""
    _need(weight, BF16, "weight")
    _need(x, BF16, "x", contiguous=False)
    out = torch.empty(x.shape, dtype=BF16, device=x.device) if out is None else out
    call("lsb_rmsnorm", out.data_ptr(), _row_stride(out, "out"), x.data_ptr(),
         _row_stride(x, "x"), weight.data_ptr(), x.shape[0], x.shape[1], eps, _stream())
    return out


def fused_add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor,
                      eps: float) -> None:
    """``flashinfer.fused_add_rmsnorm`` in place (layers/norm.py:32-38)."""
    for t, n in ((x, "x"), (residual, "residual"), (weight, "weight")):
        _need(t, BF16, n)
    call("lsb_fused_add_rmsnorm", x.data_ptr(), residual.data_ptr(), weight.data_ptr(),
         x.shape[0], x.shape[1], eps, _stream())


def sandwich_norm(x: torch.Tensor, residual: torch.Tensor, w_a: torch.Tensor,
                  w_b: torch.Tensor, eps: float, out: torch.Tensor | None = None) -> torch.Tensor:
    """``rmsnorm(x)*w_a`` then fused add-norm with ``w_b`` (ouro.py:49-50, :52 + :45)."""
    for t, n in ((x, "x"), (residual, "residual"), (w_a, "w_a"), (w_b, "w_b")):
        _need(t, BF16, n)
    out = torch.empty_like(x) if out is None else out
    call("lsb_sandwich_norm", out.data_ptr(), x.data_ptr(), residual.data_ptr(), w_a.data_ptr(),
         w_b.data_ptr(), x.shape[0], x.shape[1], eps, _stream())
    return out


# ----------------------------------------------------------- RoPE + store --

def rope_store_kv(qkv: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor,
                  hq: int, hkv: int, head_dim: int, k_cache: torch.Tensor | None = None,
                  v_cache: torch.Tensor | None = None, out_loc: torch.Tensor | None = None) -> None:
    """RoPE on q/k in place in ``qkv`` and KV store at ``out_loc`` (attention.py:88-90 +
    store_kv). ``k_cache``/``v_cache`` are ``[slots, ...]`` views with rows of hkv*head_dim."""
    _need(qkv, BF16, "qkv", contiguous=False)
    _need(positions, torch.int32, "positions")
    _need(cos_sin, torch.float32, "cos_sin")
    slot_stride, num_slots = 0, 0
    if k_cache is not None:
        _need(k_cache, BF16, "k_cache", contiguous=False)
        _need(v_cache, BF16, "v_cache", contiguous=False)
        _need(out_loc, torch.int32, "out_loc")
        if k_cache.stride(0) != v_cache.stride(0) or k_cache.shape[0] != v_cache.shape[0]:
            raise ValueError("k_cache and v_cache must share slot count and stride")
        slot_stride, num_slots = k_cache.stride(0), k_cache.shape[0]
    call("lsb_rope_store_kv", qkv.data_ptr(), _row_stride(qkv, "qkv"), positions.data_ptr(),
         cos_sin.data_ptr(), cos_sin.shape[0], _p(k_cache), _p(v_cache), slot_stride, num_slots,
         _p(out_loc), qkv.shape[0], hq, hkv, head_dim, _stream())


def store_kv(k_cache: torch.Tensor, v_cache: torch.Tensor, out_loc: torch.Tensor,
             k: torch.Tensor, v: torch.Tensor) -> None:
    """``store_cache`` (kernel/store.py:89-152): rows of k/v into slots, slot 0 skipped.
    Caches are ``[slots, ...]`` views; k/v are ``[T, row]`` (row stride free)."""
    k2 = k.reshape(k.shape[0], math.prod(k.shape[1:])) if k.dim() != 2 else k
    v2 = v.reshape(v.shape[0], math.prod(v.shape[1:])) if v.dim() != 2 else v
    for t, n in ((k2, "k"), (v2, "v")):
        _need(t, BF16, n, contiguous=False)
    _need(out_loc, torch.int32, "out_loc")
    call("lsb_store_kv", k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0),
         k_cache.shape[0], k2.data_ptr(), _row_stride(k2, "k"), v2.data_ptr(),
         _row_stride(v2, "v"), out_loc.data_ptr(), out_loc.numel(), k2.shape[1], _stream())


def rope_only(x: torch.Tensor, positions: torch.Tensor, cos_sin: torch.Tensor, heads: int,
              head_dim: int) -> None:
    """Neox RoPE in place on ``heads`` heads of each row of ``x`` (rotary.py:40-55)."""
    rope_store_kv(x, positions, cos_sin, heads, 0, head_dim)


# -------------------------------------------------------------- attention --

def paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                    page_table: torch.Tensor, cache_seqlens: torch.Tensor,
                    cu_seqlens_q: torch.Tensor, page_size: int, max_seqlen: int, scale: float,
                    hkv: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Causal paged attention (the backends' library call, attention/fa.py:82-93).

    q ``[rows, hq, D]`` (row stride may exceed hq*D, e.g. a view of the qkv buffer);
    k/v caches ``[slots, hkv, D]``-shaped slot views of one KV layer.
    """
    rows, hq, d = q.shape
    _need(q, BF16, "q", contiguous=False)
    if q.stride(2) != 1 or q.stride(1) != d:
        raise ValueError("q heads must be contiguous within a row")
    for t, n in ((page_table, "page_table"), (cache_seqlens, "cache_seqlens"),
                 (cu_seqlens_q, "cu_seqlens_q")):
        _need(t, torch.int32, n, contiguous=(n != "page_table"))
    if page_table.stride(1) != 1:
        raise ValueError("page_table must have unit column stride")
    out = torch.empty(rows, hq, d, dtype=BF16, device=q.device) if out is None else out
    nbytes = lib().lsb_paged_attention_workspace_size(rows, hq, d, max_seqlen)
    ws = Workspace.get("attention", nbytes, q.device)
    call("lsb_paged_attention", out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0),
         k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0), k_cache.shape[0],
         page_table.data_ptr(), page_table.stride(0), cache_seqlens.data_ptr(),
         cu_seqlens_q.data_ptr(), cache_seqlens.numel(), rows, hq, hkv, d, page_size,
         max_seqlen, scale, _p(ws), 0 if ws is None else ws.numel(), _stream())
    return out


def paged_attention_shared_prefix(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                                  page_table: torch.Tensor, cache_seqlens: torch.Tensor,
                                  cu_seqlens_q: torch.Tensor, page_size: int, max_seqlen: int,
                                  scale: float, hkv: int, groups,
                                  out: torch.Tensor | None = None) -> torch.Tensor:
    """``paged_attention`` for decode rows of which groups share leading KV pages
    (``prefix_cache.SharedPrefixGroups``): each group's shared keys are read once for all of
    its rows. Same result as ``paged_attention`` on the same arguments."""
    if groups is None:
        return paged_attention(q, k_cache, v_cache, page_table, cache_seqlens, cu_seqlens_q,
                               page_size, max_seqlen, scale, hkv, out)
    rows, hq, d = q.shape
    _need(q, BF16, "q", contiguous=False)
    if q.stride(2) != 1 or q.stride(1) != d:
        raise ValueError("q heads must be contiguous within a row")
    for t, n in ((page_table, "page_table"), (cache_seqlens, "cache_seqlens"),
                 (cu_seqlens_q, "cu_seqlens_q"), (groups.group_ptr, "group_ptr"),
                 (groups.group_rows, "group_rows"), (groups.group_prefix, "group_prefix"),
                 (groups.row_prefix, "row_prefix")):
        _need(t, torch.int32, n, contiguous=(n != "page_table"))
    if page_table.stride(1) != 1:
        raise ValueError("page_table must have unit column stride")
    if groups.row_prefix.numel() != rows:
        raise ValueError("row_prefix must have one entry per row")
    out = torch.empty(rows, hq, d, dtype=BF16, device=q.device) if out is None else out
    nbytes = max(lib().lsb_paged_attention_workspace_size(rows, hq, d, max_seqlen),
                 lib().lsb_paged_attention_shared_prefix_workspace_size(
                     rows, hq, d, max_seqlen, groups.max_group_prefix))
    ws = Workspace.get("attention", nbytes, q.device)
    call("lsb_paged_attention_shared_prefix", out.data_ptr(), out.stride(0), q.data_ptr(),
         q.stride(0), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.stride(0),
         k_cache.shape[0], page_table.data_ptr(), page_table.stride(0), cache_seqlens.data_ptr(),
         cu_seqlens_q.data_ptr(), cache_seqlens.numel(), rows, hq, hkv, d, page_size,
         max_seqlen, scale, groups.group_ptr.data_ptr(), groups.group_rows.data_ptr(),
         groups.group_prefix.data_ptr(), groups.row_prefix.data_ptr(), groups.num_groups,
         groups.max_group_rows, groups.max_group_prefix, _p(ws), ws.numel(), _stream())
    return out


# ------------------------------------------------------------------- GEMM --

def gemm(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
         epilogue: int = LSB_EPI_NONE, out: torch.Tensor | None = None) -> torch.Tensor:
    """``y = x . w^T`` (+ bias / SwiGLU) on tcgen05 (layers/linear.py:32-33)."""
    _need(x, BF16, "x", contiguous=False)
    _need(w, BF16, "w", contiguous=False)
    m, k = x.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"gemm: x has K={k}, w has K={w.shape[1]}")
    if bias is not None:
        _need(bias, BF16, "bias")
    cols = n // 2 if epilogue == LSB_EPI_SWIGLU else n
    out = torch.empty(m, cols, dtype=BF16, device=x.device) if out is None else out
    nbytes = lib().lsb_gemm_workspace_size(m, n, k)
    ws = Workspace.get("gemm", nbytes, x.device)
    call("lsb_gemm", out.data_ptr(), _row_stride(out, "out"), x.data_ptr(),
         _row_stride(x, "x"), w.data_ptr(), _row_stride(w, "w"), _p(bias), m, n, k, epilogue,
         _p(ws), 0 if ws is None else ws.numel(), _stream())
    return out


def gemm_rope_store(x: torch.Tensor, w: torch.Tensor, positions: torch.Tensor,
                    cos_sin: torch.Tensor, hq: int, hkv: int, head_dim: int,
                    k_cache: torch.Tensor, v_cache: torch.Tensor, out_loc: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """The QKV projection with RoPE and the KV store in its epilogue: ``gemm(x, w)`` then
    ``rope_store_kv`` on the result, in one launch (models/utils.py:119-131,
    layers/attention.py:88-90). 128-dim heads only (one head per weight tile)."""
    _need(x, BF16, "x", contiguous=False)
    _need(w, BF16, "w", contiguous=False)
    _need(positions, torch.int32, "positions")
    _need(cos_sin, torch.float32, "cos_sin")
    _need(k_cache, BF16, "k_cache", contiguous=False)
    _need(v_cache, BF16, "v_cache", contiguous=False)
    _need(out_loc, torch.int32, "out_loc")
    if k_cache.stride(0) != v_cache.stride(0) or k_cache.shape[0] != v_cache.shape[0]:
        raise ValueError("k_cache and v_cache must share slot count and stride")
    m, k = x.shape
    n = w.shape[0]
    if w.shape[1] != k:
        raise ValueError(f"gemm_rope_store: x has K={k}, w has K={w.shape[1]}")
    out = torch.empty(m, n, dtype=BF16, device=x.device) if out is None else out
    call("lsb_gemm_rope_store", out.data_ptr(), _row_stride(out, "out"), x.data_ptr(),
         _row_stride(x, "x"), w.data_ptr(), _row_stride(w, "w"), m, n, k, positions.data_ptr(),
         cos_sin.data_ptr(), cos_sin.shape[0], k_cache.data_ptr(), v_cache.data_ptr(),
         k_cache.stride(0), k_cache.shape[0], out_loc.data_ptr(), hq, hkv, head_dim, _stream())
    return out


def gemm_concat(x1: torch.Tensor, x2: torch.Tensor, w: torch.Tensor,
                bias: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``F.linear(torch.cat([x1, x2], -1), w, bias)`` without the concatenation
    (models/looped/huginn.py:162-167, Huginn's adapter)."""
    for t, n in ((x1, "x1"), (x2, "x2"), (w, "w")):
        _need(t, BF16, n, contiguous=False)
    m, k1 = x1.shape
    k2 = x2.shape[1]
    n = w.shape[0]
    if x2.shape[0] != m or w.shape[1] != k1 + k2:
        raise ValueError(f"gemm_concat: x1 [{m}, {k1}], x2 {list(x2.shape)}, w {list(w.shape)}")
    if bias is not None:
        _need(bias, BF16, "bias")
    out = torch.empty(m, n, dtype=BF16, device=x1.device) if out is None else out
    call("lsb_gemm_concat", out.data_ptr(), _row_stride(out, "out"), x1.data_ptr(),
         _row_stride(x1, "x1"), x2.data_ptr(), _row_stride(x2, "x2"), w.data_ptr(),
         _row_stride(w, "w"), _p(bias), m, n, k1, k2,
         LSB_EPI_BIAS if bias is not None else LSB_EPI_NONE, _stream())
    return out


def linear(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """``F.linear`` semantics: bias added in fp32 before the single rounding."""
    return gemm(x, w, bias, LSB_EPI_BIAS if bias is not None else LSB_EPI_NONE, out)


def swiglu_interleave(w: torch.Tensor) -> torch.Tensor:
    """Gate_up weight ``[2I, K]`` -> 128-row tiles of 64 gate + 64 up rows."""
    _need(w, BF16, "w")
    out = torch.empty_like(w)
    call("lsb_swiglu_interleave", out.data_ptr(), w.data_ptr(), w.shape[0] // 2, w.shape[1],
         _stream())
    return out


# -------------------------------------------------------- loop-step exits --

def ouro_step_exit(x: torch.Tensor, residual: torch.Tensor, w_post2: torch.Tensor,
                   w_final: torch.Tensor, eps: float, hidden_out: torch.Tensor,
                   gate_w: torch.Tensor | None = None, gate_b: torch.Tensor | None = None,
                   exit_state: torch.Tensor | None = None, signal: torch.Tensor | None = None,
                   slot: torch.Tensor | None = None, depth: torch.Tensor | int = 0,
                   threshold: float = 1.0, min_loop_steps: int = 1,
                   lookahead: bool = False) -> None:
    """Step-final sandwich norm + exit gate + state scatter (ouro.py:136, :142-155,
    cdb_model_runner.py:102-108)."""
    for t, n in ((x, "x"), (residual, "residual"), (w_post2, "w_post2"), (w_final, "w_final")):
        _need(t, BF16, n)
    if slot is not None:
        _need(slot, torch.int64, "slot")
    dt = depth if isinstance(depth, torch.Tensor) else None
    if dt is not None:
        _need(dt, torch.int32, "depth")
    call("lsb_ouro_step_exit", hidden_out.data_ptr(), _row_stride(hidden_out, "hidden_out"),
         x.data_ptr(), residual.data_ptr(), w_post2.data_ptr(), w_final.data_ptr(), _p(gate_w),
         _p(gate_b), _p(slot), _p(exit_state), _p(signal), _p(dt),
         0 if dt is not None else int(depth), int(lookahead), min_loop_steps, threshold,
         x.shape[0], x.shape[1], eps, _stream())


def huginn_step_exit(h: torch.Tensor, exit_state: torch.Tensor, hidden_out: torch.Tensor,
                     signal: torch.Tensor, threshold: float,
                     slot: torch.Tensor | None = None) -> None:
    """Huginn relative-change exit + state scatter (huginn.py:184-194)."""
    call("lsb_huginn_step_exit", hidden_out.data_ptr(), exit_state.data_ptr(), h.data_ptr(),
         _p(slot), signal.data_ptr(), threshold, h.shape[0], h.shape[1], _stream())


# ------------------------------------------------------- gathers / sample --

def embedding(ids: torch.Tensor, weight: torch.Tensor, scale: float = 1.0, vocab_start: int = 0,
              vocab_len: int | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Vocab-parallel embedding gather (layers/embedding.py:34-43, huginn.py:147-148)."""
    _need(ids, torch.int32, "ids")
    _need(weight, BF16, "weight")
    vlen = weight.shape[0] if vocab_len is None else vocab_len
    out = torch.empty(ids.numel(), weight.shape[1], dtype=BF16, device=ids.device) if out is None else out
    call("lsb_embedding", out.data_ptr(), ids.data_ptr(), weight.data_ptr(), ids.numel(),
         weight.shape[1], vocab_start, vlen, scale, _stream())
    return out


def gather_rows(src: torch.Tensor, index: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """``src.index_select(0, index)`` (cdb_model_runner.py:94-101)."""
    _need(index, torch.int64, "index")
    out = torch.empty(index.numel(), src.shape[1], dtype=src.dtype, device=src.device) if out is None else out
    call("lsb_gather_rows", out.data_ptr(), src.data_ptr(), index.data_ptr(), index.numel(),
         src.shape[1], _stream())
    return out


def argmax_pairs_buffer(rows: int, n: int, device, shards: int = 1) -> torch.Tensor:
    """A [shards * rows, tiles, 2] fp32 buffer of (value, index) pairs for ``gemm_argmax``
    over ``n`` vocabulary entries, every value -inf (tiles never scored keep it)."""
    tiles = int(lib().lsb_gemm_argmax_tiles(n))
    return torch.full((shards * rows, tiles, 2), float("-inf"), dtype=torch.float32,
                      device=device)


def gemm_argmax(x: torch.Tensor, w: torch.Tensor, pairs: torch.Tensor,
                n_valid: int | None = None) -> torch.Tensor:
    """The LM-head GEMM with greedy sampling in its epilogue: per row and 128-entry
    vocabulary tile, the largest bf16-rounded logit and its index (first on ties) into
    ``pairs`` (``argmax_pairs_buffer``); the logits are not written. ``n_valid`` scores
    only the first rows of ``w`` (a tensor-parallel rank's padded vocabulary range)."""
    _need(x, BF16, "x", contiguous=False)
    _need(w, BF16, "w", contiguous=False)
    _need(pairs, torch.float32, "pairs")
    m, k = x.shape
    n = w.shape[0] if n_valid is None else n_valid
    if w.shape[1] != k or pairs.shape[0] < m or pairs.dim() != 3 or pairs.shape[2] != 2:
        raise ValueError("gemm_argmax: bad shapes")
    call("lsb_gemm_argmax", pairs.data_ptr(), pairs.shape[1], x.data_ptr(),
         _row_stride(x, "x"), w.data_ptr(), _row_stride(w, "w"), m, n, k, _stream())
    return pairs


def argmax_pairs(pairs: torch.Tensor, shards: int, rows: int, tiles: int, shard_cols: int,
                 out: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy tokens from ``gemm_argmax`` pairs of ``shards`` vocabulary ranges of
    ``shard_cols`` entries each, stored shard-major [shards * rows, ld, 2]."""
    _need(pairs, torch.float32, "pairs")
    out = torch.empty(rows, dtype=torch.int32, device=pairs.device) if out is None else out
    call("lsb_argmax_pairs", out.data_ptr(), pairs.data_ptr(), shards, rows, tiles,
         pairs.shape[1], shard_cols, _stream())
    return out


def argmax(logits: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy sampling (model_executor/sample.py:108-112)."""
    _need(logits, BF16, "logits", contiguous=False)
    out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device) if out is None else out
    call("lsb_argmax", out.data_ptr(), logits.data_ptr(), logits.shape[0], logits.shape[1],
         _row_stride(logits, "logits"), _stream())
    return out


def argmax_sharded(gathered: torch.Tensor, shards: int, rows: int, cols: int, vocab: int,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """Greedy token over tensor-parallel logits gathered rank by rank ``[shards*rows, cols]``
    (rank r holds vocabulary entries r*cols ..), entries >= ``vocab`` being padding."""
    _need(gathered, BF16, "gathered")
    if gathered.numel() != shards * rows * cols:
        raise ValueError("argmax_sharded: gathered logits have the wrong size")
    out = torch.empty(rows, dtype=torch.int32, device=gathered.device) if out is None else out
    call("lsb_argmax_sharded", out.data_ptr(), gathered.data_ptr(), shards, rows, cols, vocab,
         _stream())
    return out


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """``flashinfer.silu_and_mul`` (layers/activation.py:9-12)."""
    _need(x, BF16, "x")
    inter = x.shape[1] // 2
    out = torch.empty(x.shape[0], inter, dtype=BF16, device=x.device)
    call("lsb_silu_and_mul", out.data_ptr(), x.data_ptr(), x.shape[0], inter, _stream())
    return out


# ------------------------------------------------------ last-exited maps --

def last_exited_resolve(logical_table: torch.Tensor, version_map: torch.Tensor,
                        cache_seqlens: torch.Tensor, cu_seqlens_q: torch.Tensor,
                        logical_out: torch.Tensor, depths: torch.Tensor | int,
                        physical_table: torch.Tensor, physical_out: torch.Tensor) -> None:
    """``prepare_last_exited_metadata`` (attention/metadata.py:220-291).

    version_map ``[steps, groups, handles]``; physical_table ``[groups, rows, cols]``;
    physical_out ``[groups, n]``.
    """
    dt = depths if isinstance(depths, torch.Tensor) else None
    groups = version_map.shape[1]
    call("lsb_last_exited_resolve", physical_table.data_ptr(), physical_table.stride(0),
         physical_table.stride(1), physical_out.data_ptr(), physical_out.stride(0),
         logical_table.data_ptr(), logical_table.stride(0), version_map.data_ptr(),
         version_map.stride(0), version_map.stride(1), cache_seqlens.data_ptr(),
         cu_seqlens_q.data_ptr(), logical_out.data_ptr(), _p(dt),
         0 if dt is not None else int(depths), cache_seqlens.numel(), logical_table.shape[1],
         groups, _stream())


def last_exited_reserve(slot_map, completed, free_slots, free_count, handles, steps, fixed,
                        core, restore_depths=None) -> None:
    """``_reserve_versions`` in handle order (kvcache/last_exited.py:15-47)."""
    call("lsb_last_exited_reserve", slot_map.data_ptr(), completed.data_ptr(), slot_map.shape[1],
         free_slots.data_ptr(), free_count.data_ptr(), handles.data_ptr(), _p(restore_depths),
         handles.numel(), steps, fixed, core, _stream())


def last_exited_release(slot_map, completed, free_slots, free_count, handles, steps, fixed, core,
                        exits=None) -> None:
    """``_release_versions`` in handle order (kvcache/last_exited.py:50-84)."""
    call("lsb_last_exited_release", slot_map.data_ptr(), completed.data_ptr(), slot_map.shape[1],
         free_slots.data_ptr(), free_count.data_ptr(), handles.data_ptr(), _p(exits),
         handles.numel(), steps, fixed, core, _stream())



def cdb_route(depth, seq_lens, ids, sampled, signal, out_count, alias_handle, alias_depth,
              reserve_handle, exited, req_to_token, req_pool_indices, max_depth: int,
              max_seq_len: int, replay_depths=None, forced_ids=None, out_tokens=None,
              out_depths=None, produced=None) -> None:
    """Device-side exit routing of one CDB core step (cdb_scheduler.py:189-267); see
    ``lsb_cdb_route``. Per-output arrays are ``[rows, out_stride]`` int32."""
    outs = [t for t in (replay_depths, forced_ids, out_tokens, out_depths) if t is not None]
    stride = outs[0].shape[1] if outs else 0
    if any(t.shape[1] != stride or t.stride(1) != 1 or t.stride(0) != stride for t in outs):
        raise ValueError("cdb_route: per-output arrays must share one contiguous [rows, n] shape")
    call("lsb_cdb_route", depth.data_ptr(), seq_lens.data_ptr(), ids.data_ptr(), sampled.data_ptr(),
         _p(signal), _p(replay_depths), _p(forced_ids), stride, out_count.data_ptr(),
         _p(out_tokens), _p(out_depths), alias_handle.data_ptr(), alias_depth.data_ptr(),
         reserve_handle.data_ptr(), exited.data_ptr(), req_to_token.data_ptr(),
         req_to_token.stride(0), req_pool_indices.data_ptr(), depth.numel(), max_depth,
         max_seq_len, _p(produced), _stream())


def cdb_admit(hidden: torch.Tensor, exit_state: torch.Tensor | None, slots: torch.Tensor,
              exited: torch.Tensor, emb: torch.Tensor) -> None:
    """Exited rows take their successor's prelude state (cdb_model_runner.py:84-91)."""
    _need(slots, torch.int64, "slots")
    call("lsb_cdb_admit", hidden.data_ptr(), hidden.stride(0), _p(exit_state), slots.data_ptr(),
         exited.data_ptr(), emb.data_ptr(), slots.numel(), hidden.shape[1], _stream())


# -------------------------------------------------------- batch metadata --

def prepare_batch_inputs(seq_lens, extend_lens, req_pool_indices, req_to_token, is_decode,
                         positions, out_loc, req_mapping=None) -> None:
    """``_prepare_batch_inputs`` (kernel/batch.py:72-129) into preallocated outputs."""
    call("lsb_prepare_batch_inputs", positions.data_ptr(), _p(req_mapping), out_loc.data_ptr(),
         seq_lens.data_ptr(), _p(extend_lens), req_pool_indices.data_ptr(),
         req_to_token.data_ptr(), req_to_token.stride(0), seq_lens.numel(), int(is_decode),
         _stream())


def set_metadata(seq_lens, extend_lens, req_to_token, req_pool_indices, max_seq_pages,
                 page_size, is_decode, cache_seqlens, cu_seqlens_k, cu_seqlens_q, page_table,
                 seq_len_delta: int = 0) -> None:
    """``_fused_metadata_kernel_general`` (attention/metadata.py:59-216)."""
    call("lsb_set_metadata", cache_seqlens.data_ptr(), cu_seqlens_k.data_ptr(),
         cu_seqlens_q.data_ptr(), page_table.data_ptr(), page_table.stride(0),
         req_to_token.data_ptr(), req_to_token.stride(0), req_pool_indices.data_ptr(),
         seq_lens.data_ptr(), _p(extend_lens), seq_lens.numel(), max_seq_pages, page_size,
         seq_len_delta, int(is_decode), _stream())


# ---------------------------------------------------------- KV snapshots --

KV_STAGING_BYTES = 256 << 20  # device staging bound of one snapshot copy


def gemm_plan(m: int, n: int, k: int) -> dict:
    """The tile plan ``gemm`` uses for an m x n x k product on the current device."""
    out = (ctypes.c_int32 * 5)()
    check(lib().lsb_gemm_plan(m, n, k, out), "gemm_plan")
    return {"tokens_per_tile": out[0], "tiles": out[1], "splits": out[2], "stages": out[3],
            "smem": out[4], "ctas": out[1] * out[2]}


def attention_plan(rows: int, hq: int, hkv: int, head_dim: int, page_size: int,
                   max_seqlen: int, slot_stride: int | None = None) -> dict:
    """The launch plan ``paged_attention`` uses for a decode call of this shape (host only)."""
    out = (ctypes.c_int32 * 6)()
    stride = hkv * head_dim if slot_stride is None else slot_stride
    check(lib().lsb_paged_attention_plan(rows, hq, hkv, head_dim, page_size, max_seqlen, stride,
                                         out), "paged_attention_plan")
    return {"kernel": "streaming" if out[0] else "per_cta", "keys_per_item": out[1],
            "splits": out[2], "stages": out[3], "keys_per_stage": out[4],
            "lane_per_page": bool(out[5])}


def kv_snapshot_bytes(n: int, row_bytes: int, num_layers: int, core_start: int = 0,
                      core_end: int = 0, steps: int = 1, versioned: bool = False) -> int:
    """Host bytes of an n-token KV snapshot (see ``lsb_kv_snapshot_bytes``)."""
    b = lib().lsb_kv_snapshot_bytes(n, row_bytes, num_layers, core_start, core_end, steps,
                                    int(versioned))
    if b < 0:
        raise ValueError("kv_snapshot_bytes: invalid pool shape")
    return b


def _staging(total: int, per_token: int, device) -> torch.Tensor:
    size = max(per_token, min(total, KV_STAGING_BYTES // per_token * per_token))
    return torch.empty(size, dtype=torch.uint8, device=device)


def kv_backup(host_out: torch.Tensor, pool: torch.Tensor, lanes: int, pool_rows: int,
              row_bytes: int, indices: torch.Tensor, num_layers: int, slot_map=None,
              completed_depth=None, core_start: int = 0, core_end: int = 0,
              steps: int = 1) -> None:
    """Gather a snapshot of ``indices`` into ``host_out`` (CPU, ideally pinned); returns
    after the copies completed. ``lsb_kv_backup``."""
    _need(pool, pool.dtype, "pool")
    _need(indices, torch.int32, "indices")
    if host_out.is_cuda or not host_out.is_contiguous():
        raise ValueError("kv_backup: host_out must be a contiguous CPU tensor")
    n = indices.numel()
    expanded = (num_layers + (core_end - core_start) * (steps - 1)) if slot_map is not None \
        else num_layers
    staging = _staging(2 * expanded * n * row_bytes, 2 * expanded * row_bytes, pool.device)
    call("lsb_kv_backup", host_out.data_ptr(), pool.data_ptr(), lanes, pool_rows, row_bytes,
         indices.data_ptr(), n, _p(slot_map), 0 if slot_map is None else slot_map.shape[1],
         _p(completed_depth), num_layers, core_start, core_end, steps, staging.data_ptr(),
         staging.numel(), _stream())


def kv_restore(pool: torch.Tensor, host_in: torch.Tensor, lanes: int, pool_rows: int,
               row_bytes: int, indices: torch.Tensor, num_layers: int, slot_map=None,
               core_start: int = 0, core_end: int = 0, steps: int = 1) -> None:
    """Scatter a snapshot back into the pool at ``indices`` (``lsb_kv_restore``)."""
    _need(pool, pool.dtype, "pool")
    _need(indices, torch.int32, "indices")
    if host_in.is_cuda or not host_in.is_contiguous():
        raise ValueError("kv_restore: host_in must be a contiguous CPU tensor")
    n = indices.numel()
    expanded = (num_layers + (core_end - core_start) * (steps - 1)) if slot_map is not None \
        else num_layers
    staging = _staging(2 * expanded * n * row_bytes, 2 * expanded * row_bytes, pool.device)
    call("lsb_kv_restore", pool.data_ptr(), host_in.data_ptr(), lanes, pool_rows, row_bytes,
         indices.data_ptr(), n, _p(slot_map), 0 if slot_map is None else slot_map.shape[1],
         num_layers, core_start, core_end, steps, staging.data_ptr(), staging.numel(), _stream())
