"""Floating-point operators of the looped-decoder hot path, restated on the CPU.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the checker for the CUDA
kernels, never a product code path.

Every function computes in fp32 on torch CPU tensors and rounds to the storage
dtype exactly where the reference's GPU path rounds, so that a bf16 CUDA kernel
can be compared against it with the bf16 tolerance (rel 2e-2). Reference
citations are paths inside the Loop-SGLang project (``python/loopsgl/...``) and,
for library arithmetic the reference delegates to, FlashInfer 0.6.x's CUDA
headers (``flashinfer/norm.cuh``, ``flashinfer/pos_enc.cuh``,
``flashinfer/activation.cuh``).
"""

from __future__ import annotations

import torch

__all__ = [
    "rmsnorm",
    "fused_add_rmsnorm",
    "rms_norm_fused",
    "rope_cos_sin_cache",
    "apply_rope_neox",
    "silu_and_mul",
    "linear",
    "linear_bias_after_rounding",
    "store_kv",
    "paged_attention",
    "cumulative_exit_probability",
    "relative_state_change",
    "ouro_exit_signal",
    "huginn_exit_signal",
    "embedding",
    "greedy_sample",
    "softmax_scale",
]


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """``y = x * rsqrt(mean(x^2) + eps) * w``, fp32 math, one rounding at the end.

    Follows ``layers/norm.py:16-17`` (``flashinfer.rmsnorm``), whose kernel
    (``flashinfer/norm.cuh`` RMSNormKernel) sums ``float(x)^2`` in fp32 and writes
    ``float(x) * rms_rcp * float(w)`` rounded to the input dtype.
    """
    xf = x.float()
    rrms = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (xf * rrms * weight.float()).to(x.dtype)


def fused_add_rmsnorm(
    x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float
) -> tuple[torch.Tensor, torch.Tensor]:
    """``residual <- x + residual``; ``x <- rmsnorm(residual)``, returned as (x, residual).

    Follows ``layers/norm.py:32-38`` (``flashinfer.fused_add_rmsnorm``). The
    FlashInfer kernel (``norm.cuh`` FusedAddRMSNormKernel) keeps the fp32 sum
    ``s = float(x) + float(r)``, stores ``r = dtype(s)``, and normalises the fp32
    ``s`` (not the rounded residual).
    """
    s = x.float() + residual.float()
    new_residual = s.to(residual.dtype)
    rrms = torch.rsqrt(s.pow(2).mean(dim=-1, keepdim=True) + eps)
    return (s * rrms * weight.float()).to(x.dtype), new_residual


def rms_norm_fused(
    x: torch.Tensor, residual: torch.Tensor | None, weight: torch.Tensor, eps: float
) -> tuple[torch.Tensor, torch.Tensor]:
    """``RMSNormFused.forward`` (``layers/norm.py:32-38``).

    With no residual it returns ``(rmsnorm(x), x)``: the un-normalised input
    becomes the residual stream.
    """
    if residual is None:
        return rmsnorm(x, weight, eps), x
    return fused_add_rmsnorm(x, residual, weight, eps)


def rope_cos_sin_cache(head_dim: int, max_position: int, base: float) -> torch.Tensor:
    """fp32 ``[max_position, head_dim]`` table ``cat(cos, sin)``.

    Same construction as ``layers/rotary.py:26-34``: ``inv_freq = 1 / base^(2i/D)``,
    ``freqs = t * inv_freq`` via einsum, both in fp32.
    """
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1)


def apply_rope_neox(
    positions: torch.Tensor, x: torch.Tensor, cos_sin_cache: torch.Tensor
) -> torch.Tensor:
    """Neox rotate-half RoPE on ``x[T, H, D]`` at ``positions[T]``.

    ``flashinfer/pos_enc.cuh`` ``vec_apply_llama_rope_cos_sin``: for ``i < D/2``
    ``y_i = x_i cos_i - x_{i+D/2} sin_i`` and ``y_{i+D/2} = x_{i+D/2} cos_i + x_i sin_i``
    in fp32, rounded to the input dtype; called in place on q and k by
    ``layers/rotary.py:40-55`` before the KV store (``layers/attention.py:90``).
    """
    d = x.shape[-1]
    half = d // 2
    cs = cos_sin_cache[positions.long()]  # [T, D]
    cos = cs[:, None, :half]
    sin = cs[:, None, half:]
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    y1 = x1 * cos - x2 * sin
    y2 = x2 * cos + x1 * sin
    return torch.cat([y1, y2], dim=-1).to(x.dtype)


def silu_and_mul(x: torch.Tensor) -> torch.Tensor:
    """``silu(x[:, :I]) * x[:, I:]`` (``layers/activation.py:9-12``).

    FlashInfer's ``act_and_mul_kernel`` (``activation.cuh``) computes
    ``silu(g) = g / (1 + exp(-g))`` and the product in fp32, then rounds once.
    """
    i = x.shape[-1] // 2
    g = x[..., :i].float()
    u = x[..., i:].float()
    return (g / (1.0 + torch.exp(-g)) * u).to(x.dtype)


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``F.linear`` as cuBLAS runs it for bf16 (``layers/linear.py:32-33``).

    fp32 accumulation, bias added in fp32, one rounding to the output dtype.
    """
    y = x.float() @ weight.float().t()
    if bias is not None:
        y = y + bias.float()
    return y.to(x.dtype)


def linear_bias_after_rounding(
    x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None
) -> torch.Tensor:
    """Huginn's QKV projection: the product is rounded, then the bias is added.

    ``models/looped/huginn.py:44-47``: ``qkv = F.linear(x, W); qkv.add_(b)``.
    """
    y = linear(x, weight)
    if bias is not None:
        y = (y.float() + bias.float()).to(y.dtype)
    return y


def store_kv(
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    indices: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    reserved_skip_index: int = 0,
) -> None:
    """Scatter K/V rows into token slots ``indices``, never touching the padding slot.

    ``kernel/store.py:89-152`` and ``kernel/csrc/jit/store.cu:127-156``: row ``i``
    goes to slot ``indices[i]`` unless it equals ``reserved_skip_index`` (0);
    a negative skip index disables the check. Caches are ``[slots, ...]``.
    """
    if indices.numel() == 0:
        return
    if ((indices < 0) | (indices >= min(k_cache.shape[0], v_cache.shape[0]))).any():
        raise ValueError("Invalid KV cache slot")
    keep = indices != reserved_skip_index if reserved_skip_index >= 0 else torch.ones_like(
        indices, dtype=torch.bool
    )
    idx = indices[keep].long()
    k_cache[idx] = k.reshape(indices.numel(), *k_cache.shape[1:])[keep].to(k_cache.dtype)
    v_cache[idx] = v.reshape(indices.numel(), *v_cache.shape[1:])[keep].to(v_cache.dtype)


def paged_attention(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    page_table: torch.Tensor,
    cache_seqlens: torch.Tensor,
    cu_seqlens_q: torch.Tensor,
    scale: float,
) -> torch.Tensor:
    """Causal attention over a paged KV layer, as the attention backends compute it.

    ``attention/fa.py:68-93`` / ``attention/trtllm.py:51-91``: q ``[T, Hq, D]``;
    ``k_cache``/``v_cache`` ``[num_pages, page_size, Hkv, D]`` (NHD, one KV layer);
    ``page_table[b, j]`` is the page holding tokens ``j*page..j*page+page-1`` of
    request ``b``; request ``b`` owns query rows ``cu_seqlens_q[b]:cu_seqlens_q[b+1]``,
    the last of which sits at position ``cache_seqlens[b]-1``. Query row ``i`` of
    ``n`` attends to keys ``0 .. cache_seqlens[b]-n+i`` (causal, cached prefix
    included). Scores ``q.k * scale`` and softmax in fp32, output rounded to
    q's dtype. Rows of a request with no keys are zero.
    """
    t, hq, d = q.shape
    page = k_cache.shape[1]
    hkv = k_cache.shape[2]
    group = hq // hkv
    out = torch.zeros(t, hq, d, dtype=torch.float32)
    bsz = cache_seqlens.numel()
    for b in range(bsz):
        q0, q1 = int(cu_seqlens_q[b]), int(cu_seqlens_q[b + 1])
        n = q1 - q0
        kv_len = int(cache_seqlens[b])
        if n == 0 or kv_len == 0:
            continue
        npages = (kv_len + page - 1) // page
        pages = page_table[b, :npages].long()
        keys = k_cache[pages].reshape(npages * page, hkv, d)[:kv_len].float()
        vals = v_cache[pages].reshape(npages * page, hkv, d)[:kv_len].float()
        keys = keys.repeat_interleave(group, dim=1)  # [kv, Hq, D]
        vals = vals.repeat_interleave(group, dim=1)
        qs = q[q0:q1].float()  # [n, Hq, D]
        scores = torch.einsum("nhd,khd->hnk", qs, keys) * scale
        qpos = torch.arange(n) + (kv_len - n)
        kpos = torch.arange(kv_len)
        mask = kpos[None, :] > qpos[:, None]
        scores = scores.masked_fill(mask[None], float("-inf"))
        probs = torch.softmax(scores, dim=-1)
        out[q0:q1] = torch.einsum("hnk,khd->nhd", probs, vals)
    return out.to(q.dtype)


def cumulative_exit_probability(logits: torch.Tensor, previous: torch.Tensor) -> torch.Tensor:
    """``p' = p + (1 - p) * sigmoid(float(logit))`` in fp32 (``models/looped/exit_gates.py:6-15``)."""
    probability = logits.float().sigmoid()
    prev = previous.float()
    return prev + (1.0 - prev) * probability


def relative_state_change(
    current: torch.Tensor, previous: torch.Tensor, eps: float = 1e-9
) -> torch.Tensor:
    """``||h - h_prev|| / max(||h||, eps)`` over the last dim in fp32 (``exit_gates.py:18-24``)."""
    s = current.float()
    p = previous.float()
    return (s - p).norm(dim=-1) / s.norm(dim=-1).clamp_min(eps)


def ouro_exit_signal(
    hidden: torch.Tensor,
    exit_state: torch.Tensor,
    loop_step: int | torch.Tensor,
    gate_weight: torch.Tensor,
    gate_bias: torch.Tensor,
    threshold: float,
    min_loop_steps: int = 1,
    lookahead_gate: bool = False,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Ouro's exit decision (``models/looped/ouro.py:142-155``).

    ``logit = bf16(h . w_g + b_g)`` (``LinearReplicated`` H->1), cumulative
    probability update in fp32, ``signal = p' >= q and step+1(+1 lookahead) >= min``.
    """
    logits = linear(hidden, gate_weight, gate_bias).squeeze(-1)
    state = cumulative_exit_probability(logits, exit_state)
    exit_depth = loop_step + 1 + int(lookahead_gate)
    signal = (state >= threshold) & (torch.as_tensor(exit_depth) >= min_loop_steps)
    return signal, state


def huginn_exit_signal(
    hidden: torch.Tensor, exit_state: torch.Tensor, threshold: float
) -> tuple[torch.Tensor, torch.Tensor]:
    """Huginn's exit decision (``models/looped/huginn.py:184-194``): relative change ``< q``."""
    return relative_state_change(hidden, exit_state) < threshold, hidden


def embedding(
    ids: torch.Tensor, weight: torch.Tensor, vocab_start: int = 0, vocab_len: int | None = None
) -> torch.Tensor:
    """Vocab-parallel embedding gather (``layers/embedding.py:34-43``).

    With a vocab shard ``[vocab_start, vocab_start+vocab_len)`` ids outside it give zero rows
    (the caller all-reduces across ranks).
    """
    if vocab_len is None:
        return weight[ids.long()]
    mask = (ids < vocab_start) | (ids >= vocab_start + vocab_len)
    local = (ids - vocab_start).masked_fill(mask, 0)
    y = weight[local.long()].clone()
    y[mask] = 0
    return y


def greedy_sample(logits: torch.Tensor) -> torch.Tensor:
    """``torch.argmax(logits, dim=-1)`` (``model_executor/sample.py:108-112``); ties pick the first."""
    return torch.argmax(logits.float(), dim=-1).to(torch.int32)


def softmax_scale(head_dim: int) -> float:
    """``head_dim ** -0.5`` (``attention/fa.py:64``, ``attention/trtllm.py:44``)."""
    return head_dim**-0.5

