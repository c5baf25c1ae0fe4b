"""Full-size parity scenarios at the Ouro-1.4B architecture (BASELINE configs[1] and [2]).

Shared by ``tests/golden/make_fullsize.py`` (which runs the oracle on the CPU and
records ``tests/golden/ouro14b_fullsize.npz``) and ``tests/test_gpu_parity_scale.py``
(which runs the CUDA path on the same seeded weights and inputs).

* CB (configs[1] shapes: 24 layers x 4 loop steps, hidden 2048, 16 heads x 128,
  SwiGLU 5632, vocab 49152, depth-indexed KV in 16-token pages): 4 requests with
  prompts of 256-1024 uniform-random ids, one real prefill, then 4 full-depth greedy
  decode steps (inputs teacher-forced with the bf16 oracle's own greedy tokens).
* CDB (configs[2] shapes: last-exited KV, exit threshold 0.2): 4 requests with prompts
  of 256-1000 ids prefilled at full depth, then the device-routed CDB engine until
  every row has 4 outputs, exit depths prescribed from the 15/25/30/30% mix.

Weights are ``oracle.model.make_weights`` (seeded CPU generator, bf16), so the
fixture generator and the GPU test rebuild the same tensors bit for bit.
"""

from __future__ import annotations

import functools
import math

import numpy as np
import torch

from oracle.model import Batch, LoopedConfig, make_weights

OURO_14B = LoopedConfig(arch="ouro", hidden=2048, heads=16, kv_heads=16, head_dim=128,
                        intermediate=5632, vocab=49152, num_core_layers=24, loop_steps=4,
                        rope_theta=1e6, rms_eps=1e-6, max_position=4096)
OURO_14B_GATED = LoopedConfig(**{**OURO_14B.__dict__, "exit_threshold": 0.2})
SEED = 14
PAGE = 16
CB_PROMPTS = [256, 448, 704, 1024]
CB_DECODE = 4
CDB_PROMPTS = [256, 416, 608, 1000]
CDB_K = 4
CDB_MAX_LEN = 1024
CDB_DEPTH_P = (0.15, 0.25, 0.30, 0.30)
PROBE_STRIDE = 24  # logits compared on every 24th vocabulary column (+ the top 8)
TOPK = 8


@functools.lru_cache(maxsize=1)
def weights() -> dict[str, torch.Tensor]:
    """The seeded bf16 weights of both scenarios (CPU)."""
    return make_weights(OURO_14B_GATED, SEED, dtype=torch.bfloat16)


def cb_prompts() -> list[torch.Tensor]:
    g = torch.Generator().manual_seed(SEED + 6)
    return [torch.randint(0, OURO_14B.vocab, (n,), generator=g, dtype=torch.int32)
            for n in CB_PROMPTS]


def cb_pages() -> tuple[torch.Tensor, int]:
    """[B, max_pages] page ids (random order, page 0 never used) and the pool's page count."""
    per = [math.ceil((n + CB_DECODE + 1) / PAGE) for n in CB_PROMPTS]
    g = torch.Generator().manual_seed(SEED + 5)
    num_pages = sum(per) + 9
    perm = torch.randperm(num_pages - 1, generator=g) + 1
    table = torch.zeros(len(per), max(per), dtype=torch.int32)
    off = 0
    for r, n in enumerate(per):
        table[r, :n] = perm[off:off + n].to(torch.int32)
        off += n
    return table, num_pages


def cb_batch(step: int, ids: torch.Tensor | None, table: torch.Tensor) -> Batch:
    """Step -1: the prefill of every prompt; step k >= 0: decode of the token at position
    prompt_len + k (``ids`` are its input ids)."""
    prompts = cb_prompts()
    lens = torch.tensor(CB_PROMPTS, dtype=torch.int32)
    b = len(prompts)
    if step < 0:
        ids = torch.cat(prompts)
        pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in CB_PROMPTS])
        rows = torch.cat([torch.full((n,), r) for r, n in enumerate(CB_PROMPTS)])
        seq = lens.clone()
        cu = torch.zeros(b + 1, dtype=torch.int32)
        cu[1:] = torch.cumsum(lens, 0)
    else:
        pos = lens + step
        rows = torch.arange(b)
        seq = lens + step + 1
        cu = torch.arange(b + 1, dtype=torch.int32)
    loc = (table[rows, (pos // PAGE).long()] * PAGE + pos % PAGE).to(torch.int32)
    return Batch(ids.to(torch.int32), pos.to(torch.int32), loc, table.clone(),
                 seq.to(torch.int32), cu, step < 0)


def probe_columns(vocab: int) -> torch.Tensor:
    return torch.arange(0, vocab, PROBE_STRIDE)


def bf16_bits(x: torch.Tensor) -> np.ndarray:
    """bf16 values as their uint16 bit patterns (exact, half the bytes of fp32)."""
    return x.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bf16_bits(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)


def logits_match(got: torch.Tensor, probe: torch.Tensor, top_v: torch.Tensor,
                 top_i: torch.Tensor, scale: torch.Tensor, rel_tol: float = 2e-2):
    """Compare full GPU logits [B, V] with the recorded oracle probe columns and top-k.

    Returns (max relative error over the probe and top-k columns, per-row verdicts:
    'agree' / 'near_tie' / 'mismatch' for the greedy token)."""
    got = got.float()
    cols = probe_columns(got.shape[1])
    err = (got[:, cols] - probe).abs().max()
    err = torch.maximum(err, (got.gather(1, top_i.long()) - top_v).abs().max())
    rel = float(err / scale.max())
    verdicts = []
    g = got.argmax(-1)
    for r in range(got.shape[0]):
        if int(g[r]) == int(top_i[r, 0]):
            verdicts.append("agree")
            continue
        hit = (top_i[r] == g[r]).nonzero()
        tie = hit.numel() and float(top_v[r, hit[0, 0]]) >= float(top_v[r, 0]) - rel_tol * float(
            scale[r])
        verdicts.append("near_tie" if tie else "mismatch")
    return rel, verdicts
