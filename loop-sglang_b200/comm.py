"""Tensor-parallel communicator plugin stack (python/loopsgl/distributed/{impl,info}.py).

``DistributedCommunicator`` keeps the reference's contract: a class-level plugin
list whose last entry serves ``all_reduce(x) -> x`` (in place, returns the same
tensor) and ``all_gather(x) -> new`` along dim 0 (distributed/impl.py:63-70).
``TorchDistributedImpl`` is the reference's torch.distributed fallback
(impl.py:25-41); it is what the multi-process CPU tests (gloo) exercise.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class DistributedInfo:
    """distributed/info.py:7-18."""

    rank: int
    size: int

    def is_primary(self) -> bool:
        return self.rank == 0


_TP_INFO: DistributedInfo | None = None


def set_tp_info(rank: int, size: int) -> None:
    """info.py:21-25 (raises if already set)."""
    global _TP_INFO
    if _TP_INFO is not None:
        raise RuntimeError("TP info has been set")
    _TP_INFO = DistributedInfo(rank, size)


def reset_tp_info() -> None:
    global _TP_INFO
    _TP_INFO = None


def tp_info() -> DistributedInfo:
    """``get_tp_info`` with a TP=1 default when nothing was set."""
    return _TP_INFO if _TP_INFO is not None else DistributedInfo(0, 1)


class DistributedImpl:
    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError


class TorchDistributedImpl(DistributedImpl):
    """impl.py:25-41."""

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if dist.get_world_size() == 1:
            return x
        dist.all_reduce(x, op=dist.ReduceOp.SUM)
        return x

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        world = dist.get_world_size()
        if world == 1:
            return x
        shape = list(x.shape)
        shape[0] *= world
        out = torch.empty(shape, dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x)
        return out


class DistributedCommunicator:
    """impl.py:63-70: the last plugin wins."""

    plugins: List[DistributedImpl] = [TorchDistributedImpl()]

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return self.plugins[-1].all_reduce(x)

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        return self.plugins[-1].all_gather(x)


def lm_head_gather(logits_local: torch.Tensor, vocab: int) -> torch.Tensor:
    """The LM-head all-gather + permute of layers/embedding.py:99-111."""
    comm = DistributedCommunicator()
    size = tp_info().size
    if size == 1:
        return logits_local
    bs, local = logits_local.shape
    out = comm.all_gather(logits_local)
    if bs == 1:
        return out.view(1, -1)[:, :vocab]
    out = out.view(size, bs, local).permute(1, 0, 2).contiguous().view(bs, size * local)
    return out[:, :vocab]
