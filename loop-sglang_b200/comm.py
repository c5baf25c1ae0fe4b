"""Tensor-parallel communicator plugin stack (python/loopsgl/distributed/{impl,info}.py).

``DistributedCommunicator`` keeps the reference's contract: a class-level plugin
list whose last entry serves ``all_reduce(x) -> x`` (in place, returns the same
tensor) and ``all_gather(x) -> new`` along dim 0 (distributed/impl.py:63-70).
``TorchDistributedImpl`` is the reference's torch.distributed fallback
(impl.py:25-41); it is what the multi-process CPU tests (gloo) exercise.

``B200Communicator`` is the NVLink path (the PyNCCL plugin's place,
impl.py:44-60): one symmetric device buffer per rank, mapped into every peer
with CUDA IPC (handles exchanged over the host process group, as the reference
exchanges its NCCL unique id, kernel/pynccl.py:59-92), and the library's
all-reduce, all-gather and fused row-parallel GEMM + all-reduce on top.
``B200CommImpl`` installs it as a ``DistributedImpl`` plugin.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List

import ctypes

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


class B200Communicator:
    """NVLink communicator of one node (one process per GPU, same calls on every rank).

    ``max_elems`` bounds the bf16 elements of one all-reduce (rows x cols) and half
    the bytes of one rank's all-gather contribution. Construction is collective over
    ``group`` (any backend that can all-gather Python objects: gloo or nccl).
    """

    def __init__(self, rank: int, world: int, max_elems: int, group=None) -> None:
        from ._lib import LSB_IPC_HANDLE_BYTES, call, lib

        self.rank, self.world = rank, world
        self._group = group
        self.max_elems = (max_elems + 7) // 8 * 8
        self._lib = lib()
        self._call = call
        nbytes = int(self._lib.lsb_comm_buffer_bytes(self.max_elems))
        local = ctypes.c_void_p()
        call("lsb_comm_alloc", nbytes, ctypes.byref(local))
        self._local = local.value
        handle = (ctypes.c_ubyte * LSB_IPC_HANDLE_BYTES)()
        call("lsb_ipc_handle", self._local, handle)
        handles: list = [None] * world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened: list[int] = []
        ptrs = (ctypes.c_void_p * world)()
        for r in range(world):
            if r == rank:
                ptrs[r] = self._local
                continue
            h = (ctypes.c_ubyte * LSB_IPC_HANDLE_BYTES).from_buffer_copy(handles[r])
            peer = ctypes.c_void_p()
            call("lsb_ipc_open", h, ctypes.byref(peer))
            self._opened.append(peer.value)
            ptrs[r] = peer.value
        comm = ctypes.c_void_p()
        call("lsb_comm_create", rank, world, ptrs, self.max_elems, ctypes.byref(comm))
        self._comm = comm.value
        # every rank has mapped every buffer before anyone sends
        dist.barrier(group=group)

    @staticmethod
    def _stream() -> int:
        return torch.cuda.current_stream().cuda_stream

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        """In-place bf16 sum over the ranks (rows of the last dimension)."""
        if x.dtype != torch.bfloat16 or x.dim() < 1 or x.stride(-1) != 1:
            raise ValueError("all_reduce needs a bf16 tensor with unit last-dim stride")
        cols = x.shape[-1]
        rows = x.numel() // cols if cols else 0
        ld = x.stride(-2) if x.dim() > 1 else cols
        if x.dim() > 2 and not x.is_contiguous():
            raise ValueError("all_reduce needs a contiguous tensor beyond two dimensions")
        self._call("lsb_allreduce", self._comm, x.data_ptr(), rows, cols, ld, self._stream())
        return x

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        """Concatenation of every rank's ``x`` along dim 0 (a new tensor)."""
        x = x.contiguous()
        nbytes = x.numel() * x.element_size()
        if nbytes % 16:
            raise ValueError("all_gather needs a multiple of 16 bytes per rank")
        shape = list(x.shape)
        shape[0] *= self.world
        out = torch.empty(shape, dtype=x.dtype, device=x.device)
        self._call("lsb_allgather", self._comm, out.data_ptr(), x.data_ptr(), nbytes,
                   self._stream())
        return out

    def gemm_allreduce(self, x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        """Row-parallel linear: ``sum_r x_r . w_r^T (+ bias per rank)`` in one kernel."""
        from ._lib import LSB_EPI_BIAS, LSB_EPI_NONE

        m, k = x.shape
        n = w.shape[0]
        if w.shape[1] != k or x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
            raise ValueError("gemm_allreduce: bf16 x[M, K] and w[N, K] expected")
        if x.stride(1) != 1 or w.stride(1) != 1:
            raise ValueError("gemm_allreduce: unit column strides expected")
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device) if out is None else out
        epi = LSB_EPI_BIAS if bias is not None else LSB_EPI_NONE
        self._call("lsb_gemm_allreduce", self._comm, out.data_ptr(), out.stride(0), x.data_ptr(),
                   x.stride(0), w.data_ptr(), w.stride(0),
                   None if bias is None else bias.data_ptr(), m, n, k, epi, self._stream())
        return out

    def close(self) -> None:
        """Release the communicator (collective: every rank calls it after its last call)."""
        if getattr(self, "_comm", None) is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self._group)  # no peer writes into this rank's buffer any more
        self._call("lsb_comm_destroy", self._comm)
        self._comm = None
        for p in self._opened:
            self._call("lsb_ipc_close", p)
        self._opened = []
        self._call("lsb_comm_free", self._local)


class B200CommImpl(DistributedImpl):
    """The reference's plugin seam (impl.py:63-64) served by ``B200Communicator``."""

    def __init__(self, comm: B200Communicator) -> None:
        self.comm = comm

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return self.comm.all_reduce(x)

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        return self.comm.all_gather(x)
