"""NVLink communicator of a tensor-parallel node, and its plugin for the reference's
communicator stack (python/loopsgl/distributed/impl.py:16-70).

``B200Communicator`` is the NVLink path (the PyNCCL plugin's place, impl.py:44-60):
one symmetric device buffer per rank, mapped into every peer with CUDA IPC (handles
exchanged over the host process group, as the reference exchanges its NCCL unique
id, kernel/pynccl.py:59-92), and the library's all-reduce, all-gather and fused
row-parallel GEMM + all-reduce on top.

``B200CommImpl`` is the plugin. When ``loopsgl`` is importable it subclasses the
reference's own ``DistributedImpl``, and ``install`` appends it to the reference's
``DistributedCommunicator.plugins`` (the last plugin wins, impl.py:63-70), so the
reference's row-parallel linears, vocab-parallel embedding and LM head all-reduce and
all-gather through it unchanged. ``install`` also makes it this package's active
communicator (``active``), which the drop-in linears of ``plugins`` use for the fused
GEMM + all-reduce.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

try:  # the reference's plugin base class and communicator stack, when installed
    from loopsgl.distributed.impl import DistributedCommunicator as RefCommunicator
    from loopsgl.distributed.impl import DistributedImpl as _PluginBase
except ImportError:
    RefCommunicator = None
    _PluginBase = object


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

    def set_protocol(self, mode: int) -> None:
        """All-reduce protocol of later calls (collective: every rank sets the same): 0
        automatic (one hop for two ranks, and for up to four while the bytes stay small), 1 one
        hop (at most 4 ranks), 2 two hops via region owners. Every rank finishes its calls in
        flight first (device synchronise + barrier), so the switch lands between calls."""
        torch.cuda.synchronize()
        dist.barrier(group=self._group)
        self._call("lsb_comm_set_protocol", self._comm, int(mode))

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


class B200CommImpl(_PluginBase):
    """The reference's plugin seam (``DistributedImpl``, impl.py:16-22) served by
    ``B200Communicator``: ``all_reduce(x) -> x`` in place, ``all_gather(x) -> new``
    along dim 0."""

    def __init__(self, comm: B200Communicator) -> None:
        self.comm = comm

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return self.comm.all_reduce(x)

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        return self.comm.all_gather(x)

    def __repr__(self) -> str:
        return f"B200CommImpl(rank={self.comm.rank}, world={self.comm.world})"

    # identity, not the field-wise equality of the reference's dataclass base: two
    # plugins over different communicators are different plugins
    __eq__ = object.__eq__
    __hash__ = object.__hash__


_ACTIVE: B200CommImpl | None = None


def install(comm: B200Communicator) -> B200CommImpl:
    """Make ``comm`` the communicator of this process: appended to the reference's
    ``DistributedCommunicator.plugins`` when ``loopsgl`` is importable, and the one the
    drop-in linears of ``plugins`` use."""
    global _ACTIVE
    impl = B200CommImpl(comm)
    if RefCommunicator is not None:
        RefCommunicator.plugins.append(impl)
    _ACTIVE = impl
    return impl


def uninstall(impl: B200CommImpl) -> None:
    """Undo ``install`` (before the communicator is closed)."""
    global _ACTIVE
    if RefCommunicator is not None and impl in RefCommunicator.plugins:
        RefCommunicator.plugins.remove(impl)
    if _ACTIVE is impl:
        _ACTIVE = None


def active() -> B200Communicator | None:
    """The installed communicator, or None."""
    return None if _ACTIVE is None else _ACTIVE.comm


def tp_size() -> int:
    """Tensor-parallel size: the reference's ``get_tp_info`` when it is set
    (distributed/info.py:21-37), else the installed communicator's world, else 1."""
    try:
        from loopsgl.distributed import try_get_tp_info

        info = try_get_tp_info()
        if info is not None:
            return info.size
    except ImportError:
        pass
    comm = active()
    return comm.world if comm is not None else 1


def reference_all_reduce(x: torch.Tensor) -> torch.Tensor:
    """All-reduce through the reference's communicator stack (its last plugin)."""
    if RefCommunicator is None:
        raise RuntimeError("tensor parallelism without an installed communicator")
    return RefCommunicator().all_reduce(x)
