"""The reference's communicator and attention-backend seams driving this package's
plugins, on the CPU.

* Two gloo ranks: ``comm.install`` appends a ``B200CommImpl`` to the reference's own
  ``DistributedCommunicator.plugins`` (python/loopsgl/distributed/impl.py:63-70); the
  reference's unmodified ``LinearOProj`` (layers/linear.py:92-107) and
  ``DistributedCommunicator`` then all-reduce and all-gather through it, with the known
  answers of the reference's communicator test (tests/kernel/test_comm.py:96-150).
  The plugin wraps a host stand-in of ``B200Communicator`` (same two methods, over gloo):
  what is checked is the seam, which needs no GPU; the NVLink data path is checked on
  two GPUs (``test_gpu_tp.py``).
* ``plugins.B200AttnBackend`` is a subclass of the reference's ``BaseAttnBackend`` and
  ``plugins.register()`` makes ``create_attention_backend("b200", config)``
  (attention/__init__.py:19-60) return it, reading the pool and page size from the
  reference's global ``Context`` as its own backends do.

Both run in fresh processes with the reference's ``python/`` directory importable, and
skip when no Loop-SGLang checkout is available.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import reference_python

REF = reference_python()
pytestmark = pytest.mark.skipif(REF is None, reason="no Loop-SGLang checkout to import")
ROOT = str(Path(__file__).resolve().parents[1])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _HostComm:
    """Host stand-in of ``B200Communicator``'s collective methods over the gloo group."""

    def __init__(self, rank: int, world: int) -> None:
        self.rank, self.world, self.calls = rank, world, 0

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        self.calls += 1
        dist.all_reduce(x)
        return x

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        self.calls += 1
        out = [torch.empty_like(x) for _ in range(self.world)]
        dist.all_gather(out, x.contiguous())
        return torch.cat(out)


def _comm_worker(rank: int, world: int, port: int, ref: str, q) -> None:
    sys.path[:0] = [ref, ROOT]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from loopsgl.distributed import DistributedCommunicator, set_tp_info
        from loopsgl.distributed.impl import DistributedImpl
        from loopsgl.layers.linear import LinearOProj

        from __graft_entry__ import load_package

        load_package()
        from loop_sglang_b200 import comm as C

        set_tp_info(rank, world)
        host = _HostComm(rank, world)
        impl = C.install(host)
        ok = isinstance(impl, DistributedImpl) and DistributedCommunicator.plugins[-1] is impl
        ok &= C.active() is host and C.tp_size() == world
        ref_comm = DistributedCommunicator()
        x = torch.ones(64)
        for _ in range(3):
            ref_comm.all_reduce(x)
        ok &= bool(torch.all(x == world ** 3))
        src = torch.full((8,), float(rank))
        ok &= bool(torch.equal(ref_comm.all_gather(src),
                               torch.arange(world, dtype=torch.float).repeat_interleave(8)))
        # the reference's own row-parallel linear: local columns, summed through the plugin
        g = torch.Generator().manual_seed(5)
        w_full = torch.randn(4, 8 * world, generator=g)
        x_full = torch.randn(3, 8 * world, generator=g)
        op = LinearOProj(8 * world, 4, has_bias=False)
        op.weight = w_full[:, rank * 8:(rank + 1) * 8].contiguous()
        y = op.forward(x_full[:, rank * 8:(rank + 1) * 8].contiguous())
        ok &= bool(torch.allclose(y, x_full @ w_full.t(), atol=1e-5))
        calls = host.calls
        C.uninstall(impl)
        ok &= impl not in DistributedCommunicator.plugins and C.active() is None
        q.put((rank, bool(ok), calls))
    except Exception as exc:  # reported to the parent
        q.put((rank, repr(exc), -1))
    finally:
        dist.destroy_process_group()


def test_communicator_plugin_through_reference_stack() -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_comm_worker, args=(r, 2, port, REF, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = {}
    for _ in procs:
        rank, ok, calls = q.get(timeout=5)
        results[rank] = (ok, calls)
    assert all(p.exitcode == 0 for p in procs)
    # 3 all-reduces + 1 all-gather + the LinearOProj all-reduce went through the plugin
    assert results == {0: (True, 5), 1: (True, 5)}, results


def _backend_worker(ref: str, q) -> None:
    sys.path[:0] = [ref, ROOT]
    try:
        from loopsgl.attention import SUPPORTED_ATTENTION_BACKENDS, create_attention_backend
        from loopsgl.attention.base import BaseAttnBackend, BaseAttnMetadata
        from loopsgl.core import Context, set_global_ctx

        from __graft_entry__ import load_package

        load_package()
        from loop_sglang_b200 import plugins as P

        ok = P.HAVE_LOOPSGL and issubclass(P.B200AttnBackend, BaseAttnBackend)
        ok &= issubclass(P.B200Metadata, BaseAttnMetadata)
        ok &= P.register() and P.register()  # idempotent
        ok &= "b200" in SUPPORTED_ATTENTION_BACKENDS.supported_names()

        class _Pool:  # a last-exited pool's attributes the backend reads at construction
            slot_map = torch.zeros(1, 1, dtype=torch.int32)
            core_start, core_end, num_kv_heads = 0, 4, 2

        class _Cfg:
            head_dim, num_kv_heads, num_qo_heads = 64, 2, 8

        ctx = Context(page_size=1)
        ctx.kv_cache = _Pool()
        ctx.page_table = torch.zeros(2, 32, dtype=torch.int32)
        set_global_ctx(ctx)
        be = create_attention_backend("b200", _Cfg())
        ok &= isinstance(be, P.B200AttnBackend) and be.last_exited and be.page_size == 1
        ok &= be.kvcache is ctx.kv_cache and abs(be.scale - 64 ** -0.5) < 1e-12
        q.put(bool(ok))
    except Exception as exc:  # reported to the parent
        q.put(repr(exc))


def test_attention_backend_registers_with_reference() -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_backend_worker, args=(REF, q))
    p.start()
    p.join(timeout=120)
    res = q.get(timeout=5)
    assert p.exitcode == 0
    assert res is True, res
