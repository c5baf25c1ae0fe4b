"""The communicator plugin stack across two CPU ranks (gloo), with the known answers of
the reference's all-reduce / all-gather test (tests/kernel/test_comm.py:96-150)."""

from __future__ import annotations

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q) -> None:
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    from __graft_entry__ import load_package

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # the package imports the CUDA library lazily; comm itself is host logic
        load_package()
        from loop_sglang_b200.comm import DistributedCommunicator, lm_head_gather, set_tp_info

        set_tp_info(rank, world)
        comm = DistributedCommunicator()
        x = torch.ones(64)
        for _ in range(3):
            comm.all_reduce(x)
        ok = bool(torch.all(x == world ** 3))
        x = torch.full((64,), float(rank))
        ok &= bool(torch.all(comm.all_reduce(x) == world * (world - 1) / 2))
        src = torch.full((8,), float(rank))
        ok &= bool(torch.equal(comm.all_gather(src),
                               torch.arange(world, dtype=torch.float).repeat_interleave(8)))
        logits = torch.arange(6, dtype=torch.float).view(2, 3) + 10 * rank
        full = lm_head_gather(logits, vocab=5)
        expect = torch.cat([torch.arange(6, dtype=torch.float).view(2, 3) + 10 * r
                            for r in range(world)], dim=1)[:, :5]
        ok &= bool(torch.equal(full, expect))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_communicator_two_ranks() -> None:
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = dict(q.get(timeout=5) for _ in procs)
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: True, 1: True}
