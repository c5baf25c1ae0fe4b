"""Tensor parallelism on two GPUs: all-reduce, all-gather and the fused
row-parallel GEMM + all-reduce, each against an exact host-side restatement, and
the Ouro looped decoder sharded over both ranks (CB under all three KV policies,
CDB phases) against the oracle.

Every rank generates every rank's inputs from per-rank seeds, so each can build
the expected result itself: the sum of the ranks' bf16 partials in rank order in
fp32, rounded once -- bit-exact up to 256 rows, where the fused kernel's partial is
the same tcgen05 GEMM (same plan, same accumulation order) as ``ops.gemm`` on that
rank's shard. The fused result is also checked against an fp32 torch reference of the
unsharded product within bf16 tolerance. Runs as two child processes (one per
GPU); skipped with fewer than two GPUs.
"""

from __future__ import annotations

import datetime
import os
import socket
import sys
import traceback

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = [pytest.mark.gpu, pytest.mark.timeout(600)]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bf(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16)


def _worker(rank: int, world: int, port: int, errq) -> None:
    try:
        sys.path.insert(0, ROOT)
        import torch.distributed as dist

        import __graft_entry__

        __graft_entry__.load_package()
        from loop_sglang_b200 import comm as C
        from loop_sglang_b200 import ops

        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=120))
        dev = torch.device("cuda", rank)
        cm = C.B200Communicator(rank, world, max_elems=256 * 4096)

        def gen(seed: int) -> torch.Generator:
            return torch.Generator().manual_seed(seed)

        # both all-reduce protocols (two hops via owners, one hop), then the default; calls
        # alternate between them on the same buffers and epochs
        for proto in (2, 1, 0):
            cm.set_protocol(proto)
            # all-reduce: bit-exact against the rank-ordered fp32 sum, on repeated calls
            for it in range(3):
                for (m, n) in [(1, 2048), (143, 2048), (7, 100), (64, 4096)]:
                    parts = [_bf(torch.randn(m, n, generator=gen(1000 * it + 10 * r + n))) for r in range(world)]
                    x = parts[rank].to(dev)
                    cm.all_reduce(x)
                    want = torch.zeros(m, n)
                    for p in parts:
                        want += p.float()
                    assert torch.equal(x.cpu(), _bf(want)), f"all_reduce {m}x{n} call {it}"

            # all-gather: exact concatenation
            for it in range(3):
                parts = [_bf(torch.randn(5, 64, generator=gen(77 + it * 10 + r))) for r in range(world)]
                got = cm.all_gather(parts[rank].to(dev))
                assert torch.equal(got.cpu(), torch.cat(parts)), f"all_gather call {it}"

            # fused row-parallel GEMM + all-reduce (o_proj / down_proj shards, ragged shapes, bias)
            # (1100, 2048, 2048): more rows than the communicator's buffer takes at once (512 x
            # 2048), so the call runs as several complete launches of resident tiles
            shapes = [(143, 2048, 2048), (143, 2048, 5632), (1, 2048, 2048), (33, 200, 192),
                      (256, 2048, 512), (1100, 2048, 2048)]
            for it in range(2):
                for (m, n, k_full) in shapes:
                    k = k_full // world
                    xs = [_bf(torch.randn(m, k, generator=gen(5 + r + 100 * it))) for r in range(world)]
                    ws = [_bf(torch.randn(n, k, generator=gen(50 + r)) * 0.05) for r in range(world)]
                    bias = _bf(torch.randn(n, generator=gen(9)) * 0.1) if n == 200 else None
                    b_dev = bias.to(dev) if bias is not None else None
                    got = cm.gemm_allreduce(xs[rank].to(dev), ws[rank].to(dev), b_dev)
                    # exact: every rank's partial through the same single-GPU kernel (up to 256
                    # rows both take the same tile plan; larger calls run as several launches
                    # with the fused variant's one-wave plan, checked by tolerance below)
                    if m <= 256:
                        want = torch.zeros(m, n)
                        for r in range(world):
                            part = ops.linear(xs[r].to(dev), ws[r].to(dev), b_dev)
                            want += part.float().cpu()
                        assert torch.equal(got.cpu(), _bf(want)), \
                            f"gemm_allreduce {m}x{n}x{k_full} call {it}"
                    ref = sum(xs[r].float() @ ws[r].float().t() for r in range(world))
                    if bias is not None:
                        ref = ref + world * bias.float()
                    # bf16 partials of magnitude ~|ref|max are rounded before the sum (as the
                    # reference's per-rank F.linear outputs are), so the absolute error scales
                    # with the largest output, not with each element
                    scale = float(ref.abs().max())
                    torch.testing.assert_close(got.float().cpu(), ref, rtol=2e-2, atol=1e-2 * scale)
        torch.cuda.synchronize()
        assert ops.device_error_word(reset=True) == 0

        # the whole looped decoder sharded over the two ranks, against the oracle
        sys.path.insert(0, os.path.join(ROOT, "tests"))
        from replay import gpu_replay_cb, gpu_replay_cdb, replay_cb, replay_cdb
        from test_gpu_model import greedy_agrees, rel_err

        for name in ("ouro_cb_depth_indexed", "ouro_cb_shared", "ouro_cb_last_exited"):
            _, got = gpu_replay_cb(name, comm=cm)
            # the oracle with the two ranks' rounding points (each rank's row-parallel
            # partial rounded to bf16 before the sum, as the reference's F.linear + NCCL)
            _, ref, _ = replay_cb(name, dtype=torch.bfloat16, tp=world)
            for prefix, logits in got.items():
                assert rel_err(logits, ref[prefix]) < 2e-2, (name, prefix)
                assert greedy_agrees(logits, ref[prefix]), (name, prefix)
        for name in ("ouro_cdb_last_exited", "ouro_cdb_shared"):
            fx, got = gpu_replay_cdb(name, comm=cm)
            _, ref = replay_cdb(name, dtype=torch.bfloat16, tp=world)
            assert rel_err(got["prefill_logits"], ref["prefill_logits"]) < 2e-2, name
            k = 0
            while f"core{k}_rows" in fx:
                assert rel_err(got[f"core{k}_hidden"], ref[f"core{k}_hidden"]) < 2e-2, (name, k)
                p = ref[f"core{k}_exit"]
                sure = (p - 0.5).abs() > 1e-3
                assert torch.equal(got[f"core{k}_gates"][sure], ref[f"core{k}_gates"][sure])
                k += 1
            assert rel_err(got["coda_logits"], ref["coda_logits"]) < 2e-2, name
            assert greedy_agrees(got["coda_logits"], ref["coda_logits"]), name
        torch.cuda.synchronize()
        assert ops.device_error_word(reset=True) == 0
        cm.close()
        dist.destroy_process_group()
    except BaseException:  # report to the parent, which fails the test
        errq.put(f"rank {rank}:\n{traceback.format_exc()}")
        raise


def test_two_gpu_exchange() -> None:
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=540)
    for p in procs:
        if p.is_alive():
            p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not errors, "\n".join(errors)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
