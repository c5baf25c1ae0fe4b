"""Single-kernel timing at the decode shapes of the looped decoder.

Runs one kernel of the library on its own, at one shape, with inputs larger than
the L2 cache, and prints one JSON line per shape with the device time per launch
and the algorithmic bytes moved per second. The launches are captured into a
CUDA graph so the host launch rate does not limit short kernels, and timed with
CUDA events on the capturing stream after warm-up replays.

    python loop-sglang_b200/kernel_bench.py attention --rows 143 --ctx 1448
    python loop-sglang_b200/kernel_bench.py gemm --tokens 143 --shape qkv o gate_up down
    python -m torch.distributed.run --nproc-per-node 2 loop-sglang_b200/kernel_bench.py \
        gemm_ar --tokens 256     # row-parallel GEMM fused with its all-reduce, per rank
    python loop-sglang_b200/kernel_bench.py snapshot --tokens 2048   # retraction copy
    python loop-sglang_b200/kernel_bench.py norm --rows 263          # Ouro sandwich norm

It is also the small case for profiler captures of one kernel (one KV layer of a
few GB instead of the whole pool that the decode benchmark holds).
"""

from __future__ import annotations

import argparse
import importlib.util
import json
import math
import pathlib
import sys

import torch


def _package():
    """Import this directory as the ``loop_sglang_b200`` package when run as a script."""
    if "loop_sglang_b200" in sys.modules:
        return sys.modules["loop_sglang_b200"]
    here = pathlib.Path(__file__).resolve().parent
    spec = importlib.util.spec_from_file_location(
        "loop_sglang_b200", here / "__init__.py", submodule_search_locations=[str(here)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["loop_sglang_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


# Ouro-1.4B per-layer GEMMs at TP1: (out rows N, reduction K, SwiGLU epilogue)
OURO_GEMMS = {
    "qkv": (3 * 2048, 2048, False),
    "o": (2048, 2048, False),
    "gate_up": (2 * 5632, 2048, True),
    "down": (2048, 5632, False),
    "lm_head": (49152, 2048, False),
}

L2_BYTES = 126 * 2**20


def _time_graph(fn, reps: int, warmup: int = 3) -> float:
    """Microseconds per call of ``fn`` (reps calls captured in one graph)."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(2):
            fn(0)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(reps):
            fn(i)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        graph.replay()
        end.record(stream)
    end.synchronize()
    ms = start.elapsed_time(end)
    del graph
    return ms * 1e3 / reps


def bench_attention(args, ops) -> dict:
    """One decode launch of paged attention over one depth-indexed KV layer."""
    dev = torch.device("cuda", 0)
    gen = torch.Generator().manual_seed(args.seed)
    rows, hq, hkv, d, page = args.rows, args.heads, args.kv_heads, args.head_dim, args.page
    if args.ctx_spread > 0:
        ctx = torch.randint(max(1, args.ctx - args.ctx_spread), args.ctx + args.ctx_spread + 1,
                            (rows,), generator=gen)
    else:
        ctx = torch.full((rows,), args.ctx)
    pages_per = (ctx + page - 1) // page
    # with --shared-prefix P, row r's first P tokens are group (r % groups)'s shared pages
    sp = args.shared_prefix // page if args.shared_prefix else 0
    groups = args.groups if sp else 0
    own = pages_per - sp
    num_pages = int(own.sum()) + groups * sp + 1
    perm = torch.randperm(num_pages - 1, generator=gen) + 1
    table = torch.zeros(rows, int(pages_per.max()), dtype=torch.int32)
    off = groups * sp
    for r in range(rows):
        if sp:
            g = r % groups
            table[r, :sp] = perm[g * sp:(g + 1) * sp].to(torch.int32)
        n = int(own[r])
        table[r, sp:sp + n] = perm[off:off + n].to(torch.int32)
        off += n
    slots = num_pages * page
    kv = torch.empty(2, slots, hkv, d, dtype=torch.bfloat16, device=dev).normal_()
    q = torch.randn(rows, hq, d, dtype=torch.bfloat16, device=dev)
    out = torch.empty_like(q)
    table_d = table.to(dev)
    seqlens = ctx.to(torch.int32).to(dev)
    cu = torch.arange(rows + 1, dtype=torch.int32, device=dev)
    max_seqlen = int(ctx.max())
    scale = d ** -0.5

    def launch(_i):
        ops.paged_attention(q, kv[0], kv[1], table_d, seqlens, cu, page, max_seqlen, scale,
                            hkv, out=out)

    us = _time_graph(launch, args.reps)
    extra = {}
    if sp:
        # the rows' groups as the engine finds them, each group's prefix read once
        from loop_sglang_b200.prefix_cache import find_shared_prefixes

        grp = find_shared_prefixes(table.numpy(), ctx.numpy(), page, dev)

        def launch_shared(_i):
            ops.paged_attention_shared_prefix(q, kv[0], kv[1], table_d, seqlens, cu, page,
                                              max_seqlen, scale, hkv, grp, out=out)

        extra = {"us_unshared": round(us, 2),
                 "prefix_groups": 0 if grp is None else grp.num_groups}
        us = _time_graph(launch_shared, args.reps)
    if args.vs_trtllm:
        extra.update(_trtllm_decode_arm(args, q, kv, table_d, seqlens, max_seqlen, scale,
                                        num_pages, out, ctx))
    kv_tokens = int(ctx.sum()) - (rows - min(rows, groups)) * sp * page  # shared pages once
    kv_bytes = kv_tokens * hkv * d * 2 * 2
    nbytes = kv_bytes + rows * hq * d * 2 * 2
    return {"kernel": "paged_attention", "rows": rows, "mean_ctx": float(ctx.float().mean()),
            "heads": hq, "kv_heads": hkv, "head_dim": d, "page_size": page,
            "kv_layer_bytes": slots * hkv * d * 2 * 2, "algorithmic_bytes": nbytes,
            "shared_prefix": sp * page, "groups": groups, **extra,
            "us": round(us, 2), "GBps": round(nbytes / us / 1e3, 1),
            "per_row_GBps": round((int(ctx.sum()) * hkv * d * 4 + rows * hq * d * 4) / us / 1e3, 1)}


def _trtllm_decode_arm(args, q, kv, table_d, seqlens, max_seqlen, scale, num_pages, out,
                       ctx) -> dict:
    """The reference's sm100 decode call on the same pool, page table and queries.

    The reference's TensorRT-LLM backend (attention/trtllm.py:80-91) calls FlashInfer's
    ``trtllm_batch_decode_with_kv_cache`` with the layer's (k, v) pages in NHD layout
    ([pages, page_size, kv_heads, head_dim], the same bytes as this library's
    [slots, kv_heads, head_dim] pool), bmm1_scale = head_dim ** -0.5, bmm2_scale = 1 and a
    zeroed 128 MiB workspace. Returns its time per launch (same graph timing) and the
    largest difference from this library's output; reads every row's own keys (the call
    has no shared-prefix form).
    """
    from flashinfer.decode import trtllm_batch_decode_with_kv_cache

    page, hkv, d = args.page, args.kv_heads, args.head_dim
    k_pages = kv[0].view(num_pages, page, hkv, d)
    v_pages = kv[1].view(num_pages, page, hkv, d)
    workspace = torch.zeros(128 * 2**20, dtype=torch.uint8, device=q.device)
    ref_out = torch.empty_like(q)

    def launch_ref(_i):
        trtllm_batch_decode_with_kv_cache(
            query=q, kv_cache=(k_pages, v_pages), workspace_buffer=workspace,
            block_tables=table_d, seq_lens=seqlens, max_seq_len=max_seqlen,
            bmm1_scale=scale, bmm2_scale=1.0, kv_layout="NHD", out=ref_out,
            out_dtype=q.dtype)

    try:
        us = _time_graph(launch_ref, args.reps)
    except Exception as exc:  # the library may lack a kernel for this shape
        return {"trtllm": f"unavailable: {type(exc).__name__}: {str(exc).splitlines()[0][:160]}"}
    diff = (ref_out.float() - out.float()).abs().max().item()
    kv_bytes = int(ctx.sum()) * hkv * d * 2 * 2
    nbytes = kv_bytes + q.shape[0] * q.shape[1] * d * 2 * 2
    return {"trtllm_us": round(us, 2), "trtllm_GBps": round(nbytes / us / 1e3, 1),
            "trtllm_max_abs_diff": round(diff, 5),
            "out_max_abs": round(out.float().abs().max().item(), 4)}


def tp_shape(name: str, tp: int) -> tuple[int, int, bool]:
    """Per-rank GEMM shape under the reference's tensor-parallel split."""
    n, k, swiglu = OURO_GEMMS[name]
    if name in ("qkv", "gate_up", "lm_head"):
        return n // tp, k, swiglu  # column-parallel: output rows split
    return n, k // tp, swiglu  # row-parallel: reduction split


def bench_gemm(args, ops, name: str) -> dict:
    """One ``y = x . w^T`` launch with the weight streamed from HBM (rotating copies)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    n, k, swiglu = tp_shape(name, args.tp)
    if args.n:
        n = args.n
    if args.k:
        k = args.k
    m = args.tokens
    w_bytes = n * k * 2
    copies = max(2, math.ceil(2 * L2_BYTES / w_bytes))
    ws = [torch.randn(n, k, dtype=torch.bfloat16, device=dev).mul_(0.02) for _ in range(copies)]
    x = torch.randn(m, k, dtype=torch.bfloat16, device=dev)
    cols = n // 2 if swiglu else n
    y = torch.empty(m, cols, dtype=torch.bfloat16, device=dev)
    epi = ops.LSB_EPI_SWIGLU if swiglu else ops.LSB_EPI_NONE

    def launch(i):
        ops.gemm(x, ws[i % copies], None, epi, out=y)

    if args.rope and name == "qkv":  # the QKV projection with RoPE + KV store fused
        hq, hkv, d = n // 3 // 128, n // 3 // 128, 128
        pos = torch.randint(0, 4000, (m,), dtype=torch.int32, device=dev)
        cs = torch.randn(4096, d, device=dev)
        loc = torch.randperm(2 * m, device=dev)[:m].to(torch.int32) + 1
        kc = torch.empty(2 * m + 2, hkv * d, dtype=torch.bfloat16, device=dev)
        vc = torch.empty_like(kc)

        def launch(i):  # noqa: F811
            ops.gemm_rope_store(x, ws[i % copies], pos, cs, hq, hkv, d, kc, vc, loc, out=y)

    if args.cublas_only:  # a process that launches only cuBLAS's kernel (profiler captures)
        yc = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        us_c = _time_graph(lambda i: torch.matmul(x, ws[i % copies].t(), out=yc), args.reps)
        return {"kernel": "cublas", "shape": name, "tokens": m, "N": n, "K": k,
                "us_cublas": round(us_c, 2)}
    us = _time_graph(launch, args.reps)
    nbytes = w_bytes + m * k * 2 + m * cols * 2
    flops = 2.0 * m * n * k
    out = {"kernel": "gemm", "shape": name, "tp": args.tp, "tokens": m, "N": n, "K": k,
           "swiglu": swiglu,
           "weight_copies": copies, "algorithmic_bytes": nbytes, "us": round(us, 2),
           "GBps": round(nbytes / us / 1e3, 1), "TFLOPs": round(flops / us / 1e6, 1)}
    if args.cublas:
        # the reference's GPU path for the same product: F.linear (cuBLAS bf16), and for
        # gate_up its separate SiLU*mul (models/utils.py:45-50); same rotating weights
        import torch.nn.functional as F

        yc = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
        us_c = _time_graph(lambda i: torch.matmul(x, ws[i % copies].t(), out=yc), args.reps)
        out["us_cublas"] = round(us_c, 2)
        if swiglu:
            half = n // 2

            def ref_swiglu(i):
                torch.matmul(x, ws[i % copies].t(), out=yc)
                torch.mul(F.silu(yc[:, :half]), yc[:, half:], out=y)

            out["us_cublas_plus_silu_mul"] = round(_time_graph(ref_swiglu, args.reps), 2)
    return out


def bench_gemm_ar(args, ops, comm, name: str, nccl=None) -> dict:
    """One row-parallel shard GEMM fused with its NVLink all-reduce (every rank runs it),
    next to the same local GEMM alone; the max over ranks of the per-launch time."""
    import torch.distributed as dist

    dev = torch.device("cuda", torch.cuda.current_device())
    tp = comm.world
    n, k, _ = tp_shape(name, tp)
    m = args.tokens
    w_bytes = n * k * 2
    copies = max(2, math.ceil(2 * L2_BYTES / w_bytes))
    ws = [torch.randn(n, k, dtype=torch.bfloat16, device=dev).mul_(0.02) for _ in range(copies)]
    x = torch.randn(m, k, dtype=torch.bfloat16, device=dev)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    comm.set_protocol(args.protocol)
    dist.barrier()
    us_ar = _time_graph(lambda i: comm.gemm_allreduce(x, ws[i % copies], out=y), args.reps)
    dist.barrier()
    us_local = _time_graph(lambda i: ops.gemm(x, ws[i % copies], out=y), args.reps)
    dist.barrier()
    us_allreduce = _time_graph(lambda i: comm.all_reduce(y), args.reps)
    comm.set_protocol(0)
    # the library's automatic rule (comm_oneshot_for): one hop for two ranks, and for up
    # to four while each rank's one-hop sends stay within 1 MB
    oneshot = args.protocol == 1 or (args.protocol == 0 and (
        tp == 2 or (tp <= 4 and (tp - 1) * m * n * 2 <= 1 << 20)))
    us_nccl = us_cublas = 0.0
    if nccl is not None:
        # the reference's path: F.linear (cuBLAS) then an NCCL all-reduce of the result
        dist.barrier()
        yc = torch.empty(m, n, dtype=torch.bfloat16, device=dev)

        def ref_path(i):
            torch.matmul(x, ws[i % copies].t(), out=yc)
            dist.all_reduce(yc, group=nccl)

        us_nccl = _time_graph(ref_path, args.reps)
        dist.barrier()
        us_cublas = _time_graph(lambda i: torch.matmul(x, ws[i % copies].t(), out=yc), args.reps)
    t = torch.tensor([us_ar, us_local, us_allreduce, us_nccl, us_cublas], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=nccl) if nccl is not None else \
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    us_ar, us_local, us_allreduce = float(t[0]), float(t[1]), float(t[2])
    # bytes each rank sends: its partial to every peer (one hop), or partials to the
    # owners and sums back (two hops)
    link = (tp - 1) * m * n * 2 if oneshot else 2 * (tp - 1) / tp * m * n * 2
    out = {"kernel": "gemm_allreduce", "shape": name, "tp": tp, "tokens": m, "N": n, "K": k,
           "protocol": "one hop" if oneshot else "two hops",
           "us": round(us_ar, 2), "us_local_gemm": round(us_local, 2),
           "us_allreduce_alone": round(us_allreduce, 2),
           "weight_GBps": round(w_bytes / us_ar / 1e3, 1),
           "nvlink_bytes": int(link), "nvlink_GBps": round(link / us_ar / 1e3, 1)}
    if nccl is not None:
        out["us_cublas_plus_nccl"] = round(float(t[3]), 2)
        out["us_cublas"] = round(float(t[4]), 2)
    # roofline of the fused kernel: the slower of the weight stream from HBM and the bytes
    # that must cross NVLink (one all-reduce's worth, (t-1)/t of the output each way)
    peaks = pathlib.Path(__file__).resolve().parents[1] / "MEASURED_PEAKS.json"
    hbm = json.loads(peaks.read_text())["hbm_gbs"] if peaks.exists() else 6650.0
    bound_us = max(w_bytes / hbm / 1e3, (tp - 1) / tp * m * n * 2 / 770.0 / 1e3)
    out["roofline_us"] = round(bound_us, 3)
    out["roofline_frac"] = round(bound_us / us_ar, 4)
    return out


def bench_norm(args, ops) -> dict:
    """The Ouro sandwich norm (rmsnorm, residual add, rmsnorm) on ``rows`` x 2048, its
    inputs resident in L2 as they are in the decode step (it reads the GEMM output just
    written); device time per launch inside a CUDA graph."""
    dev = torch.device("cuda", 0)
    x = torch.randn(args.rows, 2048, device=dev).to(torch.bfloat16)
    res = torch.randn(args.rows, 2048, device=dev).to(torch.bfloat16)
    wa = torch.rand(2048, device=dev).to(torch.bfloat16)
    wb = torch.rand(2048, device=dev).to(torch.bfloat16)
    out = torch.empty_like(x)
    us = _time_graph(lambda i: ops.sandwich_norm(x, res, wa, wb, 1e-6, out=out), args.reps)
    return {"kernel": "sandwich_norm", "rows": args.rows, "us": round(us, 2)}


def bench_snapshot(args, kvcache) -> dict:
    """Retraction snapshot of one Ouro-1.4B request under last-exited KV (24 recurrent
    layers, 4 loop steps, 16 KV heads x 128 bf16): ``get_cpu_copy`` of ``tokens`` handles
    that exited at mixed depths into pinned host memory, and ``load_cpu_copy`` back into
    freshly reserved versions of a second pool. Wall time around each call (both end
    with a stream synchronisation), best of ``reps``."""
    import time

    dev = torch.device("cuda", 0)
    n = args.tokens
    pages = 4 * n + 2
    a = kvcache.LastExitedKVCache(16, 24, 128, pages, 0, 24, 4, dev, zero=False)
    b = kvcache.LastExitedKVCache(16, 24, 128, pages, 0, 24, 4, dev, zero=False)
    handles = torch.arange(1, n + 1, dtype=torch.int32, device=dev)
    a.reserve_versions(handles)
    exits = torch.randint(1, 5, (n,), dtype=torch.int32, device=dev)
    a.alias_versions(handles, exits, int((4 - exits).sum()))
    snap = a.get_cpu_copy(handles)
    b.reserve_restore_versions(handles, snap)
    best_out = best_in = float("inf")
    for _ in range(args.reps):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        a.get_cpu_copy(handles)
        t1 = time.perf_counter()
        b.load_cpu_copy(snap, handles)
        t2 = time.perf_counter()
        best_out, best_in = min(best_out, t1 - t0), min(best_in, t2 - t1)
    nbytes = snap.numel()
    return {"kernel": "kv_snapshot", "tokens": n, "bytes": nbytes,
            "backup_ms": round(best_out * 1e3, 2), "restore_ms": round(best_in * 1e3, 2),
            "backup_GBps": round(nbytes / best_out / 1e9, 1),
            "restore_GBps": round(nbytes / best_in / 1e9, 1)}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="kernel", required=True)
    at = sub.add_parser("attention")
    at.add_argument("--rows", type=int, default=143)
    at.add_argument("--ctx", type=int, default=1448)
    at.add_argument("--ctx-spread", type=int, default=0,
                    help="contexts uniform in [ctx-spread, ctx+spread] (0: all equal)")
    at.add_argument("--heads", type=int, default=16)
    at.add_argument("--kv-heads", type=int, default=16)
    at.add_argument("--head-dim", type=int, default=128)
    at.add_argument("--page", type=int, default=16)
    at.add_argument("--reps", type=int, default=20)
    at.add_argument("--seed", type=int, default=0)
    at.add_argument("--shared-prefix", type=int, default=0,
                    help="tokens of each row's context shared with its group (page multiple)")
    at.add_argument("--groups", type=int, default=4, help="prefix groups (rows interleaved)")
    at.add_argument("--vs-trtllm", action="store_true",
                    help="also time FlashInfer's trtllm-gen decode (the reference's sm100 "
                         "backend) on the same pool and check its output")
    at.add_argument("--force", type=int, nargs="+", default=[0],
                    help="kernel selections to time: 0 automatic, 1 tensor-core kernel, 2 not")
    gm = sub.add_parser("gemm")
    gm.add_argument("--tokens", type=int, default=143)
    gm.add_argument("--shape", nargs="+", default=["qkv", "o", "gate_up", "down"],
                    choices=sorted(OURO_GEMMS))
    gm.add_argument("--reps", type=int, default=60)
    gm.add_argument("--tp", type=int, default=1, help="per-rank shard shapes of this TP size")
    gm.add_argument("--cublas", action="store_true",
                    help="also time torch.matmul (cuBLAS) on the same shapes and weights")
    gm.add_argument("--rope", action="store_true",
                    help="qkv through the RoPE + KV store epilogue (gemm_rope_store)")
    gm.add_argument("--n", type=int, default=0, help="override the shape's output rows")
    gm.add_argument("--k", type=int, default=0, help="override the shape's reduction size")
    gm.add_argument("--tile", type=int, nargs="+", default=[0],
                    help="largest token-tile widths to time (0 automatic)")
    gm.add_argument("--cublas-only", action="store_true",
                    help="time only torch.matmul (cuBLAS), launching no kernel of this library")
    gm.add_argument("--plan", type=int, nargs="+", default=[0],
                    help="tile plans to time (lsb_gemm_force_plan modes): 0 automatic, 1 one "
                         "wide tile (257-384 tokens), 2 tiles of <= 96 tokens, 3 one CTA per "
                         "SM; + 16 x tuning flags (1 K loop unrotated, 2 L2 hints, 4 "
                         "epilogue back-off)")
    ga = sub.add_parser("gemm_ar")
    ga.add_argument("--tokens", type=int, default=256)
    ga.add_argument("--shape", nargs="+", default=["o", "down"], choices=["o", "down"])
    ga.add_argument("--reps", type=int, default=60)
    ga.add_argument("--protocol", type=int, default=0, choices=[0, 1, 2],
                    help="all-reduce protocol: 0 automatic, 1 one hop, 2 two hops via owners")
    ga.add_argument("--vs-nccl", action="store_true",
                    help="also time F.linear (cuBLAS) + an NCCL all-reduce on the same shapes")
    nm = sub.add_parser("norm")
    nm.add_argument("--rows", type=int, default=263)
    nm.add_argument("--reps", type=int, default=100)
    sn = sub.add_parser("snapshot")
    sn.add_argument("--tokens", type=int, default=2048)
    sn.add_argument("--reps", type=int, default=5)
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("kernel_bench needs a CUDA device")
    _package()
    import importlib
    ops = importlib.import_module("loop_sglang_b200.ops")
    if args.kernel == "gemm_ar":
        import datetime
        import os

        import torch.distributed as dist

        C = importlib.import_module("loop_sglang_b200.comm")
        rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
        comm = C.B200Communicator(rank, world, args.tokens * 8192)
        nccl = dist.new_group(backend="nccl") if args.vs_nccl else None
        for name in args.shape:
            line = bench_gemm_ar(args, ops, comm, name, nccl)
            if rank == 0:
                print(json.dumps(line), flush=True)
        comm.close()
        dist.destroy_process_group()
        return
    torch.cuda.set_device(0)
    if args.kernel == "norm":
        print(json.dumps(bench_norm(args, ops)), flush=True)
        return
    if args.kernel == "snapshot":
        print(json.dumps(bench_snapshot(args, importlib.import_module("loop_sglang_b200.kvcache"))),
              flush=True)
        return
    if args.kernel == "attention":
        for mode in args.force:
            ops.check(ops.lib().lsb_attention_force_kernel(mode), "attention_force_kernel")
            line = bench_attention(args, ops)
            line["force"] = mode
            print(json.dumps(line), flush=True)
        ops.check(ops.lib().lsb_attention_force_kernel(0), "attention_force_kernel")
    else:
        for tile in args.tile:
            ops.check(ops.lib().lsb_gemm_force_tile_tokens(tile), "gemm_force_tile_tokens")
            for plan in args.plan:
                ops.check(ops.lib().lsb_gemm_force_plan(plan), "gemm_force_plan")
                for name in args.shape:
                    line = bench_gemm(args, ops, name)
                    line["plan"], line["tile"] = plan, tile
                    line["tile_plan"] = ops.gemm_plan(args.tokens, *tp_shape(name, args.tp)[:2])
                    print(json.dumps(line), flush=True)
        ops.check(ops.lib().lsb_gemm_force_plan(0), "gemm_force_plan")
        ops.check(ops.lib().lsb_gemm_force_tile_tokens(0), "gemm_force_tile_tokens")


if __name__ == "__main__":
    main()
