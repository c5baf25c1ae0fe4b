"""Decode throughput of the looped-decoder hot path on B200 (one JSON line on stdout).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload cdb|cb|radix]

Default workload (the metric's): Ouro-1.4B architecture (24 shared
layers x 4 loop steps, hidden 2048, 16 MHA heads x 128, SwiGLU 5632, vocab 49152),
random-init bf16, early exit under continuous-depth batching (CDB) with the last-exited
KV policy and exit threshold 0.2. 512 requests with uniform-random prompt lengths in
[256, 1024] and 512 outputs; the running batch is capacity-limited (version slots of
192 KiB) and decodes from the middle of its generation. Exit steps are prescribed per
output token at 15/25/30/30% for loop steps 1-4 (the reference's replay depths; the
gate is still evaluated every step). A step is one core step of every running row at
its own depth plus the device-side routing: exit decisions, greedy sampling of the rows
that exit, KV version alias/reserve and the successors' prelude, all from this
repository's kernels, replayed as one CUDA graph; ``value`` = output tokens / time.

``--workload cb``: full-depth CB decode with depth-indexed KV and
16-token pages, 256 requests with prompts U[512, 2048] + 256 outputs; a step is one
decode step of the running batch (4 x 24 layers, LM head, sampling).

``--workload radix``: Ouro-2.6B (48 layers) full-depth decode, 256
requests in 4 groups of 64 sharing a 2048-token prefix + 2048 unique tokens, 512 outputs;
the page tables come from the radix prefix cache, so a group's rows read one copy of the
prefix pages (the roofline counts those bytes once per group).

KV contents and token ids are synthetic (seeded random), as are the weights. ``value``
times K device-resident steps; ``e2e`` times K steps through the host (H2D of the
step's scheduler inputs, D2H of its outputs). ``--impl reference`` times the CPU oracle
restatement of the same work on a bounded sample. With N > 1 (torchrun, one process per
GPU) the model runs tensor-parallel over the N GPUs (the reference's TP split; o_proj
and down_proj fused with their NVLink all-reduce): every rank holds 1/N of the weights
and KV heads, so the KV pool admits more requests (strong scaling on the fixed
workload).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

OURO_14B = dict(arch="ouro", hidden=2048, heads=16, kv_heads=16, head_dim=128,
                intermediate=5632, vocab=49152, num_core_layers=24, loop_steps=4,
                rope_theta=1e6, rms_eps=1e-6, max_position=4096)
OURO_26B = {**OURO_14B, "num_core_layers": 48, "max_position": 8192}
PAGE = 16
NUM_REQS = 256
PROMPT_RANGE = (512, 2048)
OUT_TOKENS = 256
MID = 128  # decode position inside the generation when timing starts
SEED = 0
NVLINK_GBS = 770.0  # measured peer-copy bandwidth per direction on this pool's B200s


# Measured DRAM traffic of the decode attention kernel per context token (K+V of 16
# heads x 128 = 8192 algorithmic bytes), from an ncu capture of a one-layer case.
ATTN_DRAM_BYTES_PER_CTX_TOKEN = 8362.3


def agree_min(n: int, world: int, dev) -> int:
    """The smallest of the ranks' values (batch sizes derived from each GPU's free memory)."""
    if world == 1:
        return n
    t = torch.tensor([n], dtype=torch.int64, device=dev)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MIN)
    return int(t.item())


def init_nccl(dev, seconds: int) -> None:
    """The job's NCCL process group, created (and its communicator initialised by a first
    barrier) with file descriptor 1 pointed at stderr: NCCL may print its version banner
    on stdout, where rank 0's one JSON line must stand alone."""
    import datetime

    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=seconds),
                                             device_id=dev)
        torch.distributed.barrier()
        torch.cuda.synchronize(dev)
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


def log(msg: str) -> None:
    print(msg, file=sys.stderr, flush=True)


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def request_lengths() -> np.ndarray:
    rng = np.random.default_rng(SEED)
    return rng.integers(PROMPT_RANGE[0], PROMPT_RANGE[1] + 1, NUM_REQS)


def admit(prompts: np.ndarray, free_pages: int) -> int:
    """How many requests (in order) fit: each reserves pages for prompt + outputs."""
    need = np.cumsum((prompts + OUT_TOKENS + PAGE - 1) // PAGE)
    return int(np.searchsorted(need, free_pages, side="right"))


def gpu_weights(cfg, device, seed: int) -> dict[str, torch.Tensor]:
    """Seeded N(0, 0.02) weights (norms 1 + N(0, 0.05)) generated on the GPU."""
    g = torch.Generator(device=device).manual_seed(seed)
    w: dict[str, torch.Tensor] = {}

    def mat(name, *shape):
        w[name] = (torch.randn(*shape, generator=g, device=device) * 0.02).to(torch.bfloat16)

    def norm(name, n):
        w[name] = (1 + 0.05 * torch.randn(n, generator=g, device=device)).to(torch.bfloat16)

    h, i = cfg.hidden, cfg.intermediate
    mat("model.embed_tokens.weight", cfg.vocab, h)
    for p in cfg.layer_names():
        mat(f"{p}.self_attn.qkv_proj.weight", cfg.qkv_out, h)
        if cfg.attention_bias:
            mat(f"{p}.self_attn.qkv_proj.bias", cfg.qkv_out)
        mat(f"{p}.self_attn.o_proj.weight", h, cfg.heads * cfg.head_dim)
        mat(f"{p}.mlp.gate_up_proj.weight", 2 * i, h)
        mat(f"{p}.mlp.down_proj.weight", h, i)
        for n in ("input_layernorm", "input_layernorm_2", "post_attention_layernorm",
                  "post_attention_layernorm_2"):
            norm(f"{p}.{n}.weight", h)
    norm("model.norm.weight", h)
    if cfg.arch == "ouro":
        mat("model.early_exit_gate.weight", 1, h)
        w["model.early_exit_gate.bias"] = torch.zeros(1, dtype=torch.bfloat16, device=device)
    else:
        mat("model.adapter.weight", h, 2 * h)
        if cfg.adapter_bias:
            mat("model.adapter.bias", h)
    mat("lm_head.weight", cfg.vocab, h)
    return w


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device) -> None:
        self.proc = None
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            ident = str(device.index or 0)
        self.cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                    "-i", ident, "-lms", "50"]

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return self
        # the timed region starts only once samples are flowing, so it is covered by them
        deadline = time.perf_counter() + 5.0
        while time.perf_counter() < deadline and self.proc.poll() is None:
            self.file.flush()
            if Path(self.file.name).stat().st_size > 0:
                break
            time.sleep(0.02)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            self.proc.wait(timeout=10)

    def summary(self) -> dict:
        self.file.flush()
        return self.parse(Path(self.file.name).read_text())

    @staticmethod
    def parse(text: str) -> dict:
        """Median SM clock, max clock and the throttle reasons seen in nvidia-smi CSV rows."""
        rows = []
        for line in text.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[3 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][1]) if rows[0][1].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------- parity --

PARITY_PROMPTS = (48, 80, 112, 160)
PARITY_DECODE = 3


def parity_stamp(model, cpu_weights: dict | None, rank: int, world: int,
                 prompts: tuple[int, ...] = PARITY_PROMPTS) -> dict | None:
    """Greedy tokens of the benchmarked model object (same weights, same kernels, same
    tensor-parallel split) against the CPU oracle on the same inputs.

    4 requests with prompts of 48-160 random ids are prefilled at full depth into a fresh
    small KV pool of the model's own policy, then decoded for 3 steps, each step fed the
    CUDA path's own greedy tokens; the oracle (bf16 rounding points) runs the same
    prefill and steps on rank 0. A token agrees when the argmaxes match; it is a near tie
    when they differ but the oracle's logit of the CUDA path's token is within the bf16
    noise of its maximum -- the larger of 2e-2 x max |logit| and the step's distance
    between the bf16 oracle and the same computation in fp32 (after 96 layer passes of a
    random-init model bf16 arithmetic alone moves the logits by ~10% of their range, so
    either token may win); anything else is a mismatch. ``agree_decided`` leaves the near
    ties out (null when all are near ties: at Huginn's full depth of 132 layer passes the
    bf16 and fp32 oracles themselves disagree everywhere on random-init weights, so its
    parity rests on the per-layer full-width tests). ``vs_fp32`` compares both bf16
    computations with the fp32 one.
    Collective over the ranks: every rank runs the CUDA part.
    """
    from oracle import model as om

    from loop_sglang_b200.model import DeviceBatch

    dev = model.device
    cfg = model.cfg
    policy = model.policy
    page = 1 if policy == "last_exited" else PAGE
    g = torch.Generator().manual_seed(SEED + 11)
    prompt_lens = tuple(prompts)
    prompts = [torch.randint(0, cfg.vocab, (n,), generator=g, dtype=torch.int32)
               for n in prompt_lens]
    b = len(prompts)
    span = max(prompt_lens) + PARITY_DECODE + 1
    pages_per = (span + page - 1) // page
    table = (1 + torch.arange(b).view(-1, 1) * pages_per + torch.arange(pages_per)).to(torch.int32)
    num_pages = b * pages_per + 1
    if policy == "last_exited":  # version slots: one per loop step of every token
        tokens = sum(prompt_lens) + b * (PARITY_DECODE + 1)
        num_pages = max(num_pages, cfg.loop_steps * tokens + 1)
    lens = torch.tensor(prompt_lens, dtype=torch.int32)

    def batch(step: int, ids: torch.Tensor):
        if step < 0:
            pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in prompt_lens])
            rows = torch.cat([torch.full((n,), r) for r, n in enumerate(prompt_lens)])
            seq, cu = lens.clone(), torch.zeros(b + 1, dtype=torch.int32)
            cu[1:] = torch.cumsum(lens, 0)
        else:
            pos, rows = lens + step, torch.arange(b)
            seq, cu = lens + step + 1, torch.arange(b + 1, dtype=torch.int32)
        loc = (table[rows, (pos // page).long()] * page + pos % page).to(torch.int32)
        return om.Batch(ids.to(torch.int32), pos.to(torch.int32), loc, table.clone(),
                        seq.to(torch.int32), cu, step < 0)

    kv = model.make_kv_cache(num_pages, page)
    ids = torch.cat(prompts)
    got, fed = [], []
    for step in range(-1, PARITY_DECODE):
        ob = batch(step, ids)
        db = DeviceBatch(ob.input_ids.to(dev), ob.positions.to(dev), ob.out_loc.to(dev),
                         ob.page_table.to(dev), ob.cache_seqlens.to(dev),
                         ob.cu_seqlens_q.to(dev), ob.is_prefill, max_seqlen=pages_per * page)
        if policy == "last_exited":
            kv.reserve_versions(db.out_loc)
        logits = model.forward(db, kv).float().cpu()
        got.append(logits)
        fed.append(ids)
        ids = logits.argmax(-1).to(torch.int32)
    del kv
    if rank != 0 or cpu_weights is None:
        return None
    ocfg = om.LoopedConfig(**cfg.__dict__)

    def oracle_logits(dtype: torch.dtype) -> list[torch.Tensor]:
        w = (om.with_fp32_matrices(cpu_weights) if dtype == torch.bfloat16
             else {k: v.float() for k, v in cpu_weights.items()})
        # with the tensor-parallel ranks' rounding points (row-parallel partials rounded
        # before their sum, as the reference's per-rank F.linear + all-reduce)
        oracle = om.LoopedModel(ocfg, w, policy, tp=world)
        if policy == "last_exited":
            pool = om.SlotKVPool(oracle.slot_layout(), num_pages, cfg.kv_heads, cfg.head_dim,
                                 dtype)
        else:
            pool = om.PagedKVPool(oracle.num_kv_layers, num_pages, page, cfg.kv_heads,
                                  cfg.head_dim, dtype)
        out = []
        for i, step in enumerate(range(-1, PARITY_DECODE)):
            ob = batch(step, fed[i])
            if policy == "last_exited":
                pool.versions.reserve(ob.out_loc.numpy())
            out.append(oracle.forward(ob, pool).float())
        return out

    def rel(a: torch.Tensor, ref: torch.Tensor) -> float:
        return float((a - ref).abs().max() / ref.abs().max())

    refs, exact = oracle_logits(torch.bfloat16), oracle_logits(torch.float32)
    counts = {"agree": 0, "near_tie": 0, "mismatch": 0}
    worst = worst_exact = floor = 0.0
    agree_exact = oracle_exact = 0
    for i, ref in enumerate(refs):
        scale = ref.abs().max(-1).values
        worst = max(worst, rel(got[i], ref))
        worst_exact = max(worst_exact, rel(got[i], exact[i]))
        step_floor = rel(ref, exact[i])
        floor = max(floor, step_floor)
        # a token is decided only where the oracle's top-two margin exceeds what bf16
        # arithmetic itself moves the logits at this step (at least 2e-2 of max |logit|)
        tol = max(2e-2, step_floor)
        gi, ri = got[i].argmax(-1), ref.argmax(-1)
        agree_exact += int((gi == exact[i].argmax(-1)).sum())
        oracle_exact += int((ri == exact[i].argmax(-1)).sum())
        for r in range(b):
            if int(gi[r]) == int(ri[r]):
                counts["agree"] += 1
            elif ref[r, gi[r]] >= ref[r, ri[r]] - tol * scale[r]:
                counts["near_tie"] += 1
            else:
                counts["mismatch"] += 1
    n = sum(counts.values())
    decided = counts["agree"] + counts["mismatch"]
    return {"agree": round(counts["agree"] / n, 4),
            # null when every token is a near tie (nothing was decided)
            "agree_decided": round(counts["agree"] / decided, 4) if decided else None,
            "decided": decided, "tokens": n, "rows": b, "near_ties": counts["near_tie"],
            "mismatches": counts["mismatch"], "max_logit_rel_err": round(worst, 5),
            "vs_fp32": {"agree": round(agree_exact / n, 4),
                        "bf16_oracle_agree": round(oracle_exact / n, 4),
                        "max_logit_rel_err": round(worst_exact, 5),
                        "bf16_oracle_rel_err": round(floor, 5)},
            "tp": world, "policy": policy,
            "vs": ("CPU oracle with the reference's bf16 rounding points, same weights and "
                   "inputs (vs_fp32: the oracle in fp32 arithmetic on the same weights, and "
                   "how far the bf16 oracle itself lands from it)"),
            "sample": (f"{b} requests, prompts {list(prompt_lens)} random ids, full-depth "
                       f"prefill + {PARITY_DECODE} greedy decode steps through the benchmarked "
                       "model object")}


def rank_info(world: int, rank: int, local: int, dev) -> list | None:
    """(rank, local rank, device name, PCI bus id) of every rank that took part."""
    p = torch.cuda.get_device_properties(dev)
    me = [rank, local, p.name, f"{getattr(p, 'pci_domain_id', 0):04x}:"
          f"{getattr(p, 'pci_bus_id', 0):02x}:{getattr(p, 'pci_device_id', 0):02x}"]
    if world == 1:
        return [me]
    out: list = [None] * world
    torch.distributed.all_gather_object(out, me)
    return out


# ---------------------------------------------------------------- CPU side --

def cpu_decode_sample(steps: int, batch: int, threads: int, model_cfg: dict | None = None,
                      contexts: np.ndarray | None = None, name: str = "Ouro-1.4B",
                      policy: str = "depth_indexed", weights: dict | None = None) -> dict:
    """The oracle (CPU restatement of the reference decode step) on a bounded sample:
    ``batch`` requests of the workload (configs[1] contexts unless given), ``steps``
    full-depth decode steps (``weights``: bf16 weights to reuse instead of generating)."""
    from oracle import model as om

    torch.set_num_threads(threads)
    cfg = om.LoopedConfig(**(model_cfg or OURO_14B))
    t0 = time.perf_counter()
    if weights is None:
        weights = om.make_weights(cfg, seed=SEED, dtype=torch.bfloat16)
    w = om.with_fp32_matrices(weights)
    mdl = om.LoopedModel(cfg, w, policy)
    ctx = (request_lengths()[:batch] + MID) if contexts is None else np.asarray(contexts)[:batch]
    pages_per = [(int(c) + steps + PAGE) // PAGE for c in ctx]
    num_pages = sum(pages_per) + 1
    pool = om.PagedKVPool(mdl.num_kv_layers, num_pages, PAGE, cfg.kv_heads, cfg.head_dim,
                          torch.bfloat16)
    pool.buf.normal_(generator=torch.Generator().manual_seed(1))
    table = torch.zeros(batch, max(pages_per), dtype=torch.int32)
    nxt = 1
    for b, n in enumerate(pages_per):
        table[b, :n] = torch.arange(nxt, nxt + n, dtype=torch.int32)
        nxt += n
    setup = time.perf_counter() - t0
    ids = torch.randint(0, cfg.vocab, (batch,), generator=torch.Generator().manual_seed(2),
                        dtype=torch.int32)
    times = []
    for s in range(steps):
        pos = torch.as_tensor(ctx + s, dtype=torch.int32)
        loc = table[torch.arange(batch), pos.long() // PAGE] * PAGE + pos % PAGE
        b = om.Batch(ids, pos, loc.to(torch.int32), table, pos + 1,
                     torch.arange(batch + 1, dtype=torch.int32), False)
        t = time.perf_counter()
        logits = mdl.forward(b, pool)
        ids = logits.float().argmax(-1).to(torch.int32)
        times.append(time.perf_counter() - t)
    total = sum(times)
    return {"value": batch * steps / total, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": (f"{batch} requests at context {int(ctx.mean())} (mean), {steps} decode "
                       f"steps of {name} through the CPU oracle in torch bf16/fp32, "
                       f"{threads} threads; setup {setup:.0f}s untimed"),
            "p50_step_s": statistics.median(times)}


def cpu_prefill_sample(tokens: int, threads: int) -> dict:
    """The oracle on a bounded prefill sample: one prompt of ``tokens`` random ids at full
    depth (Ouro-1.4B, depth-indexed KV in 16-token pages)."""
    from oracle import model as om

    torch.set_num_threads(threads)
    cfg = om.LoopedConfig(**OURO_14B)
    t0 = time.perf_counter()
    mdl = om.LoopedModel(cfg, om.with_fp32_matrices(om.make_weights(cfg, seed=SEED)),
                         "depth_indexed")
    pages = (tokens + PAGE - 1) // PAGE
    pool = om.PagedKVPool(mdl.num_kv_layers, pages + 1, PAGE, cfg.kv_heads, cfg.head_dim,
                          torch.bfloat16)
    table = torch.arange(1, pages + 1, dtype=torch.int32).view(1, -1)
    pos = torch.arange(tokens, dtype=torch.int32)
    loc = (table[0, (pos // PAGE).long()] * PAGE + pos % PAGE).to(torch.int32)
    ids = torch.randint(0, cfg.vocab, (tokens,), generator=torch.Generator().manual_seed(2),
                        dtype=torch.int32)
    b = om.Batch(ids, pos, loc, table, torch.tensor([tokens], dtype=torch.int32),
                 torch.tensor([0, tokens], dtype=torch.int32), True)
    setup = time.perf_counter() - t0
    t = time.perf_counter()
    mdl.forward(b, pool)
    total = time.perf_counter() - t
    return {"value": tokens / total, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": (f"one {tokens}-token prompt prefilled at full depth through the CPU "
                       f"oracle in torch bf16/fp32, {threads} threads; setup {setup:.0f}s "
                       "untimed"),
            "p50_step_s": total}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    # a bounded sample: at most --cpu-steps decode steps (output tokens) of the batch
    steps = max(1, min(args.steps, args.cpu_steps))
    if args.workload == "cdb":
        base = cpu_cdb_sample(steps, args.cpu_batch, threads)
        metric, workload = CDB_METRIC, CDB_WORKLOAD
    elif args.workload == "radix":
        base = cpu_decode_sample(min(steps, 2), 1, threads, OURO_26B,
                                 np.array([RADIX_PREFIX + RADIX_SUFFIX + RADIX_MID]), "Ouro-2.6B")
        metric, workload = RADIX_METRIC, RADIX_WORKLOAD
    elif args.workload == "prefill":
        base = cpu_prefill_sample(512, threads)
        metric, workload = PREFILL_METRIC, PREFILL_WORKLOAD
    elif args.workload == "huginn":
        rng = np.random.default_rng(SEED)
        ctx = rng.integers(HUGINN_PROMPT_RANGE[0], HUGINN_PROMPT_RANGE[1] + 1, 8) + HUGINN_MID
        base = cpu_decode_sample(min(steps, 2), min(args.cpu_batch, 8), threads, HUGINN, ctx,
                                 "Huginn-0125", policy="shared")
        metric, workload = HUGINN_METRIC, HUGINN_WORKLOAD
    else:
        base = cpu_decode_sample(steps, args.cpu_batch, threads)
        metric, workload = METRIC, WORKLOAD
    line = {
        "impl": "reference", "metric": metric, "value": base["value"], "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * base["p50_step_s"], "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random weights, KV and token ids)",
        "config": {"workload": workload, "sample_batch": args.cpu_batch},
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# Ouro-2.6B, depth-indexed KV, radix prefix cache: 256 requests in 4
# groups of 64 sharing a 2048-token random prefix, each with a 2048-token unique suffix,
# 512 outputs. Requests are interleaved over the groups so every group is present in a
# capacity-limited batch; page tables come from this repository's radix prefix cache.
RADIX_GROUPS = 4
RADIX_REQS = 256
RADIX_PREFIX = 2048
RADIX_SUFFIX = 2048
RADIX_OUT = 512
RADIX_MID = 256
RADIX_METRIC = ("decode output tok/s, Ouro-2.6B CB full depth with a shared-prefix radix "
                "cache (configs[3]), TP over the job's GPUs")
RADIX_WORKLOAD = ("configs[3]: Ouro-2.6B random-init bf16 (48 layers x 4 loop steps), full-depth "
                  "decode, depth-indexed KV with 16-token pages, 256 requests in 4 groups of 64 "
                  "sharing a 2048-token random prefix + 2048 unique tokens, 512 outputs; page "
                  "tables built through the radix prefix cache (shared prefix pages); "
                  "capacity-limited running batch decoding at prompt+256")

METRIC = "decode output tok/s, Ouro-1.4B CB full depth (configs[1]), TP over the job's GPUs"
WORKLOAD = ("configs[1]: Ouro-1.4B random-init bf16, full-depth CB decode, depth-indexed KV, "
            "16-token pages, 256 requests prompt U[512,2048] + 256 outputs, capacity-limited "
            "running batch decoding at prompt+128")


# ---------------------------------------------------------------- GPU side --

def radix_page_tables(eng, free_pages: np.ndarray, bs: int, vocab: int, dev) -> int:
    """Page tables of the radix workload built as the reference's cache manager builds them
    (match the request's ids, lock, allocate pages for the rest, insert the prompt):
    through this repository's radix prefix cache. Returns the prompt tokens served from
    the cache (the shared prefixes)."""
    from loop_sglang_b200.prefix_cache import RadixPrefixCache

    rng = np.random.default_rng(SEED + 3)
    prefixes = rng.integers(0, vocab, (RADIX_GROUPS, RADIX_PREFIX)).astype(np.int32)
    cache = RadixPrefixCache("cpu", page_size=PAGE)
    total = RADIX_PREFIX + RADIX_SUFFIX + RADIX_OUT
    nxt, hits = 0, 0
    for r in range(bs):
        ids = np.concatenate([prefixes[r % RADIX_GROUPS],
                              rng.integers(0, vocab, RADIX_SUFFIX).astype(np.int32)])
        handle = cache.match_prefix(torch.from_numpy(ids)).cuda_handle
        cache.lock_handle(handle)
        cached = handle.cached_len
        hits += cached
        matched = handle.get_matched_indices().numpy()[::PAGE] // PAGE if cached else \
            np.zeros(0, np.int64)
        n_new = (total - cached) // PAGE
        pages = np.concatenate([matched, free_pages[nxt:nxt + n_new]]).astype(np.int64)
        nxt += n_new
        locs = (pages[:, None] * PAGE + np.arange(PAGE)).reshape(-1).astype(np.int32)
        ins = cache.insert_prefix(torch.from_numpy(ids), torch.from_numpy(locs[:ids.size]))
        cache.lock_handle(handle, unlock=True)
        cache.lock_handle(ins.handle)
        eng.assign_pages(r + 1, torch.from_numpy(pages).to(dev))
    cache.check_integrity()
    return hits


def run_b200(args) -> None:
    from __graft_entry__ import load_package

    load_package()
    from loop_sglang_b200 import _lib, ops
    from loop_sglang_b200.comm import B200Communicator
    from loop_sglang_b200.engine import DecodeEngine
    from loop_sglang_b200.model import LoopedConfig, LoopedDecoder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        init_nccl(dev, 300)
    radix = args.workload == "radix"
    cfg = LoopedConfig(**(OURO_26B if radix else OURO_14B))
    out_tokens, mid = (RADIX_OUT, RADIX_MID) if radix else (OUT_TOKENS, MID)
    t0 = time.perf_counter()
    comm = None
    if world > 1:  # symmetric buffer: the largest all-reduce / LM-head gather of a step
        vocab_local = -(-cfg.vocab // world)
        comm = B200Communicator(rank, world, NUM_REQS * max(cfg.hidden, vocab_local))
    weights = gpu_weights(cfg, dev, SEED)  # same seed on every rank: the same full model
    cpu_weights = ({k: v.cpu() for k, v in weights.items()}
                   if rank == 0 and not args.no_parity else None)
    model = LoopedDecoder(cfg, weights, "depth_indexed", dev, comm=comm)
    del weights
    torch.cuda.empty_cache()
    page_bytes = 2 * model.num_kv_layers * PAGE * model.hkv * cfg.head_dim * 2
    free, _ = torch.cuda.mem_get_info(dev)
    pool_pages = int((free - 8 * 2**30) // page_bytes)
    if radix:
        prompts = np.full(RADIX_REQS, RADIX_PREFIX + RADIX_SUFFIX)
        shared_pages = RADIX_GROUPS * RADIX_PREFIX // PAGE
        own_pages = (RADIX_SUFFIX + RADIX_OUT) // PAGE
        fit = (pool_pages - 1 - shared_pages) // own_pages
        bs = args.batch or int(max(0, min(RADIX_REQS, fit)))
    else:
        prompts = request_lengths()
        bs = args.batch or min(admit(prompts, pool_pages - 1), NUM_REQS)
    bs = agree_min(bs, world, dev)  # tensor parallel: every rank runs the same batch
    prompts = prompts[:bs]
    full = prompts + out_tokens
    pages_per = (full + PAGE - 1) // PAGE
    if radix:
        num_pages = min(pool_pages, shared_pages + bs * own_pages + 1)
    else:
        num_pages = min(pool_pages, int(pages_per.sum()) + 1)
    kv = model.make_kv_cache(num_pages, PAGE, zero=False)
    kv._kv_buffer.normal_(generator=torch.Generator(device=dev).manual_seed(SEED + 1))
    kv._kv_buffer[:, :, 0].zero_()
    max_len = int(full.max())
    eng = DecodeEngine(model, kv, bs, max_len, PAGE, max_reqs=bs)
    perm = torch.randperm(num_pages - 1, generator=torch.Generator().manual_seed(SEED + 2)) + 1
    shared_hits = 0
    if radix:
        shared_hits = radix_page_tables(eng, perm.numpy(), bs, cfg.vocab, dev)
    else:
        off = 0
        for r in range(bs):
            n = int(pages_per[r])
            eng.assign_pages(r + 1, perm[off:off + n].to(dev))
            off += n
    rows = torch.arange(1, bs + 1, dtype=torch.int32, device=dev)
    steps_total = args.warmup + args.steps
    base_seq = torch.as_tensor(prompts + mid, dtype=torch.int32, device=dev)
    sched = torch.stack([base_seq + 1 + s for s in range(steps_total + 1)])  # incl. new token
    eng.ids.copy_(torch.randint(0, cfg.vocab, (bs,), device=dev, dtype=torch.int32))
    eng.set_batch(rows, sched[0])
    prefix_groups = eng.share_prefixes() if radix else 0
    eng.capture()
    setup_s = time.perf_counter() - t0
    log(f"[bench] rank {rank}: batch {bs}, pool {num_pages} pages, setup {setup_s:.1f}s, "
        f"{eng.launches_per_step} kernels/step")

    s = eng.stream

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    with torch.cuda.stream(s):
        for k in range(args.warmup):
            eng.seq_lens.copy_(sched[k], non_blocking=True)
            eng.replay()
    barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(dev) as clocks, torch.cuda.stream(s):
        ev[0].record(s)
        for k in range(args.steps):
            eng.seq_lens.copy_(sched[args.warmup + k], non_blocking=True)
            eng.replay()
            ev[k + 1].record(s)
        s.synchronize()
    barrier()
    step_ms = [ev[k].elapsed_time(ev[k + 1]) for k in range(args.steps)]
    total_ms = ev[0].elapsed_time(ev[-1])
    clk = clocks.summary()

    # e2e: the public per-step call with host buffers (pinned H2D in, D2H out).
    host_rows = torch.arange(1, bs + 1, dtype=torch.int32).pin_memory()
    host_sched = sched.cpu().pin_memory()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for k in range(args.steps):
        eng.decode_step_host(host_rows, host_sched[k])
    e1.record(s)
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    # roofline of the dominant kernel: layer-0 attention of the same batch, timed alone
    ctx = (sched[args.warmup + args.steps - 1]).to(torch.int64)
    # context tokens whose K/V must come from HBM: with the radix workload a group's shared
    # prefix pages are one copy read by all of its rows, so they count once per group
    groups_present = min(bs, RADIX_GROUPS) if radix else 0
    kv_tokens = int(ctx.sum().item()) - (bs - groups_present) * RADIX_PREFIX * int(radix)
    attn_bytes = kv_tokens * model.hkv * cfg.head_dim * 2 * 2 \
        + 2 * bs * model.hq * cfg.head_dim * 2
    q = torch.randn(bs, model.hq, cfg.head_dim, device=dev).to(torch.bfloat16)
    kc, vc = kv.slots(0)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    with torch.cuda.stream(s):
        out = torch.empty_like(q)

        def attend():  # the step's attention call (shared prefixes read once per group)
            ops.paged_attention_shared_prefix(q, kc, vc, eng.page_table, eng.cache_seqlens,
                                              eng.cu_q, PAGE, eng.batch.max_seqlen,
                                              cfg.head_dim ** -0.5, model.hkv,
                                              eng.batch.prefix_groups, out=out)

        for _ in range(3):
            attend()
        a0.record(s)
        for _ in range(reps):
            attend()
        a1.record(s)
        s.synchronize()
    attn_s = a0.elapsed_time(a1) / 1000.0 / reps

    t_max = total_ms
    e2e_max = e2e_ms
    if world > 1:
        t = torch.tensor([total_ms, e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        t_max, e2e_max = float(t[0]), float(t[1])
    tokens = bs * args.steps  # tensor parallel: every rank decodes the same batch
    value = tokens / (t_max / 1000.0)
    mean_ctx = float(ctx.float().mean())
    weight_bytes = sum(t.numel() * 2 for lw in model.layers.values()
                       for t in (lw.qkv, lw.o, lw.gate_up, lw.down)) * cfg.loop_steps \
        + model.lm_head_w.numel() * 2 + bs * cfg.hidden * 2
    kv_bytes = kv_tokens * model.num_kv_layers * model.hkv * cfg.head_dim * 4
    step_bytes = weight_bytes + kv_bytes
    peak, peak_kind = peaks()
    # NVLink bytes each rank sends per step: 2 fused all-reduces per layer and loop step
    # (a bf16 [bs, hidden] output: partials to the owners, sums back, each (t-1)/t of
    # it), the embedding all-reduce and the LM-head gather of bs x V/t logits.
    nvlink_bytes = 0
    if world > 1:
        ar = 2 * (world - 1) / world * bs * cfg.hidden * 2
        nvlink_bytes = int(ar * (2 * cfg.num_core_layers * cfg.loop_steps + 1)
                           + (world - 1) * bs * model.vocab_local * 2)
    step_s = t_max / 1000.0 / args.steps
    ideal_s = max(step_bytes / (peak * 1e9), nvlink_bytes / (NVLINK_GBS * 1e9))
    achieved = attn_bytes / attn_s / 1e9
    # DRAM bytes per launch: ncu's dram__bytes_read.sum + dram__bytes_write.sum of one
    # launch of the same kernel on a one-layer case, per context token, scaled by this
    # batch's context tokens (traffic grows with them).
    traffic = ATTN_DRAM_BYTES_PER_CTX_TOKEN * model.hkv / cfg.kv_heads * int(ctx.sum().item())
    if radix:
        traffic = None  # shared prefix pages are L2 hits for most rows: no per-token constant
    metric, workload = (RADIX_METRIC, RADIX_WORKLOAD) if radix else (METRIC, WORKLOAD)
    line = {
        "metric": metric, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t_max / args.steps,
        "p50_tpot_ms": statistics.median(step_ms), "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded random-init weights, random KV contents and token ids",
        "config": {"workload": workload,
                   "model": ("Ouro-2.6B" if radix else "Ouro-1.4B") + " architecture (random init)",
                   "global_batch": bs, "running_batch_per_gpu": bs,
                   "mean_context": round(mean_ctx, 1), "kv_pool_pages": num_pages,
                   "page_size": PAGE, "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2 (each step streams the KV pool, ~%d GB)"
                         % (step_bytes // 10**9)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": None if traffic is None else round(traffic),
                     "kernel": "paged_attention (layer-0 decode, whole running batch)",
                     "peak_kind": peak_kind,
                     "step_frac": round(step_bytes / step_s / 1e9 / peak, 4),
                     "step_bytes": step_bytes, "nvlink_bytes_per_step": nvlink_bytes,
                     "combined_step_frac": round(ideal_s / step_s, 4)},
        **({"radix": {"shared_prefix_tokens_matched": shared_hits,
                      "prefix_groups": prefix_groups,
                      "kv_tokens_unique": kv_tokens,
                      "kv_tokens_per_row_sum": int(ctx.sum().item())}} if radix else {}),
        "e2e": {"value": tokens / (e2e_max / 1000.0), "unit": "tok/s",
                "h2d_bytes_per_step": 2 * bs * 4, "d2h_bytes_per_step": bs * 4},
        "gpu_launches": eng.launches_per_step * args.steps,
        "clocks": clk,
    }
    err = ops.device_error_word(reset=False)
    if err:
        line["device_error_word"] = err  # a bounded in-kernel wait gave up or an index was bad
    line["ranks"] = rank_info(world, rank, local, dev)
    if not args.no_parity:
        line["parity"] = parity_stamp(model, cpu_weights, rank, world)
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            if radix:
                line["cpu_baseline"] = cpu_decode_sample(
                    1, 1, os.cpu_count() or 1, OURO_26B,
                    np.array([RADIX_PREFIX + RADIX_SUFFIX + RADIX_MID]), "Ouro-2.6B")
            else:
                line["cpu_baseline"] = cpu_decode_sample(args.cpu_steps, args.cpu_batch,
                                                         os.cpu_count() or 1)
            line["cpu_baseline"].pop("p50_step_s", None)
        except Exception as exc:  # reported, never silently dropped
            line["cpu_baseline"] = {"value": None, "error": repr(exc)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.graph = None
    if comm is not None:
        comm.close()
    if world > 1:
        torch.distributed.destroy_process_group()
    _ = _lib


# ------------------------------------------------------- CDB workload --
E2E_STEPS = 30  # steps of the host-buffer e2e leg (CDB), after the timed device steps

# Ouro-1.4B with early exit under continuous-depth batching, exit
# threshold 0.2, last-exited KV; 512 requests, prompt U[256, 1024], 512 outputs. The exit
# steps follow 15/25/30/30% at loop steps 1-4, prescribed per output token (the reference's
# replay_exit_depths, cdb_scheduler.py:207-213) -- the gate is still evaluated every step.
CDB_NUM_REQS = 512
CDB_PROMPT_RANGE = (256, 1024)
CDB_OUT_TOKENS = 512
CDB_MID = 256
CDB_EXIT_P = (0.15, 0.25, 0.30, 0.30)
# DRAM bytes per context key of the attention kernel over last-exited versions (scattered
# 4 KB K and V rows), from an ncu capture of that kernel on the CDB step's layout
CDB_ATTN_DRAM_BYTES_PER_CTX_TOKEN = 8216.1
CDB_METRIC = ("decode output tok/s, Ouro-1.4B CDB (configs[2]), last-exited KV, TP over the "
              "job's GPUs")
CDB_WORKLOAD = ("configs[2]: Ouro-1.4B random-init bf16, continuous-depth batching with the "
                "routing on the device, last-exited KV, exit threshold 0.2, exit steps "
                "prescribed 15/25/30/30% at loop steps 1-4 (replay depths), 512 requests with "
                "prompt U[256,1024] + 512 outputs, capacity-limited running batch decoding "
                "from prompt+256")


def cdb_depths(n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.choice(np.arange(1, 5), size=n, p=CDB_EXIT_P).astype(np.int32)


def cpu_cdb_sample(tokens: int, batch: int, threads: int) -> dict:
    """The oracle on a bounded CDB sample: ``batch`` requests at the workload's contexts
    decode ``tokens`` output tokens each, batched: every token is the prelude of all rows,
    then loop step s for the rows whose prescribed exit depth exceeds s (the batch shrinks
    as rows exit), then the LM head and greedy sampling of all rows (shared-KV addressing;
    the per-token arithmetic is the last-exited policy's)."""
    from oracle import model as om

    torch.set_num_threads(threads)
    cfg = om.LoopedConfig(**{**OURO_14B, "exit_threshold": 0.2})
    t0 = time.perf_counter()
    w = om.with_fp32_matrices(om.make_weights(cfg, seed=SEED, dtype=torch.bfloat16))
    mdl = om.LoopedModel(cfg, w, "shared")
    rng = np.random.default_rng(SEED)
    ctx = rng.integers(CDB_PROMPT_RANGE[0], CDB_PROMPT_RANGE[1] + 1, batch) + CDB_MID
    pages_per = [(int(c) + tokens + PAGE) // PAGE for c in ctx]
    num_pages = sum(pages_per) + 1
    pool = om.PagedKVPool(mdl.num_kv_layers, num_pages, PAGE, cfg.kv_heads, cfg.head_dim,
                          torch.bfloat16)
    pool.buf.normal_(generator=torch.Generator().manual_seed(1))
    table = torch.zeros(batch, max(pages_per), dtype=torch.int32)
    nxt = 1
    for b, n in enumerate(pages_per):
        table[b, :n] = torch.arange(nxt, nxt + n, dtype=torch.int32)
        nxt += n
    setup = time.perf_counter() - t0
    depths = cdb_depths(batch * tokens, SEED + 7).reshape(batch, tokens)
    ids = torch.randint(0, cfg.vocab, (batch,), generator=torch.Generator().manual_seed(2),
                        dtype=torch.int32)
    rows = torch.arange(batch)
    t = time.perf_counter()
    passes = 0
    for k in range(tokens):
        pos = torch.as_tensor(ctx + k, dtype=torch.int32)
        loc = (table[rows, pos.long() // PAGE] * PAGE + pos % PAGE).to(torch.int32)
        full = om.Batch(ids, pos, loc, table, pos + 1, torch.arange(batch + 1, dtype=torch.int32),
                        False)
        h, _ = mdl.forward_prelude(full, pool)
        for step in range(cfg.loop_steps):
            act = torch.from_numpy(np.nonzero(depths[:, k] > step)[0])
            if act.numel() == 0:
                break
            bt = om.Batch(ids[act], pos[act], loc[act], table[act], pos[act] + 1,
                          torch.arange(act.numel() + 1, dtype=torch.int32), False)
            h[act] = mdl.core_step(h[act], step, None, bt, pool)
            passes += act.numel()
        ids = mdl.lm_head(h, None).float().argmax(-1).to(torch.int32)
    total = time.perf_counter() - t
    return {"value": batch * tokens / total, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": (f"{batch} requests at context {int(ctx.mean())} (mean), {tokens} output "
                       f"tokens each, batched ({passes} row loop steps at the prescribed exit "
                       f"depths) of Ouro-1.4B through the CPU oracle in torch bf16/fp32, "
                       f"{threads} threads; setup {setup:.0f}s untimed"),
            "p50_step_s": total / max(1, tokens)}


def run_b200_cdb(args) -> None:
    from __graft_entry__ import load_package

    load_package()
    from loop_sglang_b200 import ops
    from loop_sglang_b200.comm import B200Communicator
    from loop_sglang_b200.engine import CDBDecodeEngine
    from loop_sglang_b200.model import LoopedConfig, LoopedDecoder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        init_nccl(dev, 300)
    cfg = LoopedConfig(**{**OURO_14B, "exit_threshold": 0.2})
    t0 = time.perf_counter()
    comm = None
    if world > 1:
        vocab_local = -(-cfg.vocab // world)
        comm = B200Communicator(rank, world, CDB_NUM_REQS * max(cfg.hidden, vocab_local))
    weights = gpu_weights(cfg, dev, SEED)
    cpu_weights = ({k: v.cpu() for k, v in weights.items()}
                   if rank == 0 and not args.no_parity else None)
    model = LoopedDecoder(cfg, weights, "last_exited", dev, comm=comm)
    del weights
    torch.cuda.empty_cache()
    rng = np.random.default_rng(SEED)
    prompts = rng.integers(CDB_PROMPT_RANGE[0], CDB_PROMPT_RANGE[1] + 1, CDB_NUM_REQS)
    e2e_steps = 0 if args.no_e2e else min(args.steps, E2E_STEPS)
    steps_total = args.warmup + args.steps + 1 + e2e_steps + 1
    ctx = prompts + CDB_MID  # tokens before the one being decoded
    gen_depth = cdb_depths(CDB_NUM_REQS * CDB_MID, SEED + 1).reshape(CDB_NUM_REQS, CDB_MID)
    # exit depths of the outputs to come (the replay depths of the run)
    out_cap = steps_total + 8
    future_all = cdb_depths(CDB_NUM_REQS * out_cap, SEED + 2).reshape(CDB_NUM_REQS, out_cap)
    exits = (np.cumsum(future_all, axis=1) <= steps_total).sum(1)  # outputs finished in the run
    # the versions those outputs keep: each reserves a full-depth token and keeps its exit
    # depth's versions once it exits (the rest go back to the shared free stack)
    kept = np.array([future_all[r, :exits[r]].sum() for r in range(CDB_NUM_REQS)])
    # version slots a request holds: prompt tokens keep every loop step (prefill runs at full
    # depth), generated ones their exit depth; plus the token being decoded and one fresh
    # full-depth token per output the run finishes (reserved before the exit aliases)
    need = prompts * 4 + gen_depth.sum(1) + kept + 4 * 2  # + the token in flight, + margin
    max_len = int(ctx.max()) + steps_total + 2
    slot_bytes = 2 * cfg.num_core_layers * model.hkv * cfg.head_dim * 2
    free, _ = torch.cuda.mem_get_info(dev)
    max_slots = int((free - 8 * 2**30) // slot_bytes)
    if args.batch:
        bs = args.batch
    else:
        fit = np.cumsum(np.maximum(need, max_len)) + 1
        bs = int(min(np.searchsorted(fit, max_slots, side="right"), CDB_NUM_REQS))
    bs = agree_min(bs, world, dev)  # tensor parallel: every rank runs the same batch
    num_pages = int(max(np.maximum(need, max_len)[:bs].sum() + 1, bs * max_len + 1))
    kv = model.make_kv_cache(num_pages, 1, zero=False)
    kv._kv_buffer.normal_(generator=torch.Generator(device=dev).manual_seed(SEED + 1))
    kv._kv_buffer[:, :, 0].zero_()
    handles = (1 + torch.arange(bs, device=dev).view(-1, 1) * max_len
               + torch.arange(max_len, device=dev)).to(torch.int32)
    # context versions, request by request (prompt at full depth, outputs at their exit depth)
    ctx_b = torch.as_tensor(ctx[:bs], device=dev)
    pos = torch.arange(max_len, device=dev).view(1, -1)
    live = pos < ctx_b.view(-1, 1)
    restore = torch.full((bs, max_len), 4, dtype=torch.int32, device=dev)
    gen = torch.as_tensor(gen_depth[:bs], device=dev)
    gpos = pos - torch.as_tensor(prompts[:bs], device=dev).view(-1, 1)
    is_gen = live & (gpos >= 0)
    restore[is_gen] = gen.gather(1, gpos.clamp(0, CDB_MID - 1))[is_gen].to(torch.int32)
    ops.last_exited_reserve(kv.slot_map, kv.completed_depth, kv._free_slots, kv._free_count,
                            handles[live].contiguous(), kv.loop_steps, kv.fixed_groups,
                            kv.core_groups, restore_depths=restore[live].contiguous())
    kv.available_slots -= int(restore[live].sum().item()) * kv.core_groups
    future = torch.as_tensor(future_all[:bs], device=dev).contiguous()
    eng = CDBDecodeEngine(model, kv, bs, max_len, out_cap, replay_depths=future)
    ids0 = torch.randint(0, cfg.vocab, (bs,), device=dev, dtype=torch.int32)
    eng.start(handles, (ctx_b + 1).to(torch.int32), ids0)
    eng.capture()
    setup_s = time.perf_counter() - t0
    log(f"[bench] rank {rank}: CDB batch {bs}, {num_pages} version slots, setup {setup_s:.1f}s, "
        f"{eng.launches_per_step} kernels/step")
    s = eng.stream

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            eng.replay()
    barrier()
    p0 = int(eng.produced.item())
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(dev) as clocks, torch.cuda.stream(s):
        ev[0].record(s)
        for k in range(args.steps):
            eng.replay()
            ev[k + 1].record(s)
        s.synchronize()
    barrier()
    produced = int(eng.produced.item()) - p0
    step_ms = [ev[k].elapsed_time(ev[k + 1]) for k in range(args.steps)]
    total_ms = ev[0].elapsed_time(ev[-1])
    clk = clocks.summary()

    # e2e: each step through the host -- H2D of the running rows (the scheduler's batch),
    # one step, D2H of which rows exited and their tokens
    host_rows = torch.arange(1, bs + 1, dtype=torch.int32).pin_memory()
    host_exit = torch.zeros(bs, dtype=torch.uint8).pin_memory()
    host_ids = torch.zeros(bs, dtype=torch.int32).pin_memory()
    e2e_ms, e2e_tokens = 0.0, 0
    if not args.no_e2e:
        barrier()
        p1 = int(eng.produced.item())
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(e2e_steps):
            with torch.cuda.stream(s):
                eng.rpi.copy_(host_rows, non_blocking=True)
                eng.replay()
                host_exit.copy_(eng.exited, non_blocking=True)
                host_ids.copy_(eng.ids, non_blocking=True)
            s.synchronize()
        e1.record(s)
        barrier()
        e2e_ms = e0.elapsed_time(e1)
        e2e_tokens = int(eng.produced.item()) - p1

    # roofline of the dominant kernel: layer-0 attention over the rows' current depths
    seq = eng.cache_seqlens.to(torch.int64)
    ctx_tokens = int(seq.sum().item())
    attn_bytes = ctx_tokens * model.hkv * cfg.head_dim * 4 + 2 * bs * model.hq * cfg.head_dim * 2
    q = torch.randn(bs, model.hq, cfg.head_dim, device=dev).to(torch.bfloat16)
    kc, vc = kv.slots(0)
    table = eng.batch.core_page_table[0]
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    with torch.cuda.stream(s):
        out = torch.empty_like(q)
        for _ in range(3):
            ops.paged_attention(q, kc, vc, table, eng.cache_seqlens, eng.cu_q, 1, max_len,
                                cfg.head_dim ** -0.5, model.hkv, out=out)
        a0.record(s)
        for _ in range(reps):
            ops.paged_attention(q, kc, vc, table, eng.cache_seqlens, eng.cu_q, 1, max_len,
                                cfg.head_dim ** -0.5, model.hkv, out=out)
        a1.record(s)
        s.synchronize()
    attn_s = a0.elapsed_time(a1) / 1000.0 / reps

    t_max, e2e_max = total_ms, e2e_ms
    if world > 1:
        t = torch.tensor([total_ms, e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        t_max, e2e_max = float(t[0]), float(t[1])
    value = produced / (t_max / 1000.0)
    weight_bytes = sum(t.numel() * 2 for lw in model.layers.values()
                       for t in (lw.qkv, lw.o, lw.gate_up, lw.down)) \
        + model.lm_head_w.numel() * 2
    kv_bytes = ctx_tokens * cfg.num_core_layers * model.hkv * cfg.head_dim * 4
    step_bytes = weight_bytes + kv_bytes
    peak, peak_kind = peaks()
    achieved = attn_bytes / attn_s / 1e9
    step_s = t_max / 1000.0 / args.steps
    line = {
        "metric": CDB_METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_max / args.steps,
        "p50_tpot_ms": statistics.median(step_ms) * bs / max(1.0, produced / args.steps),
        "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded random-init weights, random KV contents and token ids",
        "config": {"workload": CDB_WORKLOAD, "model": "Ouro-1.4B architecture (random init)",
                   "global_batch": bs, "running_batch_per_gpu": bs,
                   "mean_context": round(ctx_tokens / bs, 1), "version_slots": num_pages,
                   "outputs_per_step": round(produced / args.steps, 2),
                   "step": "one loop step of every running row at its own depth + routing",
                   "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2 (each step streams ~%d GB)" % (step_bytes // 10**9)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": round(CDB_ATTN_DRAM_BYTES_PER_CTX_TOKEN * model.hkv
                                      / cfg.kv_heads * ctx_tokens),
                     "kernel": "paged_attention (layer-0 core step, rows at their own depths)",
                     "peak_kind": peak_kind,
                     "step_frac": round(step_bytes / step_s / 1e9 / peak, 4),
                     "step_bytes": step_bytes},
        "e2e": ({"value": e2e_tokens / (e2e_max / 1000.0), "unit": "tok/s",
                 "h2d_bytes_per_step": bs * 4, "d2h_bytes_per_step": bs * 5}
                if not args.no_e2e else None),
        "gpu_launches": eng.launches_per_step * args.steps,
        "clocks": clk,
    }
    err = ops.device_error_word(reset=False)
    if err:
        line["device_error_word"] = err  # a bounded in-kernel wait gave up or an index was bad
    line["ranks"] = rank_info(world, rank, local, dev)
    if not args.no_parity:
        line["parity"] = parity_stamp(model, cpu_weights, rank, world)
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            line["cpu_baseline"] = cpu_cdb_sample(args.cpu_steps, args.cpu_batch,
                                                  os.cpu_count() or 1)
            line["cpu_baseline"].pop("p50_step_s", None)
        except Exception as exc:  # reported, never silently dropped
            line["cpu_baseline"] = {"value": None, "error": repr(exc)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.graph = None
    if comm is not None:
        comm.close()
    if world > 1:
        torch.distributed.destroy_process_group()


# ------------------------------------------------------------------ prefill --
# Prefill of configs[1]'s requests (Ouro-1.4B, depth-indexed KV in 16-token pages, prompts
# U[512, 2048]): a step is one full-depth forward of PREFILL_REQS whole prompts in one
# batch (4 loop steps x 24 layers, LM head on each request's last token). Tensor-bound:
# the roofline is the GEMMs' bf16 FLOP rate.
PREFILL_REQS = 8  # ~10k tokens: the attention kernel's per-(row, head group) split counters
PREFILL_METRIC = "prefill tok/s, Ouro-1.4B full depth (configs[1] prompts), TP over the job's GPUs"
PREFILL_WORKLOAD = ("configs[1] prompts: Ouro-1.4B random-init bf16, 8 requests with prompt "
                    "U[512,2048] prefilled together at full depth (4 loop steps x 24 layers), "
                    "depth-indexed KV in 16-token pages")


def run_b200_prefill(args) -> None:
    from __graft_entry__ import load_package

    load_package()
    from loop_sglang_b200 import ops
    from loop_sglang_b200.comm import B200Communicator
    from loop_sglang_b200.model import DeviceBatch, LoopedConfig, LoopedDecoder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        init_nccl(dev, 300)
    cfg = LoopedConfig(**OURO_14B)
    prompts = request_lengths()[: args.batch or PREFILL_REQS]
    n_tok = int(prompts.sum())
    comm = None
    if world > 1:
        comm = B200Communicator(rank, world, n_tok * cfg.hidden)
    weights = gpu_weights(cfg, dev, SEED)
    model = LoopedDecoder(cfg, weights, "depth_indexed", dev, comm=comm)
    del weights
    torch.cuda.empty_cache()
    b = prompts.size
    pages_per = (prompts + PAGE - 1) // PAGE
    num_pages = int(pages_per.sum()) + 1
    kv = model.make_kv_cache(num_pages, PAGE)
    table = torch.zeros(b, int(pages_per.max()), dtype=torch.int32)
    off = 1
    for r, n in enumerate(pages_per):
        table[r, :n] = torch.arange(off, off + n, dtype=torch.int32)
        off += int(n)
    pos = torch.cat([torch.arange(n, dtype=torch.int32) for n in prompts])
    rows = torch.cat([torch.full((int(n),), r) for r, n in enumerate(prompts)])
    loc = (table[rows, (pos // PAGE).long()] * PAGE + pos % PAGE).to(torch.int32)
    cu = torch.zeros(b + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.as_tensor(prompts, dtype=torch.int32), 0)
    ids = torch.randint(0, cfg.vocab, (n_tok,), generator=torch.Generator().manual_seed(SEED),
                        dtype=torch.int32)
    batch = DeviceBatch(ids.to(dev), pos.to(dev), loc.to(dev), table.to(dev),
                        torch.as_tensor(prompts, dtype=torch.int32).to(dev), cu.to(dev), True,
                        max_seqlen=int(table.shape[1]) * PAGE)
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    from loop_sglang_b200 import _lib

    with torch.cuda.stream(s):
        before = _lib.launch_count()
        for _ in range(args.warmup):
            model.forward(batch, kv)
        launches = (_lib.launch_count() - before) // max(1, args.warmup)
    torch.cuda.synchronize(dev)
    if world > 1:
        torch.distributed.barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(dev) as clocks, torch.cuda.stream(s):
        ev[0].record(s)
        for k in range(args.steps):
            model.forward(batch, kv)
            ev[k + 1].record(s)
        s.synchronize()
    if world > 1:
        torch.distributed.barrier()
    total_ms = ev[0].elapsed_time(ev[-1])
    clk = clocks.summary()
    # e2e: host ids in, the last tokens' greedy ids out, every step
    host_ids = ids.pin_memory()
    host_out = torch.zeros(b, dtype=torch.int32).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        e0.record(s)
        for _ in range(args.steps):
            batch.input_ids.copy_(host_ids, non_blocking=True)
            toks = model.greedy(model.forward_coda(_full_depth(model, batch, kv), batch, kv), batch)
            host_out.copy_(toks, non_blocking=True)
            s.synchronize()
        e1.record(s)
        s.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    # the dominant kernel: the gate_up GEMM (+ SwiGLU) of one layer at this token count
    x = torch.randn(n_tok, cfg.hidden, device=dev).to(torch.bfloat16)
    lw = model.layers["model.layers.0"]
    out = torch.empty(n_tok, lw.gate_up.shape[0] // 2, dtype=torch.bfloat16, device=dev)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        for _ in range(3):
            ops.gemm(x, lw.gate_up, epilogue=ops.LSB_EPI_SWIGLU, out=out)
        g0.record(s)
        for _ in range(10):
            ops.gemm(x, lw.gate_up, epilogue=ops.LSB_EPI_SWIGLU, out=out)
        g1.record(s)
        s.synchronize()
    gemm_s = g0.elapsed_time(g1) / 1000.0 / 10
    t_max, e2e_max = total_ms, e2e_ms
    if world > 1:
        t = torch.tensor([total_ms, e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        t_max, e2e_max = float(t[0]), float(t[1])
    pj = ROOT / "MEASURED_PEAKS.json"
    peak_tf = float(json.loads(pj.read_text())["bf16_tflops_sustained"]) if pj.exists() else 1400.0
    gemm_flops = 2.0 * n_tok * lw.gate_up.shape[0] * cfg.hidden
    params = sum(t.numel() for lw2 in model.layers.values() for t in (lw2.qkv, lw2.o, lw2.gate_up,
                                                                        lw2.down))
    step_flops = 2.0 * n_tok * params * cfg.loop_steps * world  # whole model over the ranks
    step_s = t_max / 1000.0 / args.steps
    line = {
        "metric": PREFILL_METRIC, "value": n_tok * args.steps / (t_max / 1000.0), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t_max / args.steps, "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded random-init weights and token ids",
        "config": {"workload": PREFILL_WORKLOAD, "model": "Ouro-1.4B architecture (random init)",
                   "global_batch": b, "prompt_tokens": n_tok, "parallelism": f"tp{world}",
                   "l2": "inputs larger than L2 (~%d GB of activations and KV per step)"
                         % (n_tok * 96 * 8192 // 10**9)},
        "roofline": {"bound": "tensor", "achieved": round(gemm_flops / gemm_s / 1e12, 1),
                     "peak": peak_tf, "unit": "TFLOP/s",
                     "frac": round(gemm_flops / gemm_s / 1e12 / peak_tf, 4), "traffic": None,
                     "kernel": f"gemm (gate_up + SwiGLU, {n_tok} tokens, timed alone)",
                     "peak_kind": "measured (sustained)" if pj.exists() else "fallback",
                     "step_frac": round(step_flops / step_s / 1e12 / peak_tf / world, 4)},
        "e2e": {"value": n_tok * args.steps / (e2e_max / 1000.0), "unit": "tok/s",
                "h2d_bytes_per_step": n_tok * 4, "d2h_bytes_per_step": b * 4},
        "gpu_launches": launches * args.steps,
        "clocks": clk,
    }
    err = ops.device_error_word(reset=False)
    if err:
        line["device_error_word"] = err
    line["ranks"] = rank_info(world, rank, local, dev)
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            line["cpu_baseline"] = cpu_prefill_sample(512, os.cpu_count() or 1)
            line["cpu_baseline"].pop("p50_step_s", None)
        except Exception as exc:  # reported, never silently dropped
            line["cpu_baseline"] = {"value": None, "error": repr(exc)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if comm is not None:
        comm.close()
    if world > 1:
        torch.distributed.destroy_process_group()


def _full_depth(model, batch, kv):
    h, inj = model.forward_prelude(batch, kv)
    for step in range(model.cfg.loop_steps):
        h = model.core_step(h, step, inj, batch, kv)
    return h


# ---------------------------------------------------------- Huginn replicas --
# Huginn-0125 architecture (hidden 5280, 55 heads x 96, prelude 2 +
# core 4 x 32 recurrences + coda 2, SwiGLU 17920, vocab 65536, RoPE 5e4), random-init bf16,
# fully shared looped KV, TP=1 x one data-parallel replica per GPU (55 heads do not shard):
# 64 requests per replica with prompts U[512, 1024] and 256 outputs. The embedding scale is
# sqrt(hidden) and q/k/v carry a bias, as in Huginn-0125's published configuration; the
# recurrent state starts at zero (state_init "zero", the deterministic choice).
HUGINN = dict(arch="huginn", hidden=5280, heads=55, kv_heads=55, head_dim=96, intermediate=17920,
              vocab=65536, num_prelude_layers=2, num_core_layers=4, num_coda_layers=2,
              loop_steps=32, rope_theta=50000.0, rms_eps=1e-6, max_position=2048,
              embed_scale=5280 ** 0.5, attention_bias=True, adapter_bias=False)
HUGINN_REQS = 64
HUGINN_PROMPT_RANGE = (512, 1024)
HUGINN_OUT = 256
HUGINN_MID = 128
HUGINN_METRIC = ("decode output tok/s, Huginn-0125 architecture, shared looped KV, one "
                 "TP=1 replica per GPU (configs[4]), summed over the job's GPUs")
HUGINN_WORKLOAD = ("configs[4]: Huginn-0125 architecture random-init bf16 (prelude 2 + core 4 "
                   "x 32 recurrences + coda 2, hidden 5280, 55 heads x 96), fully shared looped "
                   "KV in 16-token pages, 64 requests per replica with prompt U[512,1024] + 256 "
                   "outputs decoding at prompt+128, one independent replica per GPU")


def run_b200_huginn(args) -> None:
    """Data-parallel replicas: every rank decodes its own 64 requests through its own
    TP=1 model; the ranks share nothing but the barrier and the max over their times."""
    from __graft_entry__ import load_package

    load_package()
    from loop_sglang_b200 import ops
    from loop_sglang_b200.engine import DecodeEngine
    from loop_sglang_b200.model import LoopedConfig, LoopedDecoder

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        init_nccl(dev, 600)
    cfg = LoopedConfig(**HUGINN)
    t0 = time.perf_counter()
    weights = gpu_weights(cfg, dev, SEED)
    cpu_weights = ({k: v.cpu() for k, v in weights.items()}
                   if rank == 0 and not args.no_parity else None)
    model = LoopedDecoder(cfg, weights, "shared", dev)
    del weights
    torch.cuda.empty_cache()
    rng = np.random.default_rng(SEED + 100 * rank)  # each replica serves its own requests
    bs = args.batch or HUGINN_REQS
    prompts = rng.integers(HUGINN_PROMPT_RANGE[0], HUGINN_PROMPT_RANGE[1] + 1, bs)
    full = prompts + HUGINN_OUT
    pages_per = (full + PAGE - 1) // PAGE
    num_pages = int(pages_per.sum()) + 1
    kv = model.make_kv_cache(num_pages, PAGE, zero=False)
    kv._kv_buffer.normal_(generator=torch.Generator(device=dev).manual_seed(SEED + 1))
    kv._kv_buffer[:, :, 0].zero_()
    max_len = int(full.max())
    eng = DecodeEngine(model, kv, bs, max_len, PAGE, max_reqs=bs)
    perm = torch.randperm(num_pages - 1, generator=torch.Generator().manual_seed(SEED + 2)) + 1
    off = 0
    for r in range(bs):
        n = int(pages_per[r])
        eng.assign_pages(r + 1, perm[off:off + n].to(dev))
        off += n
    rows = torch.arange(1, bs + 1, dtype=torch.int32, device=dev)
    steps_total = args.warmup + args.steps
    base_seq = torch.as_tensor(prompts + HUGINN_MID, dtype=torch.int32, device=dev)
    sched = torch.stack([base_seq + 1 + s for s in range(steps_total + 1)])
    eng.ids.copy_(torch.randint(0, cfg.vocab, (bs,), device=dev, dtype=torch.int32))
    eng.set_batch(rows, sched[0])
    eng.capture()
    log(f"[bench] rank {rank}: Huginn replica batch {bs}, {num_pages} pages, setup "
        f"{time.perf_counter() - t0:.1f}s, {eng.launches_per_step} kernels/step")
    s = eng.stream

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)

    with torch.cuda.stream(s):
        for k in range(args.warmup):
            eng.seq_lens.copy_(sched[k], non_blocking=True)
            eng.replay()
    barrier()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    with ClockSampler(dev) as clocks, torch.cuda.stream(s):
        ev[0].record(s)
        for k in range(args.steps):
            eng.seq_lens.copy_(sched[args.warmup + k], non_blocking=True)
            eng.replay()
            ev[k + 1].record(s)
        s.synchronize()
    barrier()
    step_ms = [ev[k].elapsed_time(ev[k + 1]) for k in range(args.steps)]
    total_ms = ev[0].elapsed_time(ev[-1])
    clk = clocks.summary()
    host_rows = torch.arange(1, bs + 1, dtype=torch.int32).pin_memory()
    host_sched = sched.cpu().pin_memory()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for k in range(args.steps):
        eng.decode_step_host(host_rows, host_sched[k])
    e1.record(s)
    barrier()
    e2e_ms = e0.elapsed_time(e1)

    # roofline of the dominant kernel: one layer's attention over the batch, timed alone
    ctx = sched[args.warmup + args.steps - 1].to(torch.int64)
    kv_row = model.hkv * cfg.head_dim * 2 * 2
    attn_bytes = int(ctx.sum().item()) * kv_row + 2 * bs * model.hq * cfg.head_dim * 2
    q = torch.randn(bs, model.hq, cfg.head_dim, device=dev).to(torch.bfloat16)
    kc, vc = kv.slots(0)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    with torch.cuda.stream(s):
        out = torch.empty_like(q)

        def attend():  # the step's attention call (shared prefixes read once per group)
            ops.paged_attention_shared_prefix(q, kc, vc, eng.page_table, eng.cache_seqlens,
                                              eng.cu_q, PAGE, eng.batch.max_seqlen,
                                              cfg.head_dim ** -0.5, model.hkv,
                                              eng.batch.prefix_groups, out=out)

        for _ in range(3):
            attend()
        a0.record(s)
        for _ in range(reps):
            attend()
        a1.record(s)
        s.synchronize()
    attn_s = a0.elapsed_time(a1) / 1000.0 / reps

    t_max, e2e_max, tokens = total_ms, e2e_ms, bs * args.steps
    if world > 1:
        t = torch.tensor([total_ms, e2e_ms, float(tokens)], device=dev)
        tt = t.clone()
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(tt, op=torch.distributed.ReduceOp.SUM)
        t_max, e2e_max, tokens = float(t[0]), float(t[1]), int(tt[2])
    # algorithmic bytes of one replica's step: every layer pass reads its weights and the
    # KV of its (shared) layer for every row; the adapter once per recurrence; LM head
    passes = cfg.num_prelude_layers + cfg.loop_steps * cfg.num_core_layers + cfg.num_coda_layers
    layer_w = sum(t.numel() * 2 for t in (model.layers["model.layers.0"].qkv,
                                          model.layers["model.layers.0"].o,
                                          model.layers["model.layers.0"].gate_up,
                                          model.layers["model.layers.0"].down))
    step_bytes = (passes * layer_w + cfg.loop_steps * model.adapter.numel() * 2
                  + model.lm_head_w.numel() * 2 + passes * int(ctx.sum().item()) * kv_row)
    peak, peak_kind = peaks()
    step_s = t_max / 1000.0 / args.steps
    achieved = attn_bytes / attn_s / 1e9
    line = {
        "metric": HUGINN_METRIC, "value": tokens / (t_max / 1000.0), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": t_max / args.steps, "p50_tpot_ms": statistics.median(step_ms),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded random-init weights, random KV contents and token ids",
        "config": {"workload": HUGINN_WORKLOAD, "model": "Huginn-0125 architecture (random init)",
                   "global_batch": bs * world, "running_batch_per_gpu": bs,
                   "mean_context": round(float(ctx.float().mean()), 1), "kv_pool_pages": num_pages,
                   "page_size": PAGE, "parallelism": f"dp{world} (replicas, TP=1 each)",
                   "l2": "inputs larger than L2 (each step streams ~%d GB)" % (step_bytes // 10**9)},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": None,
                     "kernel": "paged_attention (one shared KV layer, whole replica batch)",
                     "peak_kind": peak_kind,
                     "step_frac": round(step_bytes / step_s / 1e9 / peak, 4),
                     "step_bytes": step_bytes},
        "e2e": {"value": tokens / (e2e_max / 1000.0), "unit": "tok/s",
                "h2d_bytes_per_step": 2 * bs * 4, "d2h_bytes_per_step": bs * 4},
        "gpu_launches": eng.launches_per_step * args.steps,
        "clocks": clk,
    }
    err = ops.device_error_word(reset=False)
    if err:
        line["device_error_word"] = err
    line["ranks"] = rank_info(world, rank, local, dev)
    if not args.no_parity:
        line["parity"] = parity_stamp(model, cpu_weights, rank, world, prompts=HUGINN_PARITY)
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            line["cpu_baseline"] = cpu_decode_sample(
                min(args.cpu_steps, 2), min(args.cpu_batch, 8), os.cpu_count() or 1, HUGINN,
                (prompts + HUGINN_MID)[:8], "Huginn-0125", policy="shared", weights=cpu_weights)
            line["cpu_baseline"].pop("p50_step_s", None)
        except Exception as exc:  # reported, never silently dropped
            line["cpu_baseline"] = {"value": None, "error": repr(exc)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.graph = None
    if world > 1:
        torch.distributed.destroy_process_group()


HUGINN_PARITY = (8, 12, 16, 20)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: 120 for cdb, 40 for cb, 20 for radix -- each "
                         "about a second or more, covered by many clock samples)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--batch", type=int, default=0, help="override the admitted batch (debug)")
    ap.add_argument("--cpu-steps", type=int, default=3,
                    help="decode steps (CDB: output tokens per request) of the CPU sample")
    ap.add_argument("--cpu-batch", type=int, default=16, help="requests in the CPU sample")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer e2e leg")
    ap.add_argument("--no-parity", action="store_true",
                    help="skip the parity stamp (greedy tokens vs the CPU oracle)")
    ap.add_argument("--workload", choices=["cdb", "cb", "radix", "huginn", "prefill"],
                    default="cdb",
                    help="cdb: configs[2] (the metric's); cb: configs[1] full-depth CB; "
                         "radix: configs[3] (Ouro-2.6B, shared prefixes); huginn: configs[4] "
                         "(one Huginn replica per GPU)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {"cdb": 120, "cb": 40, "radix": 20, "huginn": 25,
                      "prefill": 10}[args.workload]
    if args.steps < 1:
        ap.error("--steps must be >= 1")
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "cdb":
        run_b200_cdb(args)
    elif args.workload == "huginn":
        run_b200_huginn(args)
    elif args.workload == "prefill":
        run_b200_prefill(args)
    else:
        run_b200(args)  # cb and radix


if __name__ == "__main__":
    main()
