"""Kernel-level parity of the CUDA path against the oracle (one C entry point each).

Floating-point kernels are compared with the bf16 tolerance (rel/abs 2e-2) against
the oracle run on the same bf16 inputs; integer and byte work (KV store, slot
maps, argmax, gathers) must match exactly.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from __graft_entry__ import load_package
from oracle import kvmeta
from oracle import ops as O

load_package()
from loop_sglang_b200 import ops  # noqa: E402
from loop_sglang_b200._lib import check  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOL = dict(rtol=2e-2, atol=2e-2)


def bf(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16)


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def close(got: torch.Tensor, ref: torch.Tensor, **tol) -> None:
    torch.testing.assert_close(got.float().cpu(), ref.float(), **(tol or TOL))


def no_device_errors() -> None:
    assert ops.device_error_word(reset=True) == 0


@pytest.mark.parametrize("dim", [96, 128, 2048, 5280])
@pytest.mark.parametrize("rows", [1, 7, 33])
def test_norms(dim: int, rows: int) -> None:
    g = gen(dim + rows)
    x = bf(torch.randn(rows, dim, generator=g) * 3)
    r = bf(torch.randn(rows, dim, generator=g))
    wa = bf(1 + 0.1 * torch.randn(dim, generator=g))
    wb = bf(1 + 0.1 * torch.randn(dim, generator=g))
    eps = 1e-6
    close(ops.rmsnorm(x.to(DEV), wa.to(DEV), eps), O.rmsnorm(x, wa, eps))
    xd, rd = x.to(DEV), r.to(DEV)
    ops.fused_add_rmsnorm(xd, rd, wa.to(DEV), eps)
    ry, rr = O.fused_add_rmsnorm(x, r, wa, eps)
    close(xd, ry)
    assert torch.equal(rd.cpu(), rr), "fused add must store the exactly rounded sum"
    xd, rd = x.to(DEV), r.to(DEV)
    out = ops.sandwich_norm(xd, rd, wa.to(DEV), wb.to(DEV), eps)
    y = O.rmsnorm(x, wa, eps)
    sy, sr = O.fused_add_rmsnorm(y, r, wb, eps)
    close(out, sy)
    close(rd, sr, rtol=1e-2, atol=1e-2)
    # the sandwich may write over its input
    xd, rd = x.to(DEV), r.to(DEV)
    ops.sandwich_norm(xd, rd, wa.to(DEV), wb.to(DEV), eps, out=xd)
    close(xd, sy)


def test_norm_rejects_bad_dim() -> None:
    with pytest.raises(ValueError):
        ops.rmsnorm(torch.zeros(2, 12, dtype=torch.bfloat16, device=DEV),
                    torch.ones(12, dtype=torch.bfloat16, device=DEV), 1e-6)


@pytest.mark.parametrize("hq,hkv,d", [(4, 4, 32), (16, 16, 128), (8, 2, 64), (3, 3, 96)])
def test_rope_store(hq: int, hkv: int, d: int) -> None:
    g = gen(hq * d)
    t, slots = 9, 40
    qkv = bf(torch.randn(t, (hq + 2 * hkv) * d, generator=g))
    pos = torch.randint(0, 200, (t,), generator=g, dtype=torch.int32)
    cs = O.rope_cos_sin_cache(d, 256, 10000.0)
    loc = torch.tensor([0, 5, 7, 0, 39, 12, 1, 2, 3], dtype=torch.int32)
    kc = torch.full((slots, hkv * d), -3.0).to(torch.bfloat16)
    vc = kc.clone()
    qkv_d, kc_d, vc_d = qkv.to(DEV), kc.to(DEV), vc.to(DEV)
    ops.rope_store_kv(qkv_d, pos.to(DEV), cs.to(DEV), hq, hkv, d, kc_d, vc_d, loc.to(DEV))
    q = O.apply_rope_neox(pos, qkv[:, : hq * d].view(t, hq, d), cs).view(t, -1)
    k = O.apply_rope_neox(pos, qkv[:, hq * d:(hq + hkv) * d].view(t, hkv, d), cs).view(t, -1)
    v = qkv[:, (hq + hkv) * d:]
    close(qkv_d[:, : hq * d], q, rtol=1e-2, atol=1e-2)
    close(qkv_d[:, hq * d:(hq + hkv) * d], k, rtol=1e-2, atol=1e-2)
    ek, ev = kc.clone(), vc.clone()
    O.store_kv(ek, ev, loc, k, v)
    assert torch.equal(vc_d.cpu(), ev), "v rows are copied bit-exactly, slot 0 untouched"
    close(kc_d, ek, rtol=1e-2, atol=1e-2)
    assert torch.equal(kc_d[0].cpu(), kc[0])
    # the stored k is the rotated k left in the QKV output, bit for bit
    live = (loc != 0).nonzero().flatten()
    assert torch.equal(kc_d[loc[live].long()].cpu(), qkv_d[live, hq * d:(hq + hkv) * d].cpu())
    no_device_errors()
    # a slot outside the pool is skipped and flagged; the other rows are stored as before
    bad = loc.clone()
    bad[2] = slots + 3
    kc2, vc2 = kc.to(DEV), vc.to(DEV)
    ops.rope_store_kv(qkv.to(DEV), pos.to(DEV), cs.to(DEV), hq, hkv, d, kc2, vc2, bad.to(DEV))
    assert ops.device_error_word(reset=True) & 2
    keep = [r for r in range(t) if r != 2 and int(loc[r]) != 0]
    assert torch.equal(vc2[loc[keep].long()].cpu(), ev[loc[keep].long()])


@pytest.mark.parametrize("hq,hkv", [(16, 16), (8, 8), (16, 4)])
@pytest.mark.parametrize("m", [1, 5, 143, 263])
def test_gemm_rope_store_equals_gemm_then_rope_store(hq: int, hkv: int, m: int) -> None:
    """The QKV GEMM with RoPE + KV store in its epilogue: the same qkv output and cache
    contents, bit for bit, as the GEMM followed by rope_store_kv (128-dim heads), and
    within tolerance of the oracle."""
    g = gen(hq * 1000 + hkv * 10 + m)
    d, k = 128, 2048
    n = (hq + 2 * hkv) * d
    x = bf(torch.randn(m, k, generator=g))
    w = bf(torch.randn(n, k, generator=g) * 0.02)
    pos = torch.randint(0, 4000, (m,), generator=g, dtype=torch.int32)
    cs = O.rope_cos_sin_cache(d, 4096, 1e6)
    slots = 2 * m + 8
    loc = (torch.randperm(slots - 1, generator=g)[:m] + 1).to(torch.int32)
    loc[::4] = 0  # padding rows: never stored
    kc0 = bf(torch.randn(slots, hkv * d, generator=g))
    vc0 = bf(torch.randn(slots, hkv * d, generator=g))
    xd, wd, posd, csd, locd = x.to(DEV), w.to(DEV), pos.to(DEV), cs.to(DEV), loc.to(DEV)
    kc1, vc1 = kc0.to(DEV), vc0.to(DEV)
    qkv1 = ops.gemm(xd, wd)
    ops.rope_store_kv(qkv1, posd, csd, hq, hkv, d, kc1, vc1, locd)
    kc2, vc2 = kc0.to(DEV), vc0.to(DEV)
    qkv2 = ops.gemm_rope_store(xd, wd, posd, csd, hq, hkv, d, kc2, vc2, locd)
    assert torch.equal(qkv2, qkv1)
    assert torch.equal(kc2, kc1) and torch.equal(vc2, vc1)
    # against the oracle: projection, rotation of q and k, the store
    ref = O.linear(x, w)
    q = O.apply_rope_neox(pos, ref[:, : hq * d].view(m, hq, d), cs).view(m, -1)
    kr = O.apply_rope_neox(pos, ref[:, hq * d:(hq + hkv) * d].view(m, hkv, d), cs).view(m, -1)
    close(qkv2[:, : hq * d], q)
    close(qkv2[:, hq * d:(hq + hkv) * d], kr)
    close(qkv2[:, (hq + hkv) * d:], ref[:, (hq + hkv) * d:])
    no_device_errors()
    # a position outside the table and a slot outside the pool are flagged, not read/written
    bad_pos, bad_loc = pos.clone(), loc.clone()
    bad_pos[0] = 4096
    bad_loc[-1] = slots + 5 if int(loc[-1]) != 0 else 0
    ops.gemm_rope_store(xd, wd, bad_pos.to(DEV), csd, hq, hkv, d, kc0.to(DEV), vc0.to(DEV),
                        bad_loc.to(DEV))
    word = ops.device_error_word(reset=True)
    assert word & 1 and (int(bad_loc[-1]) == 0 or word & 2)


def test_gemm_rope_store_rejects_other_head_dims() -> None:
    x = torch.zeros(2, 64, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(3 * 96, 64, dtype=torch.bfloat16, device=DEV)
    kc = torch.zeros(4, 96, dtype=torch.bfloat16, device=DEV)
    pos = torch.zeros(2, dtype=torch.int32, device=DEV)
    cs = torch.zeros(8, 96, dtype=torch.float32, device=DEV)
    with pytest.raises(Exception, match="head_dim"):
        ops.gemm_rope_store(x, w, pos, cs, 1, 1, 96, kc, kc.clone(), pos)


def test_store_kv_exact_and_bounds() -> None:
    g = gen(3)
    k = bf(torch.randn(5, 2, 8, generator=g))
    v = bf(torch.randn(5, 2, 8, generator=g))
    idx = torch.tensor([0, 16, 0, 11, 7], dtype=torch.int32)
    kc = torch.full((17, 16), -7.0).to(torch.bfloat16)
    vc = kc.clone()
    kd, vd = kc.to(DEV), vc.to(DEV)
    ops.store_kv(kd, vd, idx.to(DEV), k.to(DEV), v.to(DEV))
    O.store_kv(kc.view(17, 2, 8), vc.view(17, 2, 8), idx.long(), k, v)
    assert torch.equal(kd.cpu(), kc) and torch.equal(vd.cpu(), vc)
    ops.store_kv(kd, vd, idx[:0].to(DEV), k[:0].to(DEV), v[:0].to(DEV))  # empty batch
    # an out-of-range slot is skipped and flagged, never written
    ops.store_kv(kd, vd, torch.tensor([99], dtype=torch.int32, device=DEV), k[:1].to(DEV),
                 v[:1].to(DEV))
    assert ops.device_error_word(reset=True) & 2
    assert torch.equal(kd.cpu(), kc)


def _paged_case(g, hq, hkv, d, page, q_lens, kv_lens):
    bsz = len(q_lens)
    max_pages = max((n + page - 1) // page for n in kv_lens)
    num_pages = bsz * max_pages + 16
    perm = torch.randperm(num_pages - 1, generator=g)[: bsz * max_pages] + 1
    table = perm.view(bsz, max_pages).to(torch.int32)
    kc = bf(torch.randn(num_pages, page, hkv, d, generator=g))
    vc = bf(torch.randn(num_pages, page, hkv, d, generator=g))
    q = bf(torch.randn(sum(q_lens), hq, d, generator=g))
    seq = torch.tensor(kv_lens, dtype=torch.int32)
    cu = torch.zeros(bsz + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(q_lens), 0)
    return q, kc, vc, table, seq, cu


@pytest.mark.parametrize("d", [64, 96, 128])
@pytest.mark.parametrize("page", [1, 16])
@pytest.mark.parametrize("mode", ["decode", "prefill", "long"])
def test_paged_attention(d: int, page: int, mode: str) -> None:
    g = gen(d * 7 + page)
    hq, hkv = (8, 2) if d == 64 else (4, 4)
    if mode == "decode":
        q_lens, kv_lens = [1, 1, 1, 1], [1, 17, 33, 100]
    elif mode == "prefill":
        q_lens, kv_lens = [5, 1, 12], [5, 40, 30]  # fresh prompt, decode row, cached prefix
    else:
        q_lens, kv_lens = [1, 2], [3000, 4100]  # many splits: exercises the merge
    q, kc, vc, table, seq, cu = _paged_case(g, hq, hkv, d, page, q_lens, kv_lens)
    scale = d ** -0.5
    ref = O.paged_attention(q, kc, vc, table, seq, cu, scale)
    kd = kc.to(DEV).view(-1, hkv * d)
    vd = vc.to(DEV).view(-1, hkv * d)
    max_seq = int(table.shape[1] * page)
    for _ in range(2):  # second call reuses the workspace: counters must be back at zero
        got = ops.paged_attention(q.to(DEV), kd, vd, table.to(DEV), seq.to(DEV), cu.to(DEV), page,
                                  max_seq, scale, hkv)
        close(got, ref)
    no_device_errors()


@pytest.mark.parametrize("kv_lens,launches", [([40, 50, 60, 64], 1), ([40, 3000, 900, 4100], 2)])
def test_paged_attention_launch_count(kv_lens: list[int], launches: int) -> None:
    """The library counts every kernel it enqueues: a decode call whose rows each end in
    one partial is one launch; one with split rows adds the partial merge (and its output
    still matches the oracle)."""
    from loop_sglang_b200 import _lib

    hq = hkv = 16
    d, page = 128, 16
    q, kc, vc, table, seq, cu = _paged_case(gen(sum(kv_lens)), hq, hkv, d, page, [1] * 4, kv_lens)
    scale = d ** -0.5
    kd = kc.to(DEV).view(-1, hkv * d)
    vd = vc.to(DEV).view(-1, hkv * d)
    args = (q.to(DEV), kd, vd, table.to(DEV), seq.to(DEV), cu.to(DEV), page,
            int(table.shape[1] * page), scale, hkv)
    ops.paged_attention(*args)  # workspace allocation and first-call setup
    before = _lib.launch_count()
    got = ops.paged_attention(*args)
    assert _lib.launch_count() - before == launches
    close(got, O.paged_attention(q, kc, vc, table, seq, cu, scale))
    no_device_errors()


@pytest.mark.parametrize("hq,hkv,d", [(16, 16, 128), (8, 2, 64), (55, 55, 96), (4, 4, 32)])
@pytest.mark.parametrize("page", [1, 16])
def test_paged_attention_prefill_tensor_cores(hq: int, hkv: int, d: int, page: int) -> None:
    """Prefill and extend rows (several query rows per request) take the mma.sync kernel:
    fresh prompts longer than one 64-row block and one 64-key tile, a request with a
    cached prefix, a decode row in the same batch, a request with no rows."""
    g = gen(hq * d + page)
    q_lens, kv_lens = [130, 64, 1, 77, 0], [130, 200, 50, 300, 9]
    q, kc, vc, table, seq, cu = _paged_case(g, hq, hkv, d, page, q_lens, kv_lens)
    scale = d ** -0.5
    ref = O.paged_attention(q, kc, vc, table, seq, cu, scale)
    kd = kc.to(DEV).view(-1, hkv * d)
    vd = vc.to(DEV).view(-1, hkv * d)
    got = ops.paged_attention(q.to(DEV), kd, vd, table.to(DEV), seq.to(DEV), cu.to(DEV), page,
                              int(table.shape[1] * page), scale, hkv)
    close(got, ref)
    no_device_errors()


@pytest.mark.parametrize("hq,hkv,d,page", [
    (55, 55, 96, 16),   # Huginn heads: a stage would exceed 64 KB -> per-CTA kernel
    (40, 8, 64, 16),    # 3 heads per consumer warp (streaming kernel, 4-head variant)
    (20, 4, 128, 1),    # 2 heads per consumer warp, one-token pages
    (16, 16, 32, 16),   # 32 tokens per stage
    (16, 8, 128, 1),    # scattered 2 KB rows: streaming kernel, one bulk copy pair per key
    (4, 4, 128, 1),     # scattered 1 KB rows (a TP=4 rank): per-CTA kernel, a warp per head
    (2, 2, 128, 1),     # a TP=8 rank: per-CTA kernel, two key sub-streams per head
    (2, 2, 128, 16),    # a TP=8 rank on 16-token pages: four pages per stage, one per lane
    (2, 2, 128, 12),    # the same with pages whose size is not a power of two
    (4, 2, 64, 8),      # eight 8-token pages per stage, grouped-query KV
    (1, 1, 64, 1),      # one head: four key sub-streams merged in shared memory
    (3, 1, 128, 1),     # three heads: one warp idle, grouped-query KV
])
@pytest.mark.parametrize("mode", ["decode", "long"])
def test_paged_attention_heads(hq: int, hkv: int, d: int, page: int, mode: str) -> None:
    """Head counts and widths on either side of the streaming kernel's limits."""
    g = gen(hq * 13 + d + page)
    if mode == "decode":
        q_lens, kv_lens = [1, 1, 1], [7, 64, 300]
    else:
        q_lens, kv_lens = [1, 3], [2500, 1900]
    q, kc, vc, table, seq, cu = _paged_case(g, hq, hkv, d, page, q_lens, kv_lens)
    scale = d ** -0.5
    ref = O.paged_attention(q, kc, vc, table, seq, cu, scale)
    kd = kc.to(DEV).view(-1, hkv * d)
    vd = vc.to(DEV).view(-1, hkv * d)
    max_seq = int(table.shape[1] * page)
    for _ in range(2):
        got = ops.paged_attention(q.to(DEV), kd, vd, table.to(DEV), seq.to(DEV), cu.to(DEV), page,
                                  max_seq, scale, hkv)
        close(got, ref)
    no_device_errors()


@pytest.mark.parametrize("hq,hkv,d", [(16, 16, 128), (55, 55, 96)])
def test_paged_attention_bad_page_flagged(hq: int, hkv: int, d: int) -> None:
    """A page id outside the pool is never read: its keys are skipped and the slot bit of
    the device error word is set; rows that do not touch it are unaffected."""
    g = gen(hq + d)
    page = 16
    q, kc, vc, table, seq, cu = _paged_case(g, hq, hkv, d, page, [1, 1], [40, 40])
    ref = O.paged_attention(q, kc, vc, table, seq, cu, d ** -0.5)
    num_pages = kc.shape[0]
    bad = table.clone()
    bad[1, 1] = num_pages + 5
    got = ops.paged_attention(q.to(DEV), kc.to(DEV).view(-1, hkv * d), vc.to(DEV).view(-1, hkv * d),
                              bad.to(DEV), seq.to(DEV), cu.to(DEV), page, int(bad.shape[1] * page),
                              d ** -0.5, hkv)
    assert ops.device_error_word(reset=True) & 2
    close(got[:1], ref[:1])
    assert torch.isfinite(got.float()).all()


def test_paged_attention_full_size_property() -> None:
    """Ouro-1.4B decode shape at full context: with every V row equal to one vector the
    output is that vector whatever the scores (a size-independent check), and sampled
    rows match the oracle."""
    g = gen(11)
    hq = hkv = 16
    d, page, bsz = 128, 16, 64
    kv_lens = torch.randint(512, 2049, (bsz,), generator=g).tolist()
    num_pages = sum((n + page - 1) // page for n in kv_lens) + 1
    table = (torch.randperm(num_pages - 1, generator=g) + 1).to(torch.int32)
    off = 0
    max_pages = max((n + page - 1) // page for n in kv_lens)
    pt = torch.zeros(bsz, max_pages, dtype=torch.int32)
    for b, n in enumerate(kv_lens):
        np_ = (n + page - 1) // page
        pt[b, :np_] = table[off:off + np_]
        off += np_
    kc = bf(torch.randn(num_pages, page, hkv, d, generator=g))
    const = bf(torch.randn(hkv, d, generator=g))
    vc = const.expand(num_pages, page, hkv, d).contiguous()
    q = bf(torch.randn(bsz, hq, d, generator=g))
    seq = torch.tensor(kv_lens, dtype=torch.int32)
    cu = torch.arange(bsz + 1, dtype=torch.int32)
    got = ops.paged_attention(q.to(DEV), kc.to(DEV).view(-1, hkv * d), vc.to(DEV).view(-1, hkv * d),
                              pt.to(DEV), seq.to(DEV), cu.to(DEV), page, max_pages * page,
                              d ** -0.5, hkv)
    close(got, const.unsqueeze(0).expand(bsz, hq, d), rtol=1e-2, atol=1e-2)
    vc2 = bf(torch.randn(num_pages, page, hkv, d, generator=g))
    got2 = ops.paged_attention(q.to(DEV), kc.to(DEV).view(-1, hkv * d),
                               vc2.to(DEV).view(-1, hkv * d), pt.to(DEV), seq.to(DEV),
                               cu.to(DEV), page, max_pages * page, d ** -0.5, hkv)
    for b in (0, 17, 63):
        ref = O.paged_attention(q[b:b + 1], kc, vc2, pt[b:b + 1], seq[b:b + 1],
                                torch.tensor([0, 1], dtype=torch.int32), d ** -0.5)
        close(got2[b:b + 1], ref)


GEMM_SHAPES = [(1, 128, 64), (3, 256, 128), (16, 384, 512), (144, 6144, 2048), (300, 256, 256),
               (8, 2048, 5632), (256, 1024, 2048), (40, 11264, 2048),
               # more than 256 tokens: two or more token tiles (CDB batch; a TP=2 rank's rows)
               (263, 6144, 2048), (512, 3072, 2048), (263, 2048, 5632),
               # ragged N and K (Huginn: H = 5280, QKV N = 15840; tiny shapes below 64 / 128)
               (7, 288, 96), (33, 15840, 5280), (5, 100, 40), (130, 5280, 10560)]


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
def test_gemm(m: int, n: int, k: int) -> None:
    g = gen(m + n + k)
    x = bf(torch.randn(m, k, generator=g))
    w = bf(torch.randn(n, k, generator=g) * 0.05)
    ref = O.linear(x, w)
    for _ in range(2):
        got = ops.gemm(x.to(DEV), w.to(DEV))
        close(got, ref)
    no_device_errors()


@pytest.mark.parametrize("plan", [1, 2, 3, 4])
@pytest.mark.parametrize("m,n,k,epi", [
    (263, 6144, 2048, "none"), (300, 2048, 5632, "none"), (384, 1024, 2048, "swiglu"),
    (289, 640, 352, "bias"), (143, 2048, 2048, "none"), (16, 2048, 2048, "none"),
    (70, 11264, 2048, "swiglu")])
def test_gemm_every_plan(plan: int, m: int, n: int, k: int, epi: str) -> None:
    """Each tile plan (one wide tile with two MMA halves, 96-token tiles, one CTA per SM,
    256-row tiles on CTA pairs) gives the oracle's product, fused epilogues included (640
    rows: the last pair's second CTA lies wholly past N)."""
    g = gen(m + n + k + plan)
    x = bf(torch.randn(m, k, generator=g))
    w = bf(torch.randn(n, k, generator=g) * 0.05)
    b = bf(torch.randn(n, generator=g))
    check(ops.lib().lsb_gemm_force_plan(plan), "force_plan")
    try:
        for _ in range(2):
            if epi == "swiglu":
                got = ops.gemm(x.to(DEV), ops.swiglu_interleave(w.to(DEV)),
                               epilogue=ops.LSB_EPI_SWIGLU)
                close(got, O.silu_and_mul(O.linear(x, w)))
            elif epi == "bias":
                close(ops.gemm(x.to(DEV), w.to(DEV), b.to(DEV), ops.LSB_EPI_BIAS),
                      O.linear(x, w, b))
            else:
                close(ops.gemm(x.to(DEV), w.to(DEV)), O.linear(x, w))
    finally:
        check(ops.lib().lsb_gemm_force_plan(0), "force_plan")
    no_device_errors()


def _with_plan(mode: int, fn):
    check(ops.lib().lsb_gemm_force_plan(mode), "force_plan")
    try:
        return fn()
    finally:
        check(ops.lib().lsb_gemm_force_plan(0), "force_plan")


@pytest.mark.parametrize("m,n,k,epi", [
    (1024, 6144, 2048, "none"), (1100, 640, 352, "bias"), (1300, 1024, 2048, "swiglu"),
    (2100, 2000, 1024, "bias_after_round"), (300, 2048, 5632, "none"), (8256, 2048, 704, "none")])
def test_gemm_persistent_matches_oracle_and_single_tile_kernel(m: int, n: int, k: int,
                                                               epi: str) -> None:
    """The persistent kernel (one CTA per SM over all tiles, two TMEM accumulators):
    the oracle's product with every epilogue, ragged token and weight tiles included, and
    the single-tile kernel's exact bits wherever that kernel's plan cuts the same 256-token
    tiles without split-K (then every output sums its K blocks in the same order)."""
    g = gen(m * 3 + n + k)
    x = bf(torch.randn(m, k, generator=g))
    w = bf(torch.randn(n, k, generator=g) * 0.05)
    b = bf(torch.randn(n, generator=g))
    xd, wd, bd = x.to(DEV), w.to(DEV), b.to(DEV)
    if epi == "swiglu":
        wi = ops.swiglu_interleave(wd)
        run = lambda: ops.gemm(xd, wi, epilogue=ops.LSB_EPI_SWIGLU)  # noqa: E731
        ref = O.silu_and_mul(O.linear(x, w))
    elif epi == "bias":
        run = lambda: ops.gemm(xd, wd, bd, ops.LSB_EPI_BIAS)  # noqa: E731
        ref = O.linear(x, w, b)
    elif epi == "bias_after_round":
        run = lambda: ops.gemm(xd, wd, bd, ops.LSB_EPI_BIAS_AFTER_ROUND)  # noqa: E731
        ref = O.linear_bias_after_rounding(x, w, b)
    else:
        run = lambda: ops.gemm(xd, wd)  # noqa: E731
        ref = O.linear(x, w)
    got = [_with_plan(5, run) for _ in range(2)]
    assert torch.equal(got[0], got[1])
    close(got[0], ref)
    classic = _with_plan(6, run)
    plan = _with_plan(6, lambda: ops.gemm_plan(m, n, k))
    if plan["splits"] == 1 and plan["tokens_per_tile"] == 256:
        assert torch.equal(got[0], classic)
    else:
        close(got[0], classic.float().cpu())
    no_device_errors()


def test_gemm_persistent_rope_store_equals_single_tile_kernel() -> None:
    """The QKV projection with RoPE + KV store at a prefill's token count: the persistent
    kernel's row-pair exchange gives the single-tile kernel's bits, output and caches."""
    g = gen(77)
    hq, hkv, d, k, m = 16, 4, 128, 2048, 1024
    n = (hq + 2 * hkv) * d
    x = bf(torch.randn(m, k, generator=g)).to(DEV)
    w = bf(torch.randn(n, k, generator=g) * 0.02).to(DEV)
    pos = torch.randint(0, 4000, (m,), generator=g, dtype=torch.int32).to(DEV)
    cs = O.rope_cos_sin_cache(d, 4096, 1e6).to(DEV)
    slots = 2 * m + 8
    loc = (torch.randperm(slots - 1, generator=g)[:m] + 1).to(torch.int32)
    loc[::5] = 0
    loc = loc.to(DEV)
    kc0 = bf(torch.randn(slots, hkv * d, generator=g)).to(DEV)
    vc0 = bf(torch.randn(slots, hkv * d, generator=g)).to(DEV)
    outs = []
    for mode in (5, 6):
        kc, vc = kc0.clone(), vc0.clone()
        qkv = _with_plan(mode, lambda: ops.gemm_rope_store(x, w, pos, cs, hq, hkv, d, kc, vc, loc))
        outs.append((qkv, kc, vc))
    plan = _with_plan(6, lambda: ops.gemm_plan(m, n, k))
    assert plan["splits"] == 1 and plan["tokens_per_tile"] == 256
    for a, c in zip(outs[0], outs[1]):
        assert torch.equal(a, c)
    no_device_errors()


@pytest.mark.parametrize("epi", ["bias", "bias_after_round", "swiglu"])
@pytest.mark.parametrize("m", [5, 144, 263])
def test_gemm_epilogues(epi: str, m: int) -> None:
    g = gen(m)
    k, n = 512, 1024
    x = bf(torch.randn(m, k, generator=g))
    w = bf(torch.randn(n, k, generator=g) * 0.05)
    b = bf(torch.randn(n, generator=g))
    if epi == "bias":
        close(ops.gemm(x.to(DEV), w.to(DEV), b.to(DEV), ops.LSB_EPI_BIAS), O.linear(x, w, b))
    elif epi == "bias_after_round":
        close(ops.gemm(x.to(DEV), w.to(DEV), b.to(DEV), ops.LSB_EPI_BIAS_AFTER_ROUND),
              O.linear_bias_after_rounding(x, w, b))
    else:
        wi = ops.swiglu_interleave(w.to(DEV))
        got = ops.gemm(x.to(DEV), wi, epilogue=ops.LSB_EPI_SWIGLU)
        close(got, O.silu_and_mul(O.linear(x, w)))
    no_device_errors()


@pytest.mark.parametrize("m,n,k1,k2", [
    (5, 5280, 5280, 5280),    # Huginn adapter: [h | injection] . W^T, K blocks of 64 straddle
    (130, 5280, 5280, 5280),  # each segment's end (5280 = 82.5 blocks)
    (17, 256, 40, 72),        # short, unaligned segments
])
def test_gemm_concat_matches_linear_of_cat(m: int, n: int, k1: int, k2: int) -> None:
    g = gen(m + k1)
    x1 = bf(torch.randn(m, k1, generator=g))
    x2 = bf(torch.randn(m, k2, generator=g))
    w = bf(torch.randn(n, k1 + k2, generator=g) * 0.02)
    b = bf(torch.randn(n, generator=g))
    ref = O.linear(torch.cat([x1, x2], dim=-1), w, b)
    for _ in range(2):
        close(ops.gemm_concat(x1.to(DEV), x2.to(DEV), w.to(DEV), b.to(DEV)), ref)
    close(ops.gemm_concat(x1.to(DEV), x2.to(DEV), w.to(DEV)),
          O.linear(torch.cat([x1, x2], dim=-1), w))
    no_device_errors()


@pytest.mark.parametrize("m", [3, 143, 263])
def test_gemm_argmax_equals_argmax_of_logits(m: int) -> None:
    """The LM head with greedy sampling in its epilogue picks exactly torch.argmax of the
    bf16 logits the plain GEMM writes, ties included (duplicate vocabulary rows within a
    tile and across tiles: the first index wins), with and without a vocabulary split."""
    g = gen(m)
    n, k = 4096 + 96, 512  # a partial last tile
    x = bf(torch.randn(m, k, generator=g))
    w = bf(torch.randn(n, k, generator=g) * 0.05)
    w[700] = w[3000] = w[4100] = w[200]  # the same logit at four indices, three tiles
    x[0] = bf(w[200].float() * 40)       # row 0 prefers them: its argmax is a tie -> 200
    w[130] = w[131]                      # a tie inside one tile
    x[1] = bf(w[131].float() * 40)
    xd, wd = x.to(DEV), w.to(DEV)
    logits = ops.gemm(xd, wd)
    want = torch.argmax(logits.float(), dim=-1).to(torch.int32).cpu()
    assert int(want[0]) in (200, 700, 3000, 4100) and int(want[1]) in (130, 131)
    pairs = ops.argmax_pairs_buffer(m, n, DEV)
    ops.gemm_argmax(xd, wd, pairs)
    got = ops.argmax_pairs(pairs, 1, m, -(-n // 128), n)
    assert torch.equal(got.cpu(), want)
    # two vocabulary shards of 2176 rows (the second padded with zero rows past n_valid),
    # stored shard-major as the all-gather leaves them
    half = 2176
    w2 = torch.zeros(2 * half, k, dtype=torch.bfloat16)
    w2[:n] = w
    shards = []
    for s in range(2):
        valid = min(half, n - s * half)
        p = ops.argmax_pairs_buffer(m, half, DEV)
        ops.gemm_argmax(xd, w2[s * half:(s + 1) * half].contiguous().to(DEV), p, n_valid=valid)
        shards.append(p)
    got2 = ops.argmax_pairs(torch.cat(shards), 2, m, -(-half // 128), half)
    assert torch.equal(got2.cpu(), want)
    no_device_errors()


def test_gemm_rejects_bad_shapes() -> None:
    x = torch.zeros(4, 100, dtype=torch.bfloat16, device=DEV)  # row stride 200 B: not TMA-able
    w = torch.zeros(128, 100, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        ops.gemm(x, w)
    with pytest.raises(ValueError):  # SwiGLU tiles need N % 128 == 0
        ops.gemm(torch.zeros(4, 64, dtype=torch.bfloat16, device=DEV),
                 torch.zeros(192, 64, dtype=torch.bfloat16, device=DEV),
                 epilogue=ops.LSB_EPI_SWIGLU)


def test_small_ops() -> None:
    g = gen(5)
    wt = bf(torch.randn(50, 64, generator=g))
    ids = torch.tensor([3, 12, 49, 29], dtype=torch.int32)
    assert torch.equal(ops.embedding(ids.to(DEV), wt.to(DEV)).cpu(), wt[ids.long()])
    close(ops.embedding(ids.to(DEV), wt.to(DEV), scale=1.5), bf(wt[ids.long()].float() * 1.5),
          rtol=0, atol=0)
    shard = ops.embedding(ids.to(DEV), wt[10:30].contiguous().to(DEV), vocab_start=10,
                          vocab_len=20)
    assert torch.equal(shard.cpu(), O.embedding(ids, wt[10:30], 10, 20))
    idx = torch.tensor([4, 4, 0, 49], dtype=torch.int64)
    assert torch.equal(ops.gather_rows(wt.to(DEV), idx.to(DEV)).cpu(), wt[idx])
    logits = bf(torch.randn(6, 1000, generator=g))
    logits[2, 10] = logits[2, 20] = 50.0  # tie: the first index wins
    logits5 = bf(torch.randn(3, 77, generator=g))
    assert torch.equal(ops.argmax(logits.to(DEV)).cpu(), O.greedy_sample(logits))
    assert torch.equal(ops.argmax(logits5.to(DEV)).cpu(), O.greedy_sample(logits5))
    x = bf(torch.randn(7, 2 * 136, generator=g))
    close(ops.silu_and_mul(x.to(DEV)), O.silu_and_mul(x), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("slots", [False, True])
def test_ouro_step_exit(slots: bool) -> None:
    g = gen(21)
    rows, dim, cap = 6, 256, 10
    x = bf(torch.randn(rows, dim, generator=g))
    r = bf(torch.randn(rows, dim, generator=g))
    w2 = bf(1 + 0.1 * torch.randn(dim, generator=g))
    wf = bf(1 + 0.1 * torch.randn(dim, generator=g))
    gw = bf(torch.randn(1, dim, generator=g) * 0.1)
    gb = bf(torch.tensor([0.2]))
    depth = torch.tensor([0, 1, 2, 0, 1, 3], dtype=torch.int32)
    state = torch.rand(cap, generator=g) * 0.5
    slot = torch.tensor([9, 1, 4, 0, 7, 2]) if slots else torch.arange(rows)
    y = O.rmsnorm(x, w2, 1e-6)
    h, _ = O.fused_add_rmsnorm(y, r, wf, 1e-6)
    sig, new = O.ouro_exit_signal(h, state[slot], depth, gw, gb, 0.45, min_loop_steps=2)
    hid = torch.zeros(cap, dim, dtype=torch.bfloat16, device=DEV)
    st = state.to(DEV)
    signal = torch.zeros(rows, dtype=torch.uint8, device=DEV)
    ops.ouro_step_exit(x.to(DEV), r.to(DEV), w2.to(DEV), wf.to(DEV), 1e-6, hidden_out=hid,
                       gate_w=gw.to(DEV), gate_b=gb.to(DEV), exit_state=st, signal=signal,
                       slot=slot.to(DEV) if slots else None, depth=depth.to(DEV),
                       threshold=0.45, min_loop_steps=2)
    close(hid[slot.to(DEV)], h)
    close(st[slot.to(DEV)], new, rtol=1e-3, atol=1e-3)
    margin = (new - 0.45).abs() > 1e-3
    assert torch.equal(signal.cpu().bool()[margin], sig[margin])


def test_huginn_step_exit() -> None:
    g = gen(22)
    rows, dim = 4, 96
    prev = bf(torch.randn(rows + 2, dim, generator=g))
    h = bf(torch.randn(rows, dim, generator=g))
    h[1] = prev[3]  # zero change -> exits
    slot = torch.tensor([5, 3, 0, 1])
    ref, _ = O.huginn_exit_signal(h, prev[slot], 0.9)
    st, hid = prev.to(DEV), torch.zeros_like(prev, device=DEV)
    signal = torch.zeros(rows, dtype=torch.uint8, device=DEV)
    ops.huginn_step_exit(h.to(DEV), st, hid, signal, 0.9, slot=slot.to(DEV))
    assert torch.equal(signal.cpu().bool(), ref)
    assert torch.equal(st[slot.to(DEV)].cpu(), h) and torch.equal(hid[slot.to(DEV)].cpu(), h)


@pytest.mark.parametrize("layout", [(8, 2, 6, 3, 12), (6, 0, 6, 4, 24), (24, 0, 24, 4, 40)])
def test_last_exited_maps(layout) -> None:
    """Reserve / alias / free / restore-reserve and resolve, bit-exact with the oracle
    (whose order the reference's Triton kernels follow under the interpreter)."""
    num_layers, cs, ce, steps, pages = layout
    lay = kvmeta.LastExitedLayout(num_layers, cs, ce, steps)
    ver = kvmeta.LastExitedVersions(lay, pages)
    slot_map = torch.zeros(lay.slots_per_token, pages, dtype=torch.int32, device=DEV)
    completed = torch.zeros(pages, dtype=torch.int32, device=DEV)
    free = torch.arange(1, ver.num_kv_slots, dtype=torch.int32, device=DEV)
    count = torch.tensor([ver.num_kv_slots - 1], dtype=torch.int32, device=DEV)
    fixed, core = lay.fixed_groups, lay.core_groups
    i32 = lambda a: torch.tensor(a, dtype=torch.int32, device=DEV)  # noqa: E731

    def check():
        assert torch.equal(slot_map.cpu(), torch.from_numpy(ver.slot_map))
        assert torch.equal(completed.cpu(), torch.from_numpy(ver.completed_depth))
        assert torch.equal(free.cpu(), torch.from_numpy(ver.free_slots))
        assert int(count.cpu()) == ver.free_count

    h1 = [3, 5, 1, 7]
    ops.last_exited_reserve(slot_map, completed, free, count, i32(h1), steps, fixed, core)
    ver.reserve(np.array(h1))
    check()
    ops.last_exited_release(slot_map, completed, free, count, i32([3, 5]), steps, fixed, core,
                            exits=i32([1, steps]))
    ver.release(np.array([3, 5]), np.array([1, steps]))
    check()
    ops.last_exited_release(slot_map, completed, free, count, i32([1]), steps, fixed, core)
    ver.release(np.array([1]))
    check()
    ops.last_exited_reserve(slot_map, completed, free, count, i32([4, 6]), steps, fixed, core,
                            restore_depths=i32([2, 1]))
    ver.reserve(np.array([4, 6]), np.array([2, 1]))
    check()
    table = torch.tensor([[5, 7, 4, 6], [6, 4, 0, 0], [7, 7, 5, 0]], dtype=torch.int32)
    seq = torch.tensor([4, 2, 3], dtype=torch.int32)
    cu = torch.tensor([0, 1, 3, 4], dtype=torch.int32)
    lout = torch.tensor([6, 4, 6, 5], dtype=torch.int32)
    depths = torch.tensor([0, steps - 1, 1], dtype=torch.int32)
    vm = slot_map[fixed:].view(steps, core, pages)
    pt = torch.full((core, 3, 4), -1, dtype=torch.int32, device=DEV)
    po = torch.full((core, 4), -1, dtype=torch.int32, device=DEV)
    ops.last_exited_resolve(table.to(DEV), vm, seq.to(DEV), cu.to(DEV), lout.to(DEV),
                            depths.to(DEV), pt, po)
    et = np.full((core, 3, 4), -1, np.int32)
    eo = np.full((core, 4), -1, np.int32)
    kvmeta.resolve_last_exited(table.numpy(), ver.version_map, seq.numpy(), cu.numpy(),
                               lout.numpy(), depths.numpy(), et, eo)
    assert np.array_equal(pt.cpu().numpy(), et) and np.array_equal(po.cpu().numpy(), eo)


def test_batch_metadata_golden() -> None:
    """Batch inputs and page-table metadata, bit-exact with the reference's Triton kernels
    (golden vectors from kernel/batch.py and attention/metadata.py run on the CPU)."""
    from replay import load

    fx = load("metadata")
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    r2t, seq, ext, rpi = d(fx["r2t"]), d(fx["seq"]), d(fx["ext"]), d(fx["rpi"])
    for tag, is_decode in (("decode", True), ("extend", False)):
        n = 3 if is_decode else int(fx["ext"].sum())
        pos = torch.zeros(n, dtype=torch.int32, device=DEV)
        mapping = torch.zeros_like(pos)
        loc = torch.zeros_like(pos)
        ops.prepare_batch_inputs(seq, ext, rpi, r2t, is_decode, pos, loc, mapping)
        assert np.array_equal(pos.cpu().numpy(), fx[f"{tag}_positions"])
        assert np.array_equal(mapping.cpu().numpy(), fx[f"{tag}_mapping"])
        assert np.array_equal(loc.cpu().numpy(), fx[f"{tag}_outloc"])
        cache = torch.zeros(3, dtype=torch.int32, device=DEV)
        cuk = torch.zeros(4, dtype=torch.int32, device=DEV)
        cuq = torch.zeros(4, dtype=torch.int32, device=DEV)
        pt = torch.full((3, 8), -1, dtype=torch.int32, device=DEV)
        maxp = (int(fx["seq"].max()) + 3) // 4
        ops.set_metadata(seq, ext, r2t, rpi, maxp, 4, is_decode, cache, cuk, cuq, pt)
        for got, key in ((cache, "cache"), (cuk, "cuk"), (cuq, "cuq"), (pt, "pt")):
            assert np.array_equal(got.cpu().numpy(), fx[f"{tag}_{key}"]), (tag, key)
