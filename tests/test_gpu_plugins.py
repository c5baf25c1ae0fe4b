"""The drop-in classes of ``plugins`` driven the way the reference's model code drives
them, against the oracle.

* ``B200AttnBackend`` through the reference's call sequence: ``prepare_metadata`` then
  ``forward`` for every layer of a prefill (attention/base.py:19-38, layers/attention.py
  :93-99); ``init_capture_graph`` / ``prepare_for_capture`` / ``forward`` captured in a
  CUDA graph, then ``prepare_for_replay`` + replay for a decode batch (the graph runner's
  order); under the last-exited policy ``prepare_core_metadata`` at layer 0 of every
  core step, with a scalar depth (prefill) and per-row depths (CDB decode), in the graph
  too. Outputs and the stored K/V are checked against the oracle's KV store and paged
  attention on the same tensors; tables and locations are integers and must match.
* The TP linear layers at TP=1, the norms, RoPE, SiLU*mul and ``store_cache`` against
  the oracle's restatements.
The batch is a structural stand-in of the reference's ``ForwardBatch`` (core.py:217-252).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from __graft_entry__ import load_package
from oracle import kvmeta
from oracle import ops as O
from oracle.model import SlotKVPool

load_package()
from loop_sglang_b200 import ops, plugins  # noqa: E402
from loop_sglang_b200.kvcache import LastExitedKVCache, MHAKVCache  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
HQ, HKV, D = 8, 2, 64
REL = 2e-2


@dataclass
class FwdBatch:
    """The fields of ``ForwardBatch`` the backend reads."""

    size: int
    phase: str
    req_pool_indices: torch.Tensor
    seq_lens: torch.Tensor
    extend_lens: torch.Tensor
    seq_lens_cpu: tuple
    extend_lens_cpu: tuple
    out_loc: torch.Tensor | None = None
    attn_metadata: object = field(default=None)

    @property
    def is_prefill(self) -> bool:
        return self.phase == "prefill"

    @property
    def is_decode(self) -> bool:
        return self.phase == "decode"

    @property
    def padded_size(self) -> int:
        return len(self.seq_lens_cpu)


def _close(got: torch.Tensor, want: torch.Tensor, what: str) -> None:
    got, want = got.float().cpu(), want.float().cpu()
    err = float((got - want).abs().max() / want.abs().max().clamp_min(1e-6))
    assert err < REL, f"{what}: rel err {err:.3e}"


def _token_table(rows: int, max_len: int, page: int, seed: int) -> torch.Tensor:
    """Token-granular request table [rows + 1, max_len] (row 0 padding): each request's
    tokens sit in its own random pages (location = page * page_size + offset)."""
    pages_per = (max_len + page - 1) // page
    g = torch.Generator().manual_seed(seed)
    perm = torch.randperm(rows * pages_per, generator=g) + 1
    t = torch.zeros(rows + 1, max_len, dtype=torch.int32)
    for r in range(rows):
        pages = perm[r * pages_per:(r + 1) * pages_per]
        locs = (pages.view(-1, 1) * page + torch.arange(page)).view(-1)[:max_len]
        t[r + 1] = locs.to(torch.int32)
    return t


def _batch(phase: str, table: torch.Tensor, rows: list[int], seq: list[int], ext: list[int]):
    """A batch and its (host) out_loc / positions, as prepare_batch_inputs would make them."""
    pos = torch.cat([torch.arange(s - e, s) for s, e in zip(seq, ext)]).to(torch.int32)
    rr = torch.cat([torch.full((e,), r) for r, e in zip(rows, ext)])
    out_loc = table[rr, pos.long()].to(torch.int32)
    b = FwdBatch(len(rows), phase, torch.tensor(rows, dtype=torch.int32, device=DEV),
                 torch.tensor(seq, dtype=torch.int32, device=DEV),
                 torch.tensor(ext, dtype=torch.int32, device=DEV), tuple(seq), tuple(ext),
                 out_loc.to(DEV))
    return b, out_loc, pos


def _qkv(t: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(t, HQ, D, generator=g).to(torch.bfloat16)
    k = torch.randn(t, HKV * D, generator=g).to(torch.bfloat16)
    v = torch.randn(t, HKV * D, generator=g).to(torch.bfloat16)
    return q, k, v


def _cu(ext: list[int]) -> torch.Tensor:
    cu = torch.zeros(len(ext) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(ext), 0)
    return cu


def test_attention_backend_paged_prefill_and_graph_decode() -> None:
    page, layers, max_len = 16, 2, 96
    rows = [1, 2, 3]
    table = _token_table(3, max_len, page, seed=1)
    num_pages = 3 * (max_len // page) + 1
    kv = MHAKVCache(HKV, layers, D, num_pages, page, DEV)
    ctx = SimpleNamespace(page_size=page, page_table=table.to(DEV), kv_cache=kv)
    cfg = SimpleNamespace(head_dim=D, num_kv_heads=HKV, num_qo_heads=HQ)
    be = plugins.B200AttnBackend(cfg, ctx)
    assert isinstance(be, plugins.BaseAttnBackend)
    okc = torch.zeros(layers, num_pages * page, HKV, D, dtype=torch.bfloat16)
    ovc = torch.zeros_like(okc)
    page_ids = (table[1:, ::page] // page).contiguous()

    def oracle(layer, q, k, v, out_loc, seq, cu):
        O.store_kv(okc[layer], ovc[layer], out_loc, k.view(-1, HKV, D), v.view(-1, HKV, D))
        kc = okc[layer].view(num_pages, page, HKV, D)
        vc = ovc[layer].view(num_pages, page, HKV, D)
        return O.paged_attention(q, kc, vc, page_ids, torch.tensor(seq, dtype=torch.int32), cu,
                                 D ** -0.5)

    # prefill: prompts of 5, 40 and 77 tokens
    seq = [5, 40, 77]
    b, out_loc, _ = _batch("prefill", table, rows, seq, seq)
    be.prepare_metadata(b)
    assert torch.equal(b.attn_metadata.get_last_indices(3).cpu(), _cu(seq)[1:] - 1)
    for layer in range(layers):
        q, k, v = _qkv(sum(seq), 10 + layer)
        got = be.forward(q.to(DEV), k.to(DEV), v.to(DEV), layer, b)
        _close(got, oracle(layer, q, k, v, out_loc, seq, _cu(seq)), f"prefill layer {layer}")
    for layer in range(layers):
        kc, _ = kv.slots(layer)
        assert torch.equal(kc.cpu().view(-1, HKV, D)[out_loc.long()],
                           okc[layer][out_loc.long()]), "stored K rows"

    # decode through captured graphs (one per layer): capture once, replay at later lengths
    be.init_capture_graph(max_len, [3])
    seq_c = [x + 1 for x in seq]
    cap, _, _ = _batch("decode", table, rows, seq_c, [1, 1, 1])
    static = {"q": torch.zeros(3, HQ, D, dtype=torch.bfloat16, device=DEV),
              "k": torch.zeros(3, HKV * D, dtype=torch.bfloat16, device=DEV),
              "v": torch.zeros(3, HKV * D, dtype=torch.bfloat16, device=DEV)}
    be.prepare_for_capture(cap)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graphs, outs = [], []
    with torch.cuda.stream(s):
        be.prepare_for_replay(cap)
        for layer in range(layers):  # warm-up sizes the workspace, then capture
            be.forward(static["q"], static["k"], static["v"], layer, cap)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                outs.append(be.forward(static["q"], static["k"], static["v"], layer, cap))
            graphs.append(g)
    torch.cuda.synchronize()
    for step in range(3):
        seq_s = [x + 1 + step for x in seq]
        rb, out_loc, _ = _batch("decode", table, rows, seq_s, [1, 1, 1])
        cap.seq_lens.copy_(rb.seq_lens)
        cap.seq_lens_cpu = rb.seq_lens_cpu
        cap.out_loc.copy_(rb.out_loc)
        be.prepare_for_replay(cap)
        for layer in range(layers):
            q, k, v = _qkv(3, 100 + 10 * step + layer)
            static["q"].copy_(q)
            static["k"].copy_(k)
            static["v"].copy_(v)
            graphs[layer].replay()
            torch.cuda.synchronize()
            ref = oracle(layer, q, k, v, out_loc, seq_s, torch.arange(4, dtype=torch.int32))
            _close(outs[layer], ref, f"decode step {step} layer {layer}")
    assert ops.device_error_word(reset=True) == 0


def test_attention_backend_last_exited_core_steps() -> None:
    steps, layers, max_len = 3, 2, 64
    rows = [1, 2, 3]
    prompts = [7, 20, 33]
    handles = (1 + torch.arange(3).view(-1, 1) * max_len + torch.arange(max_len)).to(torch.int32)
    table = torch.zeros(4, max_len, dtype=torch.int32)
    table[1:] = handles
    num_pages = 3 * max_len * steps + 1
    kv = LastExitedKVCache(HKV, layers, D, num_pages, 0, layers, steps, DEV)
    layout = kvmeta.LastExitedLayout(layers, 0, layers, steps)
    pool = SlotKVPool(layout, num_pages, HKV, D, torch.bfloat16)
    ctx = SimpleNamespace(page_size=1, page_table=table.to(DEV), kv_cache=kv)
    cfg = SimpleNamespace(head_dim=D, num_kv_heads=HKV, num_qo_heads=HQ)
    be = plugins.B200AttnBackend(cfg, ctx)
    assert be.last_exited

    def run(phase, seq, ext, depths, seed):
        b, out_loc, _ = _batch(phase, table, rows, seq, ext)
        be.prepare_metadata(b)
        md = b.attn_metadata
        be.prepare_core_metadata(b, depths if isinstance(depths, int)
                                 else torch.tensor(depths, dtype=torch.int32, device=DEV))
        cu = _cu(ext)
        ptab, oloc = kvmeta.resolve_last_exited(
            handles.numpy(), pool.versions.version_map, np.array(seq, np.int32), cu.numpy(),
            out_loc.numpy(), depths if isinstance(depths, int) else np.array(depths, np.int32))
        for r in range(3):
            assert np.array_equal(md.core_page_table[0, r, : seq[r]].cpu().numpy(),
                                  ptab[0, r, : seq[r]]), "resolved page table"
        assert np.array_equal(md.core_out_loc[0].cpu().numpy(), oloc[0]), "resolved out_loc"
        for layer in range(layers):
            q, k, v = _qkv(sum(ext), seed + layer)
            got = be.forward(q.to(DEV), k.to(DEV), v.to(DEV), layer, b)
            _, lane = layout.group_and_lane(layer)
            O.store_kv(pool.buf[0, lane], pool.buf[1, lane], torch.from_numpy(oloc[0]),
                       k.view(-1, HKV, D), v.view(-1, HKV, D))
            ref = O.paged_attention(q, pool.k_cache(layer), pool.v_cache(layer),
                                    torch.from_numpy(ptab[0]), torch.tensor(seq, dtype=torch.int32),
                                    cu, D ** -0.5)
            _close(got, ref, f"{phase} depths {depths} layer {layer}")

    b, out_loc, _ = _batch("prefill", table, rows, prompts, prompts)
    kv.reserve_versions(b.out_loc)
    pool.versions.reserve(out_loc.numpy())
    for step in range(steps):  # full-depth prefill: every loop step at its own depth
        run("prefill", prompts, prompts, step, 200 + 10 * step)
    seq = [p + 1 for p in prompts]
    b, out_loc, _ = _batch("decode", table, rows, seq, [1, 1, 1])
    kv.reserve_versions(b.out_loc)
    pool.versions.reserve(out_loc.numpy())
    run("decode", seq, [1, 1, 1], [0, 2, 1], 300)  # CDB rows at their own depths
    run("decode", seq, [1, 1, 1], [1, 0, 2], 310)
    assert ops.device_error_word(reset=True) == 0


def test_linear_norm_rope_plugins_match_oracle() -> None:
    g = torch.Generator().manual_seed(3)

    def r(*shape, s=0.05):
        return (torch.randn(*shape, generator=g) * s).to(torch.bfloat16)

    x = r(37, 256, s=1.0)
    for cls, args in ((plugins.LinearReplicated, (256, 192, True)),
                      (plugins.LinearOProj, (256, 128, False)),
                      (plugins.LinearRowParallel, (256, 320, True)),
                      (plugins.LinearColParallelMerged, (256, [128, 128], False)),
                      (plugins.LinearQKVMerged, (256, 32, 4, 2, True))):
        op = cls(*args)
        op.weight = r(*op.weight.shape)
        op.bias = None if op.bias is None else r(*op.bias.shape)
        op.weight = op.weight.to(DEV)
        op.bias = None if op.bias is None else op.bias.to(DEV)
        got = op.forward(x.to(DEV))
        want = O.linear(x, op.weight.cpu(), None if op.bias is None else op.bias.cpu())
        _close(got, want, cls.__name__)
    w = (1 + r(256, s=0.1).float()).to(torch.bfloat16)
    norm = plugins.RMSNorm(256, 1e-6)
    norm.weight = w.to(DEV)
    _close(norm.forward(x.to(DEV)), O.rmsnorm(x, w, 1e-6), "RMSNorm")
    fused = plugins.RMSNormFused(256, 1e-6)
    fused.weight = w.to(DEV)
    res = r(37, 256, s=1.0)
    xd, rd = x.to(DEV).clone(), res.to(DEV).clone()
    y, r2 = fused.forward(xd, rd)
    want_y, want_r = O.fused_add_rmsnorm(x, res, w, 1e-6)
    assert torch.equal(r2.cpu(), want_r), "fused residual is the bf16 sum, bit-exact"
    _close(y, want_y, "RMSNormFused")
    rope = plugins.RotaryEmbedding(64, 64, 512, 10000.0, device=DEV)
    pos = torch.randint(0, 512, (37,), generator=g, dtype=torch.int32)
    qh, kh = r(37, 4 * 64, s=1.0), r(37, 2 * 64, s=1.0)
    gq, gk = rope.forward(pos.to(DEV), qh.to(DEV).clone(), kh.to(DEV).clone())
    cs = O.rope_cos_sin_cache(64, 512, 10000.0)
    _close(gq, O.apply_rope_neox(pos, qh.view(37, 4, 64), cs).view(37, -1), "rope q")
    _close(gk, O.apply_rope_neox(pos, kh.view(37, 2, 64), cs).view(37, -1), "rope k")
    gu = r(37, 2 * 96, s=1.0)
    _close(plugins.silu_and_mul(gu.to(DEV)), O.silu_and_mul(gu), "silu_and_mul")
    kc = torch.zeros(64, 2, 64, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    idx = torch.tensor([5, 0, 9, 63], dtype=torch.int32, device=DEV)  # slot 0 is skipped
    kk, vv = r(4, 2, 64, s=1.0), r(4, 2, 64, s=1.0)
    plugins.store_cache(kc, vc, idx, kk.to(DEV), vv.to(DEV))
    okc, ovc = torch.zeros(64, 2, 64, dtype=torch.bfloat16), torch.zeros(64, 2, 64,
                                                                          dtype=torch.bfloat16)
    O.store_kv(okc, ovc, idx.cpu(), kk, vv)
    assert torch.equal(kc.cpu(), okc) and torch.equal(vc.cpu(), ovc), "store_cache"
