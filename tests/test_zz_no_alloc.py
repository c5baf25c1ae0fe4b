"""The allocation-free paged-attention entry point matches the workspace one.

``lsb_paged_attention_noalloc`` exists for callers that cannot allocate device memory
(a plugin whose host framework owns all device memory and passes only inputs and
outputs, or a loop that must not pay cudaMalloc's device-wide synchronisation); its
split-KV scratch is a static device array. This file is collected last so that a
failure here leaves every other test already run; it also passes alone in a fresh
process (its first call sets up the array on the device).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from __graft_entry__ import load_package

load_package()
from loop_sglang_b200 import _lib, ops  # noqa: E402

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _case(seed: int, q_lens, kv_lens, hq=4, hkv=4, d=128, page=16):
    g = torch.Generator().manual_seed(seed)
    bsz = len(q_lens)
    max_pages = max((n + page - 1) // page for n in kv_lens)
    num_pages = bsz * max_pages + 4
    table = (torch.randperm(num_pages - 1, generator=g)[: bsz * max_pages] + 1).view(bsz, -1)
    kc = torch.randn(num_pages * page, hkv * d, generator=g).to(torch.bfloat16)
    vc = torch.randn(num_pages * page, hkv * d, generator=g).to(torch.bfloat16)
    q = torch.randn(sum(q_lens), hq, d, generator=g).to(torch.bfloat16)
    cu = torch.zeros(bsz + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(q_lens), 0)
    t = lambda x: x.to(DEV)  # noqa: E731
    return (t(q), t(kc), t(vc), t(table.to(torch.int32).contiguous()),
            t(torch.tensor(kv_lens, dtype=torch.int32)), t(cu), hq, hkv, d, page,
            max_pages * page)


def _noalloc(q, kc, vc, table, seq, cu, hq, hkv, d, page, max_seq) -> torch.Tensor:
    out = torch.empty_like(q)
    rc = _lib.lib().lsb_paged_attention_noalloc(
        out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), kc.data_ptr(), vc.data_ptr(),
        kc.stride(0), kc.shape[0], table.data_ptr(), table.stride(0), seq.data_ptr(),
        cu.data_ptr(), seq.numel(), q.shape[0], hq, hkv, d, page, max_seq,
        ctypes.c_float(d ** -0.5), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "lsb_paged_attention_noalloc")
    return out


@pytest.mark.parametrize("q_lens,kv_lens,shape", [
    ([1, 1, 1], [40, 300, 2000], {}),   # decode rows, several splits (streaming kernel)
    ([1, 2], [3000, 4100], {}),         # long rows: many splits merged through the scratch
    ([5, 1, 12], [5, 40, 30], {}),      # prefill rows with a cached prefix
    # one-token pages with 2 KV heads of 128 (under 2 KB of K per key): the per-CTA
    # kernel, whose split partials and (row, head group) counters also use the scratch
    ([1, 1, 3], [700, 2900, 1500], {"hq": 8, "hkv": 2, "page": 1}),
])
def test_noalloc_matches_workspace_entry_point(q_lens, kv_lens, shape) -> None:
    args = _case(7, q_lens, kv_lens, **shape)
    q, kc, vc, table, seq, cu, hq, hkv, d, page, max_seq = args
    ref = ops.paged_attention(q, kc, vc, table, seq, cu, page, max_seq, d ** -0.5, hkv)
    for _ in range(2):  # two calls in a row: the shared scratch must come back clean
        got = _noalloc(*args)
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), ref.float(), rtol=2e-2, atol=2e-2)
    assert ops.device_error_word(reset=True) == 0


def test_noalloc_rejects_oversized_calls() -> None:
    cap = 16 * 1024 * 1024
    need = _lib.lib().lsb_paged_attention_workspace_size(60000, 64, 128, 1 << 20)
    assert need > cap
    dummy = torch.zeros(16, dtype=torch.bfloat16, device=DEV)
    idx = torch.zeros(4, dtype=torch.int32, device=DEV)
    rc = _lib.lib().lsb_paged_attention_noalloc(
        dummy.data_ptr(), 8192, dummy.data_ptr(), 8192, dummy.data_ptr(), dummy.data_ptr(), 128,
        1, idx.data_ptr(), 1, idx.data_ptr(), idx.data_ptr(), 1, 60000, 64, 64, 128, 16, 1 << 20,
        ctypes.c_float(1.0), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.LSB_ERR_INVALID
    assert b"static" in _lib.lib().lsb_last_error()
