"""Batched full-depth decode over a paged KV pool, replayed as one CUDA graph per step.

This is the decode step of the continuous-batching path (managers/scheduler.py:132-174
-> ModelRunner.forward_batch, model_executor/model_runner.py:258-277, graph replay
graph.py:164-171) with every kernel from ``libloopsgl_b200.so``:

  batch inputs (kernel/batch.py:72-129) -> attention metadata (attention/metadata.py:59-216)
  -> embedding -> loop_steps x core layers -> LM head -> greedy argmax.

The scheduler-side inputs of a step are the requests' sequence lengths and request
rows (``seq_lens`` counts the token being decoded); the sampled tokens are written
back into the input-id buffer, so consecutive replays decode consecutive tokens.
"""

from __future__ import annotations

import torch

from . import _lib, ops
from .model import DeviceBatch, LoopedDecoder


def align32(n: int) -> int:
    return (n + 31) // 32 * 32


class DecodeEngine:
    """Fixed-size decode batch with static device buffers (CUDA-graph friendly)."""

    def __init__(self, model: LoopedDecoder, kv, batch_size: int, max_len: int, page_size: int,
                 max_reqs: int | None = None) -> None:
        dev = model.device
        self.model, self.kv, self.bs, self.page = model, kv, batch_size, page_size
        self.max_pages = (max_len + page_size - 1) // page_size
        rows = (max_reqs or batch_size) + 1
        i32 = dict(dtype=torch.int32, device=dev)
        # ModelRunner's token-granular page table [max_running_req+1, align32(max_seq_len)]
        # (model_runner.py:104-111); row 0 is the padding row.
        self.req_to_token = torch.zeros(rows, align32(self.max_pages * page_size), **i32)
        self.ids = torch.zeros(batch_size, **i32)
        self.seq_lens = torch.ones(batch_size, **i32)
        self.rpi = torch.ones(batch_size, **i32)
        self.positions = torch.zeros(batch_size, **i32)
        self.out_loc = torch.zeros(batch_size, **i32)
        self.cache_seqlens = torch.ones(batch_size, **i32)
        self.cu_k = torch.arange(batch_size + 1, **i32)
        self.cu_q = torch.arange(batch_size + 1, **i32)
        self.page_table = torch.zeros(batch_size, self.max_pages, **i32)
        self.batch = DeviceBatch(self.ids, self.positions, self.out_loc, self.page_table,
                                 self.cache_seqlens, self.cu_q, False,
                                 max_seqlen=self.max_pages * page_size)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.launches_per_step = 0
        self.stream = torch.cuda.Stream(device=dev)
        self._host_tokens = torch.zeros(batch_size, dtype=torch.int32, pin_memory=True)

    # ------------------------------------------------------------------ setup --
    def assign_pages(self, row: int, pages: torch.Tensor) -> None:
        """Give request row ``row`` the page ids ``pages`` (in order) for its whole length."""
        p = self.page
        locs = (pages.to(torch.int64).view(-1, 1) * p + torch.arange(p, device=pages.device)).view(-1)
        n = min(locs.numel(), self.req_to_token.shape[1])
        self.req_to_token[row, :n] = locs[:n].to(torch.int32).to(self.req_to_token.device)

    def set_batch(self, req_rows: torch.Tensor, seq_lens: torch.Tensor) -> None:
        """Scheduler inputs of the next step: request rows and lengths (incl. the new token)."""
        self.rpi.copy_(req_rows, non_blocking=True)
        self.seq_lens.copy_(seq_lens, non_blocking=True)

    # ------------------------------------------------------------------- step --
    def _body(self) -> None:
        m, b = self.model, self.batch
        ops.prepare_batch_inputs(self.seq_lens, None, self.rpi, self.req_to_token, True,
                                 self.positions, self.out_loc)
        ops.set_metadata(self.seq_lens, None, self.req_to_token, self.rpi, self.max_pages,
                         self.page, True, self.cache_seqlens, self.cu_k, self.cu_q,
                         self.page_table)
        h, inj = m.forward_prelude(b, self.kv)
        for step in range(m.cfg.loop_steps):
            h = m.core_step(h, step, inj, b, self.kv)
        m.greedy(m.forward_coda(h, b, self.kv), b, out=self.ids)

    def capture(self) -> None:
        """Warm up (sizes every workspace), then capture one decode step."""
        with torch.cuda.stream(self.stream):
            before = _lib.launch_count()
            self._body()
            self.launches_per_step = _lib.launch_count() - before
            self.stream.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=self.stream):
                self._body()
        self.stream.synchronize()

    def replay(self) -> None:
        """One decode step on the device (inputs already resident)."""
        assert self.graph is not None, "capture() first"
        self.graph.replay()

    def decode_step_host(self, req_rows: torch.Tensor, seq_lens: torch.Tensor) -> torch.Tensor:
        """The public per-step call with host buffers: H2D of the scheduler inputs (pinned),
        one step, D2H of the sampled tokens (the CDB/CB token readback,
        cdb_model_runner.py:184-194)."""
        with torch.cuda.stream(self.stream):
            self.set_batch(req_rows, seq_lens)
            self.graph.replay()
            self._host_tokens.copy_(self.ids, non_blocking=True)
        self.stream.synchronize()
        return self._host_tokens
