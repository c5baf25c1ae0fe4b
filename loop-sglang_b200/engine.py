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
from .kvcache import LastExitedKVCache
from .model import DeviceBatch, LoopedDecoder
from .prefix_cache import find_shared_prefixes


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

    def share_prefixes(self) -> int:
        """Find the rows of the current batch whose page tables start with the same pages
        (requests that matched one radix-cache prefix) and let every attention call read a
        group's prefix once for all of its rows. Call after ``set_batch`` whenever the batch's
        rows change, before ``capture``; the groups stay valid while the rows only grow.
        Returns the number of groups."""
        ops.set_metadata(self.seq_lens, None, self.req_to_token, self.rpi, self.max_pages,
                         self.page, True, self.cache_seqlens, self.cu_k, self.cu_q,
                         self.page_table)
        groups = find_shared_prefixes(self.page_table.cpu().numpy(),
                                      self.cache_seqlens.cpu().numpy(), self.page,
                                      self.model.device)
        self.batch.prefix_groups = groups
        return 0 if groups is None else groups.num_groups

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
        self.stream.wait_stream(torch.cuda.current_stream())  # set-up work comes first
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


class CDBDecodeEngine:
    """Continuous-depth batching with the routing on the device (Ouro, last-exited KV).

    Every replay is one core step for every running row at its own depth
    (CDBModelRunner's core phase, cdb_model_runner.py:94-109), then, on the device:
    the exit decision of every row (gate, prescribed replay depth, or full depth;
    cdb_scheduler.py:189-267 with direct exit timing), greedy sampling of the rows
    that exit (the coda phase; Ouro's coda is the LM head), aliasing of their KV
    versions at the exit depth (cache.py:224-248), fresh versions for the successor
    position, and the successor's prelude (embedding) written into the row's state
    slot. The rows keep the batch full (the reference's refill mode); no host round
    trip is needed between steps, so steps replay back to back from one CUDA graph.
    Outputs (tokens and exit depths) accumulate on the device per row.
    """

    def __init__(self, model: LoopedDecoder, kv: LastExitedKVCache, batch_size: int,
                 max_len: int, out_capacity: int, replay_depths: torch.Tensor | None = None,
                 forced_ids: torch.Tensor | None = None) -> None:
        if model.cfg.arch != "ouro" or not isinstance(kv, LastExitedKVCache):
            raise ValueError("the device-routed CDB engine runs Ouro over a last-exited KV pool")
        dev = model.device
        self.model, self.kv, self.bs = model, kv, batch_size
        self.max_len = max_len
        b = batch_size
        i32 = dict(dtype=torch.int32, device=dev)
        self.req_to_token = torch.zeros(b + 1, align32(max_len), **i32)
        self.rpi = torch.arange(1, b + 1, **i32)
        self.slots = torch.arange(1, b + 1, dtype=torch.int64, device=dev)
        self.seq_lens = torch.ones(b, **i32)
        self.depth = torch.zeros(b, **i32)
        self.ids = torch.zeros(b, **i32)
        self.sampled = torch.zeros(b, **i32)
        self.signal = torch.zeros(b, dtype=torch.uint8, device=dev)
        self.exited = torch.zeros(b, dtype=torch.uint8, device=dev)
        self.alias_handle = torch.full((b,), -1, **i32)
        self.alias_depth = torch.zeros(b, **i32)
        self.reserve_handle = torch.full((b,), -1, **i32)
        self.out_count = torch.zeros(b, **i32)
        self.out_tokens = torch.zeros(b, out_capacity, **i32)
        self.out_depths = torch.zeros(b, out_capacity, **i32)
        self.produced = torch.zeros(1, **i32)
        self.replay_depths = replay_depths
        self.forced_ids = forced_ids
        h = model.cfg.hidden
        self.state = {"hidden": torch.zeros(b + 1, h, dtype=torch.bfloat16, device=dev),
                      "exit": torch.zeros(b + 1, dtype=torch.float32, device=dev)}
        self.positions = torch.zeros(b, **i32)
        self.out_loc = torch.zeros(b, **i32)
        self.cache_seqlens = torch.ones(b, **i32)
        self.cu_k = torch.arange(b + 1, **i32)
        self.cu_q = torch.arange(b + 1, **i32)
        self.page_table = torch.zeros(b, max_len, **i32)
        self.batch = DeviceBatch(self.ids, self.positions, self.out_loc, self.page_table,
                                 self.cache_seqlens, self.cu_q, False, max_seqlen=max_len)
        self.hidden_rows = torch.empty(b, h, dtype=torch.bfloat16, device=dev)
        self.emb = torch.empty(b, h, dtype=torch.bfloat16, device=dev)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.launches_per_step = 0
        self.stream = torch.cuda.Stream(device=dev)

    # ------------------------------------------------------------------ setup --
    def start(self, handles: torch.Tensor, seq_lens: torch.Tensor, ids: torch.Tensor) -> None:
        """Rows' token locations ``handles`` [B, >= max_len], lengths including the token
        about to be decoded, and that token's id: its versions are reserved (full depth)
        and its prelude written, at depth 0."""
        n = handles.shape[1]
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):  # the engine's stream orders every step after it
            self.req_to_token[1:, :n].copy_(handles)
            self.seq_lens.copy_(seq_lens)
            self.ids.copy_(ids)
            self.depth.zero_()
            cur = self.req_to_token[1:].gather(1, (self.seq_lens - 1).long().view(-1, 1)).view(-1)
            self.kv.reserve_versions(cur)
            self.model.embed_tokens(self.ids, out=self.emb)
            self.exited.fill_(1)
            ops.cdb_admit(self.state["hidden"], self.state["exit"], self.slots, self.exited,
                          self.emb)

    # ------------------------------------------------------------------- step --
    def _body(self) -> None:
        m, b, kv = self.model, self.batch, self.kv
        ops.prepare_batch_inputs(self.seq_lens, None, self.rpi, self.req_to_token, True,
                                 self.positions, self.out_loc)
        ops.set_metadata(self.seq_lens, None, self.req_to_token, self.rpi, self.max_len, 1, True,
                         self.cache_seqlens, self.cu_k, self.cu_q, self.page_table)
        m.core_step_exit(self.state, self.slots, self.depth, b, kv, self.signal)
        ops.gather_rows(self.state["hidden"], self.slots, out=self.hidden_rows)
        m.greedy(self.hidden_rows, None, out=self.sampled)
        ops.cdb_route(self.depth, self.seq_lens, self.ids, self.sampled,
                      self.signal if m.cfg.exit_threshold is not None else None, self.out_count,
                      self.alias_handle, self.alias_depth, self.reserve_handle, self.exited,
                      self.req_to_token, self.rpi, m.cfg.loop_steps, self.max_len,
                      replay_depths=self.replay_depths, forced_ids=self.forced_ids,
                      out_tokens=self.out_tokens, out_depths=self.out_depths,
                      produced=self.produced)
        ops.last_exited_release(kv.slot_map, kv.completed_depth, kv._free_slots, kv._free_count,
                                self.alias_handle, kv.loop_steps, kv.fixed_groups,
                                kv.core_groups, exits=self.alias_depth)
        ops.last_exited_reserve(kv.slot_map, kv.completed_depth, kv._free_slots, kv._free_count,
                                self.reserve_handle, kv.loop_steps, kv.fixed_groups,
                                kv.core_groups)
        m.embed_tokens(self.ids, out=self.emb)
        ops.cdb_admit(self.state["hidden"], self.state["exit"], self.slots, self.exited, self.emb)

    def step(self) -> None:
        """One core step, eagerly (no graph)."""
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            self._body()

    def capture(self) -> None:
        """One warm-up step (sizes every workspace), then capture one step. The warm-up is a
        real step: it advances the rows."""
        self.stream.wait_stream(torch.cuda.current_stream())
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
        assert self.graph is not None, "capture() first"
        self.graph.replay()
