"""CPU oracle for the looped-decoder hot path.

TEST INFRASTRUCTURE ONLY. This package restates, on the CPU, the arithmetic and
integer bookkeeping of Loop-SGLang's looped-decoder hot path so that the CUDA
kernels of ``loop_sglang_b200`` can be checked against it. Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it, and there only as the checker or as the timed CPU
baseline. The product path never imports, calls or links anything here.

Parity pin: the restatements are checked against golden vectors produced by
running the reference's own Python and Triton code on the CPU
(``tests/golden/make_golden.py``; Triton kernels through the Triton
interpreter) and against the known answers of the reference's own unit tests.

Modules:
  ops     -- floating-point operators (norms, RoPE, SiLU*mul, linear, attention,
             exit gates, KV store).
  kvmeta  -- integer work: KV slot indices per looped-KV policy, page-table and
             batch-input metadata, last-exited version maps.
  model   -- Ouro / Huginn looped decoders built from ``ops`` over a paged KV pool.
  cdb     -- continuous-depth-batching exit routing.
  kvsnap  -- retraction snapshots of both KV pools (the reference's byte layout).
  radix   -- the radix prefix tree (match, split, insert, lock, evict).
  prefix_share -- attention over shared prefix pages split into per-group prefix and
             per-row suffix parts (the specification of a prefix-sharing pass).
"""
