"""B200 (sm_100a) looped-decoder hot path of Loop-SGLang.

Hand-written CUDA kernels (``csrc/``) behind a C ABI (``include/loopsgl_b200.h``),
loaded with ctypes from the in-tree ``libloopsgl_b200.so``:

* ``ops``      -- one wrapper per C entry point (torch tensors in, kernel launch out);
* ``kvcache``  -- device KV pools of the depth-indexed / shared / last-exited policies;
* ``model``    -- Ouro and Huginn looped decoders built from the fused kernels;
* ``plugins``  -- drop-ins with the reference's attention-backend, TP-linear and
                  communicator interfaces;
* ``engine``   -- batched decode runner (CUDA graphs) used by ``bench.py``.

The directory name carries a hyphen, so the package is imported as
``loop_sglang_b200`` through ``__graft_entry__.load_package``.
"""

from . import _lib  # noqa: F401  (fails loudly if the library is missing)

__all__ = ["_lib"]
