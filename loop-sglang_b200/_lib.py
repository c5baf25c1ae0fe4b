"""ctypes binding of ``libloopsgl_b200.so`` (the C ABI declared in ``include/loopsgl_b200.h``).

The shared library is built in-tree by ``build.py``. Loading fails loudly when it
is missing: there is no Python or CPU fallback for any kernel.
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int32, c_int64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libloopsgl_b200.so")

LSB_OK = 0
LSB_ERR_INVALID = 1
LSB_ERR_CUDA = 2
LSB_ERR_TIMEOUT = 3
LSB_ERR_UNSUPPORTED = 4

LSB_EPI_NONE = 0
LSB_EPI_BIAS = 1
LSB_EPI_BIAS_AFTER_ROUND = 2
LSB_EPI_SWIGLU = 3

LSB_DEVERR_POSITION = 1
LSB_DEVERR_SLOT = 2
LSB_DEVERR_SEQLEN = 4
LSB_DEVERR_TIMEOUT = 8
LSB_DEVERR_COMM_TIMEOUT = 16

LSB_IPC_HANDLE_BYTES = 64

P = c_void_p
I64 = c_int64
I32 = c_int32
F = c_float

# name -> (restype, argtypes); every entry point of include/loopsgl_b200.h
SIGNATURES: dict[str, tuple[object, list]] = {
    "lsb_last_error": (ctypes.c_char_p, []),
    "lsb_abi_version": (ctypes.c_int, []),
    "lsb_kernel_launch_count": (c_int64, []),
    "lsb_device_error_word": (ctypes.c_int, [P, I32, P]),
    "lsb_rmsnorm": (ctypes.c_int, [P, I64, P, I64, P, I64, I64, F, P]),
    "lsb_fused_add_rmsnorm": (ctypes.c_int, [P, P, P, I64, I64, F, P]),
    "lsb_sandwich_norm": (ctypes.c_int, [P, P, P, P, P, I64, I64, F, P]),
    "lsb_rope_store_kv": (ctypes.c_int, [P, I64, P, P, I64, P, P, I64, I64, P, I64, I32, I32, I32,
                                         P]),
    "lsb_store_kv": (ctypes.c_int, [P, P, I64, I64, P, I64, P, I64, P, I64, I64, P]),
    "lsb_paged_attention_workspace_size": (c_int64, [I64, I32, I32, I64]),
    "lsb_paged_attention_plan": (ctypes.c_int, [I64, I32, I32, I32, I32, I64, I64, P]),
    "lsb_paged_attention": (ctypes.c_int, [P, I64, P, I64, P, P, I64, I64, P, I64, P, P, I64, I64,
                                           I32, I32, I32, I32, I64, F, P, I64, P]),
    "lsb_paged_attention_noalloc": (ctypes.c_int, [P, I64, P, I64, P, P, I64, I64, P, I64, P, P,
                                                   I64, I64, I32, I32, I32, I32, I64, F, P]),
    "lsb_paged_attention_shared_prefix_workspace_size": (c_int64, [I64, I32, I32, I64, I64]),
    "lsb_paged_attention_shared_prefix": (ctypes.c_int, [P, I64, P, I64, P, P, I64, I64, P, I64,
                                                         P, P, I64, I64, I32, I32, I32, I32, I64,
                                                         F, P, P, P, P, I64, I64, I64, P, I64,
                                                         P]),
    "lsb_gemm_workspace_size": (c_int64, [I64, I64, I64]),
    "lsb_gemm": (ctypes.c_int, [P, I64, P, I64, P, I64, P, I64, I64, I64, I32, P, I64, P]),
    "lsb_gemm_plan": (ctypes.c_int, [I64, I64, I64, P]),
    "lsb_gemm_argmax_tiles": (I64, [I64]),
    "lsb_gemm_force_plan": (ctypes.c_int, [I32]),
    "lsb_gemm_rope_store": (ctypes.c_int, [P, I64, P, I64, P, I64, I64, I64, I64, P, P, I64, P,
                                           P, I64, I64, P, I32, I32, I32, P]),
    "lsb_comm_set_protocol": (ctypes.c_int, [P, I32]),
    "lsb_gemm_force_tile_tokens": (ctypes.c_int, [I32]),
    "lsb_attention_force_kernel": (ctypes.c_int, [I32]),
    "lsb_gemm_argmax": (ctypes.c_int, [P, I64, P, I64, P, I64, I64, I64, I64, P]),
    "lsb_argmax_pairs": (ctypes.c_int, [P, P, I64, I64, I64, I64, I64, P]),
    "lsb_gemm_concat": (ctypes.c_int, [P, I64, P, I64, P, I64, P, I64, P, I64, I64, I64, I64,
                                       I32, P]),
    "lsb_swiglu_interleave": (ctypes.c_int, [P, P, I64, I64, P]),
    "lsb_ouro_step_exit": (ctypes.c_int, [P, I64, P, P, P, P, P, P, P, P, P, P, I32, I32, I32, F,
                                          I64, I64, F, P]),
    "lsb_huginn_step_exit": (ctypes.c_int, [P, P, P, P, P, F, I64, I64, P]),
    "lsb_embedding": (ctypes.c_int, [P, P, P, I64, I64, I64, I64, F, P]),
    "lsb_gather_rows": (ctypes.c_int, [P, P, P, I64, I64, P]),
    "lsb_argmax": (ctypes.c_int, [P, P, I64, I64, I64, P]),
    "lsb_argmax_sharded": (ctypes.c_int, [P, P, I64, I64, I64, I64, P]),
    "lsb_silu_and_mul": (ctypes.c_int, [P, P, I64, I64, P]),
    "lsb_last_exited_resolve": (ctypes.c_int, [P, I64, I64, P, I64, P, I64, P, I64, I64, P, P, P,
                                               P, I32, I64, I64, I32, P]),
    "lsb_prepare_batch_inputs": (ctypes.c_int, [P, P, P, P, P, P, P, I64, I64, I32, P]),
    "lsb_set_metadata": (ctypes.c_int, [P, P, P, P, I64, P, I64, P, P, P, I64, I64, I32, I32, I32,
                                        P]),
    "lsb_last_exited_reserve": (ctypes.c_int, [P, P, I64, P, P, P, P, I64, I32, I32, I32, P]),
    "lsb_last_exited_release": (ctypes.c_int, [P, P, I64, P, P, P, P, I64, I32, I32, I32, P]),
    "lsb_cdb_route": (ctypes.c_int, [P, P, P, P, P, P, P, I64, P, P, P, P, P, P, P, P, I64, P, I64,
                                     I32, I32, P, P]),
    "lsb_cdb_admit": (ctypes.c_int, [P, I64, P, P, P, P, I64, I64, P]),
    "lsb_comm_buffer_bytes": (c_int64, [I64]),
    "lsb_comm_alloc": (ctypes.c_int, [I64, P]),
    "lsb_comm_free": (ctypes.c_int, [P]),
    "lsb_ipc_handle": (ctypes.c_int, [P, P]),
    "lsb_ipc_open": (ctypes.c_int, [P, P]),
    "lsb_ipc_close": (ctypes.c_int, [P]),
    "lsb_comm_create": (ctypes.c_int, [I32, I32, P, I64, P]),
    "lsb_comm_destroy": (ctypes.c_int, [P]),
    "lsb_allreduce": (ctypes.c_int, [P, P, I64, I64, I64, P]),
    "lsb_allgather": (ctypes.c_int, [P, P, P, I64, P]),
    "lsb_gemm_allreduce": (ctypes.c_int, [P, P, I64, P, I64, P, I64, P, I64, I64, I64, I32, P]),
    "lsb_kv_snapshot_bytes": (c_int64, [I64, I64, I32, I32, I32, I32, I32]),
    "lsb_kv_backup": (ctypes.c_int, [P, P, I64, I64, I64, P, I64, P, I64, P, I32, I32, I32, I32, P,
                                     I64, P]),
    "lsb_kv_restore": (ctypes.c_int, [P, P, I64, I64, I64, P, I64, P, I64, I32, I32, I32, I32, P,
                                      I64, P]),
    "lsb_fast_compare_key": (ctypes.c_int, [P, I64, P, I64, I32, P]),
    "lsb_radix_create": (ctypes.c_int, [I32, P]),
    "lsb_radix_destroy": (ctypes.c_int, [P]),
    "lsb_radix_match": (ctypes.c_int, [P, P, I64, P, P]),
    "lsb_radix_insert": (ctypes.c_int, [P, P, P, I64, P, P, P]),
    "lsb_radix_lock": (ctypes.c_int, [P, I64, I32]),
    "lsb_radix_indices": (ctypes.c_int, [P, I64, P, I64, P]),
    "lsb_radix_evict": (ctypes.c_int, [P, I64, P, I64, P]),
    "lsb_radix_size_info": (ctypes.c_int, [P, P, P]),
    "lsb_radix_check": (ctypes.c_int, [P]),
}

_lib: ctypes.CDLL | None = None


class LsbError(RuntimeError):
    """A C entry point returned a non-zero status."""


def lib() -> ctypes.CDLL:
    """Load the shared library once and declare every signature."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run loop-sglang_b200/build.py (needs nvcc)"
            )
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    """Turn a non-zero status into an exception carrying ``lsb_last_error``."""
    if rc == LSB_OK:
        return
    msg = lib().lsb_last_error().decode(errors="replace")
    if rc == LSB_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    raise LsbError(f"{what} failed ({rc}): {msg}")


def launch_count() -> int:
    """Kernels the library has enqueued so far in this process (its own count, taken at
    every successful launch inside the C entry points)."""
    return int(lib().lsb_kernel_launch_count())


def call(name: str, *args) -> None:
    """Invoke an entry point and raise on a non-zero status."""
    check(getattr(lib(), name)(*args), name)
