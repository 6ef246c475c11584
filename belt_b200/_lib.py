"""ctypes binding of ``libbelt_b200.so`` (the C ABI declared in ``include/belt_b200.h``).

The library is built in-tree by ``python -m belt_b200.build``. There is no fallback: if it is missing or does not
load, every operator raises.
"""

from __future__ import annotations

import ctypes
import os

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libbelt_b200.so")

c_i32, c_i64, c_f32, c_vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p
c_i32p = ctypes.POINTER(ctypes.c_int32)

# name -> argument types (all return int status)
SIGNATURES = {
    "belt_decode_schedule": [c_vp, c_i32, c_i32, c_i32, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp],
    "belt_decode_schedule_weighted": [c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_i64, c_vp, c_vp, c_vp, c_vp],
    "belt_decode_schedule_balanced": [c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp, c_vp, c_vp, c_i64, c_vp, c_vp,
                                      c_vp, c_vp],
    "belt_block_diag_query": [c_vp, c_i64, c_i64, c_i64, c_vp, c_i32, c_i32p, c_vp, c_vp, c_vp],
    "belt_up_project": [c_vp, c_i64, c_i64, c_i64, c_i32, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp],
    "belt_latent_rows_to_cache": [c_vp, c_i64, c_i64, c_vp, c_i32, c_vp, c_i64, c_i32, c_i32, c_i64, c_i64, c_vp,
                                  c_i32, c_i32p, c_f32, c_vp],
    "belt_latent_proj_rows_to_cache": [c_vp, c_i64, c_i64, c_i32, c_vp, c_i64, c_vp, c_i32, c_vp, c_i64, c_i32, c_i32,
                                       c_i64, c_i64, c_vp, c_i32, c_i32p, c_f32, c_vp, c_vp],
    "belt_latent_decode": [c_vp, c_i32, c_i32, c_vp, c_i64, c_i32, c_i32, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp,
                           c_vp, c_i32, c_vp, c_i64, c_i64, c_f32, c_i32, c_i32, c_i32p, c_vp, c_i32, c_vp, c_i32,
                           c_vp, c_vp],
    "belt_latent_decode_timed": [c_vp, c_i32, c_i32, c_vp, c_i64, c_i32, c_i32, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp,
                                 c_vp, c_i32, c_vp, c_i64, c_i64, c_f32, c_i32, c_i32, c_i32p, c_vp, c_i32, c_vp,
                                 c_i32, c_vp, c_vp, c_vp],
    "belt_merge_segments": [c_vp, c_i64, c_i64, c_vp, c_i32, c_i32, c_i32, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp],
    "belt_latent_decode_noalloc": [c_vp, c_i32, c_i32, c_vp, c_i64, c_i32, c_i32, c_i64, c_i64, c_vp, c_i64, c_vp,
                                   c_i32, c_i32, c_f32, c_i32, c_i32, c_i32p, c_vp, c_i32, c_vp, c_i32, c_vp, c_i64,
                                   c_i64, c_vp, c_i64, c_vp, c_vp],
    "belt_latent_decompress": [c_vp, c_i64, c_i32, c_i32, c_i64, c_i64, c_vp, c_i32, c_i32, c_i32, c_vp, c_i32,
                               c_i32p, c_vp, c_i32, c_i32, c_vp, c_i32, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp],
    "belt_latent_decompress_varlen": [c_vp, c_i64, c_i32, c_i32, c_i64, c_i64, c_vp, c_i64, c_i32, c_i32p, c_vp,
                                      c_i32, c_i32p, c_vp, c_i32, c_i32, c_vp, c_i32, c_vp, c_vp, c_i64, c_i64, c_vp,
                                      c_vp],
    "belt_prefill_attention_varlen": [c_vp, c_i64, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, c_i64, c_i32, c_i32p, c_i32,
                                      c_f32, c_vp, c_vp, c_i64, c_i64, c_vp, c_vp, c_i64, c_vp, c_vp],
    "belt_attn_fold": [c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_i32, c_i32p, c_vp],
    "belt_prefill_attention": [c_vp, c_i32, c_i64, c_i64, c_vp, c_vp, c_i32, c_i64, c_i64, c_i32, c_i32, c_i32, c_f32,
                               c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp],
    "belt_q_norm_rope": [c_vp, c_i32, c_i64, c_i64, c_vp, c_f32, c_vp, c_i32, c_i32, c_vp, c_i32, c_vp, c_i64, c_i64,
                         c_vp],
    "belt_gate_mul": [c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_i32, c_vp, c_i64, c_i64, c_vp],
    "belt_merge_up_project": [c_vp, c_i64, c_i64, c_vp, c_i32, c_i32, c_vp, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp,
                              c_vp],
    "belt_gemm_bf16": [c_vp, c_i64, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp],
    "belt_selftest_bounded_wait": [c_vp, c_vp, c_vp],
    "belt_num_sms": [c_i32],
    "belt_path_counts": [c_vp, c_i32],
    "belt_abi_version": [],
}

_lib = None


class BeltError(RuntimeError):
    """A belt_* C call returned an error status."""


def lib_path() -> str:
    return _LIB_PATH


def load():
    """The loaded library (loads it on first use). Raises ``BeltError`` if it is not built or does not load."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        raise BeltError(f"{_LIB_PATH} is not built: run `python -m belt_b200.build` (needs nvcc)")
    import torch  # noqa: F401  (loads the CUDA runtime the library links against first)
    lib = ctypes.CDLL(_LIB_PATH)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    lib.belt_last_error.argtypes = []
    lib.belt_last_error.restype = ctypes.c_char_p
    _lib = lib
    return lib


def call(name: str, *args) -> None:
    """Call ``name`` and raise ``ValueError`` (invalid argument) or ``BeltError`` (CUDA failure) on a bad status."""
    lib = load()
    status = getattr(lib, name)(*args)
    if status != 0:
        msg = lib.belt_last_error().decode(errors="replace")
        if status == -1:
            raise ValueError(f"{name}: {msg}")
        raise BeltError(f"{name}: {msg}")


def int_array(values) -> ctypes.Array:
    vals = [int(v) for v in values]
    return (ctypes.c_int32 * len(vals))(*vals)


def path_counts() -> dict:
    """Launches that took a CUDA-core fallback because TMA could not describe the operands (``belt_path_counts``)."""
    out = (ctypes.c_int64 * 2)()
    call("belt_path_counts", ctypes.cast(out, ctypes.c_void_p), 2)
    return {"simt_group_gemm": int(out[0]), "simt_cache_write": int(out[1])}
