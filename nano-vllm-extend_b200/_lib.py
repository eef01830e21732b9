"""ctypes binding of libgdn_b200.so (the C ABI declared in include/gdn_b200.h).

The library is the product's only compute path: there is no CPU or PyTorch
fallback.  Loading fails loudly (``ImportError``) when the built library is
missing; build it with ``python nano-vllm-extend_b200/build.py`` or
``__graft_entry__.build()``.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libgdn_b200.so")

GDN_OK = 0
GDN_ERR_INVALID_ARGUMENT = 1
GDN_ERR_UNSUPPORTED = 2
GDN_ERR_CUDA = 3
GDN_STATUS_BAD_SLOT = 0x1
GDN_STATUS_BAD_SEQLEN = 0x2
GDN_STATUS_TIMEOUT = 0x4
GDN_DTYPE_F32 = 0
GDN_DTYPE_BF16 = 1

vp, i32, i64, f32 = C.c_void_p, C.c_int32, C.c_int64, C.c_float

# name -> argtypes, in the order of include/gdn_b200.h
SIGNATURES = {
    "gdn_abi_version": [],
    "gdn_last_error": [],
    "gdn_set_wait_limit": [i64],
    "gdn_fused_g_beta": [vp, vp, i64, i64, i32, vp, vp, i32, vp, vp, vp, vp],
    "gdn_conv_decode_step": [vp, i64, vp, i64, i64, vp, i32, i32, i32, vp, vp, i64, vp, vp],
    "gdn_causal_conv_silu_varlen": [vp, i64, vp, i64, i64, vp, vp, i32, i64, i32, i32, vp, vp,
                                    i64, vp, vp],
    "gdn_conv_gate_varlen": [vp, i64, vp, i64, i64, vp, vp, i32, i64, i32, i32, vp, vp, i64,
                             vp, vp, i64, i32, vp, vp, i32, vp, vp, vp, vp],
    "gdn_recurrent_inplace": [vp, i64, vp, i64, vp, i64, vp, vp, vp, i64, i64, vp, vp, i32, i32,
                              i32, i32, i32, f32, vp, i64, vp, f32, vp, vp],
    "gdn_chunk_prefill_workspace_bytes": [i64, i32, i32, i32, i32],
    "gdn_chunk_prefill_varlen": [vp, i64, vp, i64, vp, i64, vp, vp, vp, i64, i64, vp, vp, i32,
                                 i64, i32, vp, i32, i32, i32, i32, f32, vp, i64, vp, f32, vp, i64,
                                 vp, vp],
    "gdn_rms_norm_gated": [vp, vp, i64, i32, vp, vp, i64, i32, f32, vp],
    "gdn_decode_fused": [vp, i64, vp, i64, vp, vp, i64, vp, i64, vp, i32, vp, vp, i32, vp, i64,
                         i64, vp, vp, f32, vp, i32, i32, i32, i32, f32, vp, vp, vp],
    "gdn_decode_fused_static": [vp, i64, vp, i64, vp, vp, i64, vp, i64, vp, i32, vp, vp, i32, vp,
                                i64, i64, vp, vp, f32, vp, i32, i32, i32, i32, f32, vp, vp],
}

_LIB = None


def load() -> C.CDLL:
    """Load (once) and return the library with its signatures set."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libgdn_b200.so not found at {LIB_PATH}; build it with "
            "`python nano-vllm-extend_b200/build.py` (there is no fallback path)")
    lib = C.CDLL(LIB_PATH)
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = {"gdn_last_error": C.c_char_p, "gdn_set_wait_limit": None,
                      "gdn_chunk_prefill_workspace_bytes": C.c_int64}.get(name, C.c_int)
    _LIB = lib
    return lib


class GdnError(RuntimeError):
    """A CUDA-side failure reported by the library (GDN_ERR_CUDA)."""


def check(rc: int, fn: str) -> None:
    """Raise the Python error matching a library return code."""
    if rc == GDN_OK:
        return
    msg = load().gdn_last_error().decode(errors="replace") or fn
    if rc == GDN_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    if rc == GDN_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise GdnError(msg)
