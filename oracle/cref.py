"""ctypes wrapper of the C restatement (oracle/gdn_ref.c) — test
infrastructure only (checker and timed CPU baseline).

Build with ``make -C oracle``; arrays are numpy float32 (bf16 activations
widened), strides in elements.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libgdn_ref.so")
_LIB = None


def load():
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} missing: run `make -C oracle`")
        lib = C.CDLL(LIB_PATH)
        vp, i64, i32, f32 = C.c_void_p, C.c_int64, C.c_int, C.c_float
        lib.gdn_ref_num_threads.restype = C.c_int
        lib.gdn_ref_set_num_threads.argtypes = [C.c_int]
        lib.gdn_ref_set_num_threads.restype = None
        lib.gdn_ref_recurrent_inplace.argtypes = [vp, i64, vp, i64, vp, i64, vp, vp, vp, i64, vp,
                                                  i32, i32, i32, i32, i32, f32, vp]
        lib.gdn_ref_chunk_prefill.argtypes = [vp, i64, vp, i64, vp, i64, vp, vp, vp, i64, vp, vp,
                                              i32, i32, i32, i32, i32, f32, vp]
        _LIB = lib
    return _LIB


def num_threads() -> int:
    return load().gdn_ref_num_threads()


def use_all_cores() -> int:
    """Run the C restatement and numpy's BLAS on every host core (torchrun
    exports OMP_NUM_THREADS=1 to its workers); returns the thread count."""
    n = os.cpu_count() or 1
    load().gdn_ref_set_num_threads(n)
    try:
        import threadpoolctl
        threadpoolctl.threadpool_limits(limits=n)
    except Exception:   # BLAS thread control is best effort
        pass
    return num_threads()


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a


def _ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def recurrent_inplace(q, k, v, g, beta, s_pool, ids):
    """q/k [B, HK, DK], v [B, HV, DV], g/beta [B, HV]; s_pool float32
    [slots, HV, DK, DV] (contiguous; rows ids updated in place).  Returns
    out [B, HV, DV] float32."""
    q, k, v, g, beta = (_f32(x) for x in (q, k, v, g, beta))
    assert s_pool.dtype == np.float32 and s_pool.flags.c_contiguous
    B, HK, DK = q.shape
    HV, DV = v.shape[1], v.shape[2]
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    out = np.empty((B, HV, DV), np.float32)
    load().gdn_ref_recurrent_inplace(
        _ptr(q), HK * DK, _ptr(k), HK * DK, _ptr(v), HV * DV, _ptr(g), _ptr(beta), _ptr(s_pool),
        s_pool.strides[0] // 4, _ptr(ids), B, HK, HV, DK, DV, DK ** -0.5, _ptr(out))
    return out


def chunk_prefill(q, k, v, g, beta, s_pool, ids, cu_seqlens):
    """Varlen chunked prefill; q/k [N, HK, DK], v [N, HV, DV], g/beta
    [N, HV]; s_pool as recurrent_inplace.  Returns out [N, HV, DV]."""
    q, k, v, g, beta = (_f32(x) for x in (q, k, v, g, beta))
    assert s_pool.dtype == np.float32 and s_pool.flags.c_contiguous
    N, HK, DK = q.shape
    HV, DV = v.shape[1], v.shape[2]
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
    out = np.zeros((N, HV, DV), np.float32)
    load().gdn_ref_chunk_prefill(
        _ptr(q), HK * DK, _ptr(k), HK * DK, _ptr(v), HV * DV, _ptr(g), _ptr(beta), _ptr(s_pool),
        s_pool.strides[0] // 4, _ptr(ids), _ptr(cu), len(ids), HK, HV, DK, DV, DK ** -0.5,
        _ptr(out))
    return out
