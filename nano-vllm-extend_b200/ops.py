"""Tensor-level GDN operators over the C ABI (libgdn_b200.so).

Each function keeps the name and argument meaning of the reference operator it
replaces (sileaver/nano-vllm-extend, nanovllm/models/qwen3_5.py) and raises on
the same contract violations (``AssertionError`` for the layout asserts the
reference makes, ``ValueError`` / ``NotImplementedError`` for what the library
rejects).  Kernels launch on the current CUDA stream and never synchronise, so
every operator is CUDA-graph capturable.  Where the reference gathers and
scatters pool rows around a kernel, these operators take the pool view and the
slot ids and update the slots in place.

Slot-id faults never touch memory: the kernels skip such rows and raise a bit
in a per-device status word.  Two ways read it:

* :func:`check_status` synchronises, reads and clears it (tests, debug paths);
* :func:`publish_status` enqueues an asynchronous copy of the word into pinned
  host memory on the current stream (capturable: a CUDA graph replays it), and
  :func:`poll_status` reads that host copy without synchronising and raises if
  a bit is set.  Every layer polls before it runs; one layer per device (the
  first to run, :func:`is_status_publisher`) publishes after its kernels — a
  copy node costs ~12 us inside a decode graph, so one per step rather than
  one per layer.  A fault is published at the latest in the step after the
  one whose kernels saw it and raises at the next poll after that; an engine
  that replays whole decode steps from a CUDA graph calls
  :func:`poll_status` between steps.

Optional host-side checks (:func:`set_debug_checks`, or ``GDN_DEBUG_CHECKS=1``)
validate slot ids and ``cu_seqlens`` before each launch and raise at once.
"""
from __future__ import annotations

import os
import weakref

import numpy as np
import torch

from . import _lib

_STATUS: dict[int, torch.Tensor] = {}


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def status_word(device) -> torch.Tensor:
    """The int32 device status word the kernels OR fault bits into."""
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _STATUS.get(idx)
    if t is None:
        # a normal tensor even when first made under inference_mode, so that
        # check_status can clear it anywhere
        with torch.inference_mode(False):
            t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _STATUS[idx] = t
    return t


def _raise_for(v: int) -> int:
    if v & _lib.GDN_STATUS_BAD_SLOT:
        raise IndexError(f"GDN kernel saw a slot id outside the pool (status {v:#x})")
    if v & _lib.GDN_STATUS_TIMEOUT:
        raise _lib.GdnError(f"GDN kernel gave up a bounded device-side wait (status {v:#x})")
    if v & _lib.GDN_STATUS_BAD_SEQLEN:
        raise ValueError(f"GDN kernel saw malformed cu_seqlens / max_seqlen (status {v:#x})")
    return v


def check_status(device=None, clear: bool = True) -> int:
    """Read (and clear) the status word; raise if a kernel flagged a fault.
    Synchronises with the device."""
    device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
    st = status_word(device)
    v = int(st.item())
    if clear:
        st.zero_()
        h = _HOST_STATUS.get(st.device.index)
        if h is not None:
            h.zero_()
    return _raise_for(v)


_HOST_STATUS: dict[int, torch.Tensor] = {}


def _host_status(idx: int) -> torch.Tensor:
    t = _HOST_STATUS.get(idx)
    if t is None:
        with torch.inference_mode(False):
            t = torch.zeros(1, dtype=torch.int32).pin_memory()
        _HOST_STATUS[idx] = t
    return t


def publish_status(device) -> None:
    """Enqueue a copy of the device status word into this device's pinned host
    mirror on the current stream (no synchronisation; recorded into a CUDA
    graph when called under capture)."""
    st = status_word(device)
    _host_status(st.device.index).copy_(st, non_blocking=True)


_PUBLISHER: dict[int, weakref.ref] = {}


def is_status_publisher(module, device) -> bool:
    """Whether ``module`` publishes the status word of ``device``: the first
    module to ask claims it and keeps it while it is alive (a model built later
    claims it once the earlier one is gone)."""
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ref = _PUBLISHER.get(idx)
    owner = ref() if ref is not None else None
    if owner is None:
        _PUBLISHER[idx] = weakref.ref(module)
        return True
    return owner is module


def reset_status_publisher(device=None) -> None:
    """Forget the publishing module of ``device`` (all devices when None), so
    the next module to run claims it."""
    if device is None:
        _PUBLISHER.clear()
        return
    device = torch.device(device)
    _PUBLISHER.pop(device.index if device.index is not None else torch.cuda.current_device(),
                   None)


def poll_status(device=None) -> int:
    """Raise if the pinned host mirror holds a fault bit (no synchronisation:
    it reflects the last published copy that has completed).  Raising clears
    the device word (stream-ordered) and the mirror.  Returns the mirrored
    value (0 when clean)."""
    device = torch.device(device) if device is not None else \
        torch.device("cuda", torch.cuda.current_device())
    idx = device.index if device.index is not None else torch.cuda.current_device()
    h = _HOST_STATUS.get(idx)
    if h is None:
        return 0
    v = int(h[0])
    if v:
        status_word(device).zero_()
        h.zero_()
        _raise_for(v)
    return v


def set_wait_limit(polls: int | None) -> None:
    """Test hook (gdn_set_wait_limit): the poll limit of the head-per-CTA
    decode form's bounded wait for its state copy; None restores the
    default.  Calls made while a limit is set give invalid results."""
    _lib.load().gdn_set_wait_limit(-1 if polls is None else int(polls))


_DEBUG_CHECKS = os.environ.get("GDN_DEBUG_CHECKS", "0") not in ("", "0")


def set_debug_checks(on: bool) -> None:
    """Host-side argument checks before every launch (off by default; also
    on with ``GDN_DEBUG_CHECKS=1``): slot ids inside the pool and not repeated
    within one call, except the pool's last slot (the engine's dummy slot,
    which CUDA-graph pad rows share); ``cu_seqlens`` starting at 0,
    non-decreasing and ending at the row count.  Each check copies the ids /
    ``cu_seqlens`` to the host, a synchronisation, so checks are skipped while
    a CUDA graph is being captured.  The kernels' own handling stays as it is:
    without the checks a bad slot is skipped and flagged in the status word,
    and repeated slots are undefined, as in the reference."""
    global _DEBUG_CHECKS
    _DEBUG_CHECKS = bool(on)


def check_slot_ids(ids, num_slots: int) -> None:
    """Raise IndexError for a slot id outside [0, num_slots) and ValueError
    for a slot id given more than once (the last slot excepted)."""
    v = np.asarray(ids.cpu() if isinstance(ids, torch.Tensor) else ids, np.int64).reshape(-1)
    bad = (v < 0) | (v >= num_slots)
    if bad.any():
        raise IndexError(f"slot id {int(v[bad][0])} outside the pool of {num_slots} slots")
    u, n = np.unique(v[v != num_slots - 1], return_counts=True)
    if (n > 1).any():
        raise ValueError(f"slot id {int(u[n > 1][0])} appears {int(n[n > 1][0])} times in "
                         "one call (the rows would race on its state)")


def check_cu_seqlens(cu, n_rows: int, max_seqlen: int | None = None) -> None:
    """Raise ValueError unless cu starts at 0, never decreases and ends at
    n_rows, and (when given) no sequence is longer than max_seqlen."""
    c = np.asarray(cu.cpu() if isinstance(cu, torch.Tensor) else cu, np.int64).reshape(-1)
    if c.size == 0 or c[0] != 0 or c[-1] != n_rows or (np.diff(c) < 0).any():
        raise ValueError(f"cu_seqlens must start at 0, not decrease and end at {n_rows} "
                         f"(got {c[:4].tolist()} ... {c[-2:].tolist()})")
    if max_seqlen is not None and c.size > 1 and int(np.diff(c).max()) > max_seqlen:
        raise ValueError(f"a sequence of {int(np.diff(c).max())} rows exceeds max_seqlen "
                         f"{max_seqlen}")


def _debug_checks(ids=None, num_slots: int = 0, cu=None, n_rows: int = 0,
                  max_seqlen: int | None = None) -> None:
    if not _DEBUG_CHECKS or torch.cuda.is_current_stream_capturing():
        return
    if ids is not None:
        check_slot_ids(ids, num_slots)
    if cu is not None:
        check_cu_seqlens(cu, n_rows, max_seqlen)


def _out_buffer(out, shape, device) -> torch.Tensor:
    """A bf16 output of `shape`: `out` itself when given (a contiguous tensor of
    that shape, e.g. a row slice of a larger buffer), else a new tensor."""
    if out is None:
        return torch.empty(*shape, dtype=torch.bfloat16, device=device)
    assert tuple(out.shape) == tuple(shape) and out.dtype == torch.bfloat16 and \
        out.is_contiguous() and out.device == torch.device(device), \
        f"out must be a contiguous bf16 tensor of shape {tuple(shape)}"
    return out


def _p(t) -> int:
    return 0 if t is None else t.data_ptr()


def _cuda(*ts):
    for t in ts:
        if t is not None:
            assert t.is_cuda, "GDN operators take CUDA tensors"


def _ids64(ids: torch.Tensor) -> torch.Tensor:
    assert ids.dim() == 1, "linear_state_ids must be 1-D"
    if ids.dtype != torch.int64 or not ids.is_contiguous():
        ids = ids.to(torch.int64).contiguous()
    return ids


def _rows2d(x: torch.Tensor, width: int) -> tuple[torch.Tensor, int]:
    """View x as [rows, width] rows with a row stride (last dim dense)."""
    x2 = x.reshape(-1, width) if x.is_contiguous() else x
    if x2.dim() != 2:
        x2 = x.reshape(-1, width)
    assert x2.stride(-1) == 1, "last dimension must be dense"
    return x2, x2.stride(0)


# ---------------------------------------------------------------------------
# (b) gate
# ---------------------------------------------------------------------------


def fused_g_beta(b: torch.Tensor, a: torch.Tensor, a_log: torch.Tensor,
                 dt_bias: torch.Tensor, mask: torch.Tensor | None = None):
    """qwen3_5.py:346-360.  b/a [.., Vh] bf16 (rows may be strided views);
    a_log/dt_bias [Vh]; mask [..] bool or None (False rows get g = 0).
    Returns (g fp32 [.., Vh], beta bf16 [.., Vh]), both contiguous."""
    _cuda(b, a, a_log, dt_bias, mask)
    assert b.dtype == torch.bfloat16 and a.dtype == torch.bfloat16
    assert a.shape == b.shape
    vh = a.shape[-1]
    assert a_log.numel() == vh and dt_bias.numel() == vh
    lead = a.shape[:-1]
    if a.dim() != 2 or b.dim() != 2 or a.stride(0) != b.stride(0) or a.stride(1) != 1 \
            or b.stride(1) != 1:
        a = a.reshape(-1, vh).contiguous()
        b = b.reshape(-1, vh).contiguous()
    n = a.shape[0]
    assert a_log.dtype == dt_bias.dtype
    pdt = _lib.GDN_DTYPE_BF16 if a_log.dtype == torch.bfloat16 else _lib.GDN_DTYPE_F32
    if pdt == _lib.GDN_DTYPE_F32:
        a_log, dt_bias = a_log.float().contiguous(), dt_bias.float().contiguous()
    else:
        a_log, dt_bias = a_log.contiguous(), dt_bias.contiguous()
    g = torch.empty(*lead, vh, dtype=torch.float32, device=a.device)
    beta = torch.empty(*lead, vh, dtype=torch.bfloat16, device=a.device)
    m = None
    if mask is not None:
        m = mask.reshape(-1).to(torch.uint8).contiguous()
        assert m.numel() == n
    rc = _lib.load().gdn_fused_g_beta(
        _p(b), _p(a), a.stride(0), n, vh, _p(a_log), _p(dt_bias), pdt, _p(m), _p(g), _p(beta),
        _stream_ptr(a.device))
    _lib.check(rc, "gdn_fused_g_beta")
    return g, beta


# ---------------------------------------------------------------------------
# (a) conv
# ---------------------------------------------------------------------------


def _slot_stride(pool: torch.Tensor) -> int:
    """Distance between consecutive slots; for a one-slot pool the stride of
    the slot dim is meaningless (torch/numpy may report 0), so use the
    slot's own size."""
    if pool.shape[0] > 1:
        return pool.stride(0)
    return max(pool.stride(0), pool[0].numel())


def _pool_view_check(pool: torch.Tensor, taps: int, channels: int):
    assert pool.dim() == 3 and pool.shape[1] == channels and pool.shape[2] == taps, \
        f"conv pool view must be [slots, {channels}, {taps}]"
    assert pool.stride(2) == 1 and pool.stride(1) == taps, "conv pool taps must be dense"
    assert pool.dtype == torch.bfloat16


def conv_decode_step(x: torch.Tensor, state_pool: torch.Tensor, ids: torch.Tensor,
                     weight: torch.Tensor) -> torch.Tensor:
    """qwen3_5.py:550-558.  x [n, C] (rows may be strided); state_pool
    [slots, C, K-1] rolled in place at rows ``ids``; weight [C, K] (or the
    conv1d weight [C, 1, K]).  Returns y [n, C]."""
    _cuda(x, state_pool, ids, weight)
    C = x.shape[-1]
    w = weight.reshape(C, -1).contiguous()
    K = w.shape[1]
    _pool_view_check(state_pool, K - 1, C)
    assert x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
    x2, xs = _rows2d(x, C)
    n = x2.shape[0]
    ids = _ids64(ids)
    assert ids.numel() == n
    _debug_checks(ids, state_pool.shape[0])
    y = torch.empty(n, C, dtype=x.dtype, device=x.device)
    rc = _lib.load().gdn_conv_decode_step(
        _p(x2), xs, _p(state_pool), _slot_stride(state_pool), state_pool.shape[0], _p(ids), n, C, K,
        _p(w), _p(y), y.stride(0), _p(status_word(x.device)), _stream_ptr(x.device))
    _lib.check(rc, "gdn_conv_decode_step")
    return y


def causal_conv_silu_varlen(x: torch.Tensor, state_pool: torch.Tensor, ids: torch.Tensor,
                            weight: torch.Tensor, cu_seqlens: torch.Tensor) -> torch.Tensor:
    """Varlen causal conv + SiLU (qwen3_5.py:459-473), with each sequence's
    prefix state read from and rolled in place in ``state_pool[ids[r]]``
    (the gather/scatter of qwen3_5.py:941-946 is not needed).  x [N, C];
    cu_seqlens int32 [n+1] on the device.  Returns y [N, C] (the reference's
    [3, N, C/3] slabs are its own layout; q/k/v are column views of y here)."""
    _cuda(x, state_pool, ids, weight, cu_seqlens)
    C = x.shape[-1]
    w = weight.reshape(C, -1).contiguous()
    K = w.shape[1]
    _pool_view_check(state_pool, K - 1, C)
    x2, xs = _rows2d(x, C)
    N = x2.shape[0]
    ids = _ids64(ids)
    cu = cu_seqlens.to(torch.int32).contiguous() if cu_seqlens.dtype != torch.int32 \
        else cu_seqlens.contiguous()
    assert cu.numel() == ids.numel() + 1, "cu_seqlens must have n_seqs + 1 entries"
    _debug_checks(ids, state_pool.shape[0], cu, N)
    y = torch.empty(N, C, dtype=x.dtype, device=x.device)
    rc = _lib.load().gdn_causal_conv_silu_varlen(
        _p(x2), xs, _p(state_pool), _slot_stride(state_pool), state_pool.shape[0], _p(ids), _p(cu),
        ids.numel(), N, C, K, _p(w), _p(y), y.stride(0), _p(status_word(x.device)),
        _stream_ptr(x.device))
    _lib.check(rc, "gdn_causal_conv_silu_varlen")
    return y


def conv_gate_varlen(x: torch.Tensor, state_pool: torch.Tensor, ids: torch.Tensor,
                     weight: torch.Tensor, cu_seqlens: torch.Tensor, b: torch.Tensor,
                     a: torch.Tensor, a_log: torch.Tensor, dt_bias: torch.Tensor):
    """:func:`causal_conv_silu_varlen` and :func:`fused_g_beta` (no mask) of
    the same prefill rows in one call (qwen3_5.py:929-946): the gate runs as an
    extra row of the conv launch.  Bit-identical to the two calls.
    Returns (y [N, C], g fp32 [N, Vh], beta bf16 [N, Vh])."""
    _cuda(x, state_pool, ids, weight, cu_seqlens, b, a, a_log, dt_bias)
    C = x.shape[-1]
    w = weight.reshape(C, -1).contiguous()
    K = w.shape[1]
    _pool_view_check(state_pool, K - 1, C)
    x2, xs = _rows2d(x, C)
    N = x2.shape[0]
    ids = _ids64(ids)
    cu = cu_seqlens.to(torch.int32).contiguous() if cu_seqlens.dtype != torch.int32 \
        else cu_seqlens.contiguous()
    assert cu.numel() == ids.numel() + 1, "cu_seqlens must have n_seqs + 1 entries"
    _debug_checks(ids, state_pool.shape[0], cu, N)
    assert b.dtype == torch.bfloat16 and a.dtype == torch.bfloat16 and a.shape == b.shape
    vh = a.shape[-1]
    assert a.reshape(-1, vh).shape[0] == N, "b / a need one row per token"
    assert a_log.numel() == vh and dt_bias.numel() == vh and a_log.dtype == dt_bias.dtype
    if a.dim() != 2 or b.dim() != 2 or a.stride(0) != b.stride(0) or a.stride(1) != 1 \
            or b.stride(1) != 1:
        a = a.reshape(-1, vh).contiguous()
        b = b.reshape(-1, vh).contiguous()
    pdt = _lib.GDN_DTYPE_BF16 if a_log.dtype == torch.bfloat16 else _lib.GDN_DTYPE_F32
    if pdt == _lib.GDN_DTYPE_F32:
        a_log, dt_bias = a_log.float().contiguous(), dt_bias.float().contiguous()
    else:
        a_log, dt_bias = a_log.contiguous(), dt_bias.contiguous()
    y = torch.empty(N, C, dtype=x.dtype, device=x.device)
    g = torch.empty(N, vh, dtype=torch.float32, device=x.device)
    beta = torch.empty(N, vh, dtype=torch.bfloat16, device=x.device)
    rc = _lib.load().gdn_conv_gate_varlen(
        _p(x2), xs, _p(state_pool), _slot_stride(state_pool), state_pool.shape[0], _p(ids), _p(cu),
        ids.numel(), N, C, K, _p(w), _p(y), y.stride(0), _p(b), _p(a), a.stride(0), vh,
        _p(a_log), _p(dt_bias), pdt, _p(g), _p(beta), _p(status_word(x.device)),
        _stream_ptr(x.device))
    _lib.check(rc, "gdn_conv_gate_varlen")
    return y, g, beta


# ---------------------------------------------------------------------------
# (d) recurrent decode, (c) chunk prefill
# ---------------------------------------------------------------------------


def _heads(t: torch.Tensor, name: str):
    """[rows, (1,) H, D] view -> (rows, H, D, row_stride); heads dense."""
    if t.dim() == 4:
        assert t.shape[1] == 1, f"{name}: expected [bs, 1, H, D]"
        t = t[:, 0]
    assert t.dim() == 3, f"{name}: expected [rows, H, D]"
    rows, H, D = t.shape
    assert t.stride(2) == 1 and (H == 1 or t.stride(1) == D), \
        f"{name}: heads must be dense within a row (stride(2) == {D})"
    return rows, H, D, t.stride(0)


def _state_view_check(s_pool: torch.Tensor, HV: int, DK: int, DV: int):
    assert s_pool.dim() == 4 and tuple(s_pool.shape[1:]) == (HV, DK, DV), \
        f"state pool view must be [slots, {HV}, {DK}, {DV}]"
    assert s_pool.dtype == torch.float32
    assert s_pool.stride(1) == DK * DV and s_pool.stride(2) == DV and s_pool.stride(3) == 1


def _norm_args(z, norm_weight, rows, HV, DV):
    """(z pointer, z row stride, weight pointer) of the optional fused
    gated-RMSNorm epilogue; z is [rows, HV, DV] (token stride may exceed
    HV*DV, heads dense) or None."""
    if z is None:
        return None, 0, None
    assert norm_weight is not None and norm_weight.dtype == torch.bfloat16
    assert norm_weight.numel() == DV
    z3 = z.reshape(rows, HV, DV) if z.is_contiguous() else z
    assert z3.dim() == 3 and tuple(z3.shape) == (rows, HV, DV) and z3.dtype == torch.bfloat16
    assert z3.stride(2) == 1 and (HV == 1 or z3.stride(1) == DV), "z heads must be dense"
    return z3, z3.stride(0), norm_weight.contiguous()


def recurrent_gdn_inplace(q, k, v, g, beta, s_pool, ids, z=None, norm_weight=None,
                          eps: float = 1e-6) -> torch.Tensor:
    """qwen3_5.py:596-613.  q/k [bs, 1, HK, DK] (or HK == HV, already
    repeated), v [bs, 1, HV, DV] — strided row views allowed; g fp32 /
    beta bf16 [bs, 1, HV]; s_pool [slots, HV, DK, DV] fp32 per-layer view,
    rows ``ids`` updated in place.  Returns out [bs, 1, HV, DV] bf16.
    With ``z`` ([bs, HV, DV]) and ``norm_weight`` the output is the gated
    RMSNorm of the core output (Qwen3_5RMSNormGated, qwen3_5.py:697-709),
    fused into the kernel's epilogue."""
    _cuda(q, k, v, g, beta, s_pool, ids)
    bs, HK, DK, qs = _heads(q, "q")
    bs_k, HK_k, DK_k, ks = _heads(k, "k")
    bs_v, HV, DV, vs = _heads(v, "v")
    assert bs_k == bs and bs_v == bs and HK_k == HK and DK_k == DK
    assert HV % HK == 0
    g = g.reshape(bs, HV)
    beta = beta.reshape(bs, HV)
    assert g.dtype == torch.float32 and g.is_contiguous() and beta.is_contiguous(), \
        "g / beta must be contiguous"
    _state_view_check(s_pool, HV, DK, DV)
    ids = _ids64(ids)
    assert ids.numel() == bs
    _debug_checks(ids, s_pool.shape[0])
    z3, zs, nw = _norm_args(z, norm_weight, bs, HV, DV)
    out = torch.empty(bs, 1, HV, DV, dtype=v.dtype, device=v.device)
    rc = _lib.load().gdn_recurrent_inplace(
        _p(q), qs, _p(k), ks, _p(v), vs, _p(g), _p(beta), _p(s_pool), _slot_stride(s_pool),
        s_pool.shape[0], _p(ids), _p(out), bs, HK, HV, DK, DV, DK ** -0.5, _p(z3), zs, _p(nw),
        float(eps), _p(status_word(v.device)), _stream_ptr(v.device))
    _lib.check(rc, "gdn_recurrent_inplace")
    return out


def chunk_prefill_workspace_bytes(n_tokens: int, n_seqs: int, HV: int, DK: int, DV: int) -> int:
    """Device scratch the split chunk prefill needs (0: the shape has no split form)."""
    return int(_lib.load().gdn_chunk_prefill_workspace_bytes(n_tokens, n_seqs, HV, DK, DV))


_CHUNK_WS: dict[tuple, torch.Tensor] = {}


def chunk_workspace(device, nbytes: int) -> torch.Tensor:
    """The split chunk prefill's scratch for the current stream of ``device``:
    at least ``nbytes``, kept between calls and grown when a larger prefill
    arrives (a multi-GB request per call can make the caching allocator go to
    cudaMalloc next to a large resident pool).  One buffer per stream, so calls
    on different streams never share it; a call uses it only in stream order."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, torch.cuda.current_stream(idx).cuda_stream)
    t = _CHUNK_WS.get(key)
    if t is None or t.numel() < nbytes:
        _CHUNK_WS.pop(key, None)
        t = None
        with torch.inference_mode(False):
            t = torch.empty(nbytes, dtype=torch.uint8, device=torch.device("cuda", idx))
        _CHUNK_WS[key] = t
    return t


def chunk_gated_delta_rule_varlen(q, k, v, g, beta, s_pool, ids, cu_seqlens,
                                  max_seqlen: int, z=None, norm_weight=None,
                                  eps: float = 1e-6, out=None,
                                  split: bool = True) -> torch.Tensor:
    """Varlen chunked prefill (the chunk rule of qwen3_5.py:140-227 driven by
    cu_seqlens as at :956-961), initial state read from and final state
    written to ``s_pool[ids[r]]``.  q/k [N, HK, DK], v [N, HV, DV] (row
    views allowed), g fp32 / beta bf16 [N, HV].  Returns out [N, HV, DV]; with ``z`` /
    ``norm_weight`` the gated RMSNorm is fused as in
    :func:`recurrent_gdn_inplace`.  ``split`` (head dim 128) runs the split
    form with the per-stream workspace of :func:`chunk_workspace` (the
    reference allocates its chunk intermediates per call); False runs the
    one-kernel form (same bits, no workspace)."""
    _cuda(q, k, v, g, beta, s_pool, ids, cu_seqlens)
    N, HK, DK, qs = _heads(q, "q")
    N_k, HK_k, DK_k, ks = _heads(k, "k")
    N_v, HV, DV, vs = _heads(v, "v")
    assert N_k == N and N_v == N and HK_k == HK and DK_k == DK and HV % HK == 0
    g = g.reshape(N, HV)
    beta = beta.reshape(N, HV)
    assert g.dtype == torch.float32 and g.is_contiguous() and beta.is_contiguous()
    _state_view_check(s_pool, HV, DK, DV)
    ids = _ids64(ids)
    cu = cu_seqlens.to(torch.int32).contiguous() if cu_seqlens.dtype != torch.int32 \
        else cu_seqlens.contiguous()
    assert cu.numel() == ids.numel() + 1
    _debug_checks(ids, s_pool.shape[0], cu, N, int(max_seqlen))
    z3, zs, nw = _norm_args(z, norm_weight, N, HV, DV)
    out = _out_buffer(out, (N, HV, DV), v.device)
    ws_bytes = chunk_prefill_workspace_bytes(N, ids.numel(), HV, DK, DV) if split else 0
    ws = chunk_workspace(v.device, ws_bytes) if ws_bytes else None
    ws_bytes = ws.numel() if ws is not None else 0
    rc = _lib.load().gdn_chunk_prefill_varlen(
        _p(q), qs, _p(k), ks, _p(v), vs, _p(g), _p(beta), _p(s_pool), _slot_stride(s_pool),
        s_pool.shape[0], _p(ids), _p(cu), ids.numel(), N, int(max_seqlen), _p(out), HK, HV, DK,
        DV, DK ** -0.5, _p(z3), zs, _p(nw), float(eps), _p(ws), ws_bytes,
        _p(status_word(v.device)), _stream_ptr(v.device))
    _lib.check(rc, "gdn_chunk_prefill_varlen")
    return out


def rms_norm_gated(x: torch.Tensor, gate: torch.Tensor, weight: torch.Tensor,
                   eps: float) -> torch.Tensor:
    """qwen3_5.py:121-131 (Qwen3_5RMSNormGated.forward).  x [.., D] bf16,
    gate with x's shape; for a [tokens, heads, D] gate the token stride may
    exceed heads*D (a column slice of a fused projection).  weight [D].
    Returns y with x's shape."""
    _cuda(x, gate, weight)
    D = x.shape[-1]
    assert x.dtype == torch.bfloat16 and gate.dtype == torch.bfloat16 and \
        weight.dtype == torch.bfloat16
    assert gate.shape == x.shape
    x = x.contiguous()
    n = x.numel() // D
    if gate.dim() == 3 and gate.stride(2) == 1 and (gate.shape[1] == 1 or gate.stride(1) == D):
        g3 = gate
    else:
        g3 = gate.reshape(-1, 1, D).contiguous() if gate.dim() != 3 else gate.contiguous()
    heads = g3.shape[1]
    y = torch.empty_like(x)
    rc = _lib.load().gdn_rms_norm_gated(
        _p(x), _p(g3), g3.stride(0), heads, _p(weight.contiguous()), _p(y), n, D, float(eps),
        _stream_ptr(x.device))
    _lib.check(rc, "gdn_rms_norm_gated")
    return y


# ---------------------------------------------------------------------------
# the fused decode core (conv step + gate + recurrence + gated norm)
# ---------------------------------------------------------------------------


def decode_fused_supported(num_k_heads: int, num_v_heads: int, head_k_dim: int,
                           head_v_dim: int, conv_kernel: int) -> bool:
    """Whether :func:`decode_fused` serves this layer shape."""
    return (head_k_dim == head_v_dim and head_k_dim in (64, 128) and
            num_v_heads % num_k_heads == 0 and num_v_heads // num_k_heads <= 4 and
            2 <= conv_kernel <= 4)


_COUNTERS: dict[int, torch.Tensor] = {}
_RETIRED_COUNTERS: list[torch.Tensor] = []


def group_counters(device, n: int) -> torch.Tensor:
    """The per-device int32 scratch of decode_fused's group counters (at least
    n entries; all zero between calls — the kernel leaves them zero).  Made
    outside inference mode so it is a normal tensor, 65536 entries (256 KiB)
    at first so it practically never grows; a buffer that is outgrown stays
    allocated, because CUDA graphs captured earlier keep its address.  One
    buffer per device serves every stream (a graph captured on a side stream
    reuses the buffer of the eager warm-up calls), so decode_fused calls on
    one device must not run concurrently on different streams: their
    counters would mix."""
    device = torch.device(device)
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _COUNTERS.get(idx)
    if t is None or t.numel() < n:
        if t is not None:
            _RETIRED_COUNTERS.append(t)
        with torch.inference_mode(False):
            t = torch.zeros(max(n, 1 << 16), dtype=torch.int32,
                            device=torch.device("cuda", idx))
        _COUNTERS[idx] = t
    return t


def decode_fused(mixed: torch.Tensor, z: torch.Tensor, b: torch.Tensor, a: torch.Tensor,
                 conv_pool: torch.Tensor, conv_weight: torch.Tensor, a_log: torch.Tensor,
                 dt_bias: torch.Tensor, s_pool: torch.Tensor, ids: torch.Tensor,
                 norm_weight: torch.Tensor, eps: float = 1e-6,
                 counters: bool = True, out=None) -> torch.Tensor:
    """The decode branch of Qwen3_5GatedDeltaNet.forward for T == 1 rows in one
    kernel: conv_decode_step (qwen3_5.py:1008-1012) + fused_g_beta (:976-982)
    + recurrent_gdn_inplace (:1013-1026) + the gated norm (:1083-1085).
    mixed [bs, conv_dim] (the [q | k | v] columns of the projection, rows may
    be strided), z [bs, HV, D] (token stride may exceed HV*D), b / a [bs, HV]
    (shared row stride); conv_pool [slots, conv_dim, K-1] and s_pool [slots,
    HV, D, D] per-layer views rolled / updated in place at rows ``ids``.
    Returns the normed core output [bs, HV, D] (bit-identical to the
    four-operator sequence).  ``counters`` passes this device's group-counter
    scratch (:func:`group_counters`), which lets batches that fit one wave of
    the GPU run the low-latency head-per-CTA kernel; False always runs the
    persistent kernel, which needs no scratch."""
    _cuda(mixed, z, b, a, conv_pool, conv_weight, a_log, dt_bias, s_pool, ids, norm_weight)
    bs = mixed.shape[0]
    HV, DK, DV = s_pool.shape[1], s_pool.shape[2], s_pool.shape[3]
    D = DV
    C = mixed.shape[-1]
    assert DK == DV, "decode_fused needs head_k_dim == head_v_dim"
    assert (C // D - HV) % 2 == 0 and C % D == 0, "mixed must hold [q | k | v] of whole heads"
    HK = (C // D - HV) // 2
    w = conv_weight.reshape(C, -1).contiguous()
    K = w.shape[1]
    _pool_view_check(conv_pool, K - 1, C)
    _state_view_check(s_pool, HV, D, D)
    assert mixed.dtype == torch.bfloat16 and w.dtype == torch.bfloat16
    m2, ms = _rows2d(mixed, C)
    assert m2.shape[0] == bs
    z3, zs, nw = _norm_args(z, norm_weight, bs, HV, D)
    assert b.shape == (bs, HV) and a.shape == (bs, HV) and b.stride(1) == 1 and \
        a.stride(1) == 1 and a.stride(0) == b.stride(0), "b / a must share a row stride"
    assert b.dtype == torch.bfloat16 and a.dtype == torch.bfloat16
    assert a_log.dtype == dt_bias.dtype and a_log.dtype in (torch.float32, torch.bfloat16)
    assert a_log.numel() == HV and dt_bias.numel() == HV
    pdt = _lib.GDN_DTYPE_F32 if a_log.dtype == torch.float32 else _lib.GDN_DTYPE_BF16
    ids = _ids64(ids)
    assert ids.numel() == bs
    assert conv_pool.shape[0] == s_pool.shape[0], "both pools index the same slots"
    _debug_checks(ids, s_pool.shape[0])
    out = _out_buffer(out, (bs, HV, D), mixed.device)
    cnt = group_counters(mixed.device, bs * HK) if counters else None
    rc = _lib.load().gdn_decode_fused(
        _p(m2), ms, _p(z3), zs, _p(b), _p(a), b.stride(0), _p(conv_pool), _slot_stride(conv_pool),
        _p(w), K, _p(a_log.contiguous()), _p(dt_bias.contiguous()), pdt, _p(s_pool),
        _slot_stride(s_pool), s_pool.shape[0], _p(ids), _p(nw), float(eps), _p(out), bs, HK, HV,
        D, D ** -0.5, _p(cnt), _p(status_word(mixed.device)), _stream_ptr(mixed.device))
    _lib.check(rc, "gdn_decode_fused")
    return out
