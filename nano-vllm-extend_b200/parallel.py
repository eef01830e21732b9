"""Tensor / pipeline parallel plumbing for the GDN layer path.

Mirrors the reference's parallel state (nanovllm/utils/parallel.py) — rank
layout ``rank = pp_rank * tp_size + tp_rank``, one TP group per pipeline
stage — and its column / row parallel linear layers (nanovllm/layers/
linear.py), and adds the two multi-GPU pieces of the GDN path:

* V-head sharding (qwen3_5.py:796-835, 840-851): rank r of a TP group owns
  the contiguous v-head block [r*HV/G, (r+1)*HV/G) and the matching k-head
  block, so h_k = h_v // (HV/HK) stays local; conv channels and the
  recurrent state shard with them and the core needs no exchange.  The only
  collective is out_proj's partial-sum all-reduce.
* The pipeline stage handoff (engine/model_runner.py:795-810): the
  reference sends ``hidden`` and ``residual`` as two blocking messages on the
  compute stream.  :class:`PipelineHandoff` packs them into one buffer and
  moves it with NCCL point-to-point on a dedicated communication stream,
  ordered against compute with CUDA events, so the transfer overlaps
  whatever the stage does next; a ``presum`` mode sends the single tensor
  bf16(hidden + residual) that the next stage's input RMSNorm computes first.
"""
from __future__ import annotations

from datetime import timedelta

import torch
import torch.distributed as dist
import torch.nn.functional as F
from torch import nn

# ---------------------------------------------------------------------------
# parallel state (utils/parallel.py:17-106)
# ---------------------------------------------------------------------------

_rank = 0
_world_size = 1
_tp_rank = 0
_tp_size = 1
_pp_rank = 0
_pp_size = 1
_tp_group = None
_initialized = False


def init_parallel_state(rank: int, world_size: int, tp_size: int, pp_size: int):
    """Record this process's coordinates and create the per-stage TP groups.
    Collective over the default group when world_size > 1 (new_group)."""
    global _rank, _world_size, _tp_rank, _tp_size, _pp_rank, _pp_size, _tp_group, _initialized
    assert world_size == tp_size * pp_size
    _rank, _world_size, _tp_size, _pp_size = rank, world_size, tp_size, pp_size
    _pp_rank, _tp_rank = rank // tp_size, rank % tp_size
    _tp_group = None
    for pp in range(pp_size):
        ranks = list(range(pp * tp_size, (pp + 1) * tp_size))
        group = dist.new_group(ranks, timeout=make_process_group_timeout()) \
            if world_size > 1 else None
        if pp == _pp_rank:
            _tp_group = group
    _initialized = True


def reset_parallel_state():
    global _rank, _world_size, _tp_rank, _tp_size, _pp_rank, _pp_size, _tp_group, _initialized
    _rank, _world_size, _tp_rank, _tp_size, _pp_rank, _pp_size = 0, 1, 0, 1, 0, 1
    _tp_group, _initialized = None, False


def get_rank() -> int: return _rank
def get_world_size() -> int: return _world_size
def get_tp_rank() -> int: return _tp_rank
def get_tp_size() -> int: return _tp_size
def get_tp_group(): return _tp_group
def get_pp_rank() -> int: return _pp_rank
def get_pp_size() -> int: return _pp_size
def is_first_pp_stage() -> bool: return _pp_rank == 0
def is_last_pp_stage() -> bool: return _pp_rank == _pp_size - 1


def pp_peers(rank: int, tp_size: int, pp_size: int) -> tuple[int | None, int | None]:
    """Previous / next stage peers of ``rank`` (same tp rank), as
    engine/model_runner.py:44-47 computes them; None at the ends."""
    pp, tp = rank // tp_size, rank % tp_size
    prev = (pp - 1) * tp_size + tp if pp > 0 else None
    nxt = (pp + 1) * tp_size + tp if pp < pp_size - 1 else None
    return prev, nxt


def split_layers(num_layers: int, pp_size: int, pp_rank: int) -> tuple[int, int]:
    """Contiguous layer range of one stage: ceil(L / P) layers per stage
    (models/qwen3.py:24-28)."""
    per = (num_layers + pp_size - 1) // pp_size
    start = pp_rank * per
    return start, min(num_layers, start + per)


# ---------------------------------------------------------------------------
# V-head sharding
# ---------------------------------------------------------------------------


def head_shard(total_v_heads: int, total_k_heads: int, tp_size: int, tp_rank: int):
    """(v-head slice, k-head slice) owned by ``tp_rank`` (qwen3_5.py:796-801,
    831-832).  Requires both head counts divisible by tp_size
    (config.py:86-89)."""
    assert total_v_heads % total_k_heads == 0
    assert total_k_heads % tp_size == 0 and total_v_heads % tp_size == 0, \
        "head counts must be divisible by the tensor-parallel size"
    hv, hk = total_v_heads // tp_size, total_k_heads // tp_size
    return slice(tp_rank * hv, (tp_rank + 1) * hv), slice(tp_rank * hk, (tp_rank + 1) * hk)


def conv_layout_shard(loaded: torch.Tensor, key_dim_total: int, value_dim_total: int,
                      tp_size: int, tp_rank: int) -> torch.Tensor:
    """Shard a [q | k | v] stacked dim-0 tensor (in_proj_qkv.weight or
    conv1d.weight) part by part at head granularity — the rule of
    _conv_layout_loader (qwen3_5.py:840-851)."""
    q, k, v = loaded.split([key_dim_total, key_dim_total, value_dim_total], dim=0)
    return torch.cat([t.chunk(tp_size, dim=0)[tp_rank] for t in (q, k, v)], dim=0)


# ---------------------------------------------------------------------------
# column / row parallel linear layers (layers/linear.py:56-158)
# ---------------------------------------------------------------------------


class ColumnParallelLinear(nn.Module):
    """y = x W^T with W sharded along the output dim (dim 0)."""

    def __init__(self, input_size: int, output_size: int, tp_rank: int = 0, tp_size: int = 1,
                 weight: torch.Tensor | None = None):
        super().__init__()
        assert output_size % tp_size == 0
        self.tp_rank, self.tp_size, self.tp_dim = tp_rank, tp_size, 0
        shape = (output_size // tp_size, input_size)
        if weight is None:
            weight = torch.empty(shape)
        assert tuple(weight.shape) == shape
        self.weight = nn.Parameter(weight, requires_grad=False)
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param: nn.Parameter, loaded: torch.Tensor):
        n = param.data.size(0)
        param.data.copy_(loaded.narrow(0, self.tp_rank * n, n))

    def forward(self, x):
        return F.linear(x, self.weight)


class RowParallelLinear(nn.Module):
    """y = all_reduce(x_shard W_shard^T) with W sharded along the input dim."""

    def __init__(self, input_size: int, output_size: int, tp_rank: int = 0, tp_size: int = 1,
                 tp_group=None):
        super().__init__()
        assert input_size % tp_size == 0
        self.tp_rank, self.tp_size, self.tp_dim, self.tp_group = tp_rank, tp_size, 1, tp_group
        self.weight = nn.Parameter(torch.empty(output_size, input_size // tp_size),
                                   requires_grad=False)
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param: nn.Parameter, loaded: torch.Tensor):
        if param.data.ndim == 1:
            param.data.copy_(loaded)
            return
        n = param.data.size(1)
        param.data.copy_(loaded.narrow(1, self.tp_rank * n, n))

    def forward(self, x):
        y = F.linear(x, self.weight)
        if self.tp_size > 1:
            dist.all_reduce(y, group=self.tp_group)
        return y


# ---------------------------------------------------------------------------
# pipeline stage handoff
# ---------------------------------------------------------------------------


class PipelineHandoff:
    """Stage-boundary transfer of the fused-residual chain (hidden, residual).

    The reference (engine/model_runner.py:795-810) issues two blocking
    ``dist.send`` / ``dist.recv`` per boundary on the compute stream.  Here
    one message per boundary carries both tensors (``mode="packed"``: a
    [2, N, H] buffer) or their sum (``mode="presum"``: bf16(hidden +
    residual), which the receiver feeds as hidden with residual=None — the
    receiving layer's add-RMSNorm computes exactly that sum first, so the
    result is bit-identical on the torch norm path and half the bytes cross
    NVLink).  On CUDA, sends and receives run on a dedicated stream: the
    sender records an event after the producing kernels and returns at once;
    the receiver's compute stream waits on an event recorded after the
    receive, never on the host.  Buffers are double-buffered so a step's send
    may still be in flight while the next step produces its outputs.
    """

    def __init__(self, hidden_size: int, max_tokens: int, dtype: torch.dtype,
                 device: torch.device, peer_prev: int | None, peer_next: int | None,
                 group=None, mode: str = "packed", recv_group=None, send_group=None):
        """``group`` carries both directions unless ``recv_group`` /
        ``send_group`` (e.g. a two-rank group per stage boundary, so one
        boundary's messages never queue behind another's) are given.  Peers
        are global ranks."""
        assert mode in ("packed", "presum")
        self.H, self.max_tokens, self.dtype, self.device = hidden_size, max_tokens, dtype, device
        self.prev, self.next, self.group, self.mode = peer_prev, peer_next, group, mode
        self.recv_group = recv_group if recv_group is not None else group
        self.send_group = send_group if send_group is not None else group
        self.parts = 2 if mode == "packed" else 1
        # flat buffers: a message of n tokens is the contiguous prefix viewed
        # as [parts, n, H], so each part is itself a contiguous [n, H] tensor
        self._send = [torch.empty(self.parts * max_tokens * hidden_size, dtype=dtype,
                                  device=device) for _ in range(2)]
        self._recv = [torch.empty(self.parts * max_tokens * hidden_size, dtype=dtype,
                                  device=device) for _ in range(2)]
        self._send_work = [None, None]
        self._slot = 0
        self._rslot = 0
        self._recv_free = [None, None]   # per receive buffer: its readers are done
        self._last_recv = None
        self.cuda = device.type == "cuda"
        self.stream = torch.cuda.Stream(device=device) if self.cuda else None

    def _wait_send(self, i):
        w = self._send_work[i]
        if w is not None:
            w.wait()
            self._send_work[i] = None

    def send(self, hidden: torch.Tensor, residual: torch.Tensor):
        """Queue (hidden, residual) [N, H] for the next stage; returns at once."""
        assert self.next is not None, "send() on the last pipeline stage"
        n = hidden.shape[0]
        assert n <= self.max_tokens
        i = self._slot
        self._slot ^= 1
        self._wait_send(i)   # the send that last used this buffer has completed
        buf = self._send[i][:self.parts * n * self.H].view(self.parts, n, self.H)
        if self.mode == "packed":
            buf[0].copy_(hidden)
            buf[1].copy_(residual)
        else:
            buf[0].copy_((hidden.float() + residual.float()).to(self.dtype))
        if self.cuda:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.stream):
                self.stream.wait_event(ev)
                self._send_work[i] = dist.isend(buf, self.next, group=self.send_group)
        else:
            self._send_work[i] = dist.isend(buf, self.next, group=self.send_group)

    def recv(self, n: int):
        """Receive the previous stage's message for ``n`` tokens; returns
        (hidden, residual) — residual is None in presum mode.  On CUDA the
        current stream is ordered after the receive (no host wait)."""
        assert self.prev is not None, "recv() on the first pipeline stage"
        assert n <= self.max_tokens
        i = self._rslot
        self._rslot ^= 1
        buf = self._recv[i][:self.parts * n * self.H].view(self.parts, n, self.H)
        if self.cuda:
            cur = torch.cuda.current_stream(self.device)
            ev0 = self._recv_free[i]
            if ev0 is None:          # no consumed() mark: wait for all the stream has queued
                ev0 = torch.cuda.Event()
                ev0.record(cur)
            self._recv_free[i] = None
            with torch.cuda.stream(self.stream):
                self.stream.wait_event(ev0)
                w = dist.irecv(buf, self.prev, group=self.recv_group)
                w.wait()             # orders the comm stream, not the host
                ev = torch.cuda.Event()
                ev.record(self.stream)
            cur.wait_event(ev)
        else:
            dist.irecv(buf, self.prev, group=self.recv_group).wait()
        self._last_recv = i
        if self.mode == "packed":
            return buf[0], buf[1]
        return buf[0], None

    def consumed(self):
        """Mark the tensors of the last recv() as read by the work queued so far
        on the current stream (e.g. after copying them into the stage's input).
        The next receive into that buffer then waits only for those reads, not
        for everything the stream queued later (the stage's own compute), so the
        transfer overlaps the compute.  Optional: without it a receive waits for
        all work queued before it."""
        if self.cuda and self._last_recv is not None:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self._recv_free[self._last_recv] = ev
        self._last_recv = None

    def flush(self):
        """Wait for every outstanding send (call before tearing down)."""
        for i in range(2):
            self._wait_send(i)


def boundary_groups(world_size: int):
    """One two-rank process group per pipeline boundary (stage b -> b + 1),
    created in the same order on every rank (new_group is collective over
    the default group).  Returns the list indexed by boundary."""
    return [dist.new_group([b, b + 1], timeout=make_process_group_timeout())
            for b in range(world_size - 1)]


def make_process_group_timeout(seconds: float = 60.0) -> timedelta:
    """Short default timeout for GDN process groups: ranks that wait on a
    peer that died end with an error instead of hanging."""
    return timedelta(seconds=seconds)
