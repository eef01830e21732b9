"""Drop-in Qwen3_5GatedDeltaNet backed by the sm_100a kernels.

Same constructor ``(config)``, same ``forward(positions, hidden_states)``,
same attributes and parameter names as the reference layer
(sileaver/nano-vllm-extend, nanovllm/models/qwen3_5.py:780-1087), so the
engine binds ``s_cache`` / ``conv_cache`` and loads checkpoints exactly as it
does for the reference class.  :func:`install` swaps the class inside an
imported reference package; ``model_runner.py`` and ``LLM.generate`` stay
unchanged.

What differs is the execution, B200-first:

* one GEMM for the four input projections: ``in_proj_qkv``, ``in_proj_z``,
  ``in_proj_b`` and ``in_proj_a`` are views into one fused weight buffer, so
  the layer issues a single cuBLAS call over all rows and the kernels read
  their operands as column views of its output (no splits, no copies);
* no padding: decode rows (length 1, which the scheduler puts first) go to
  the slot-indexed conv step + in-place recurrent kernels, the remaining
  rows to the varlen conv + chunked-prefill kernels driven by cu_seqlens;
* no gather / scatter of pool rows: every kernel reads and writes the state
  in its slot;
* no host synchronisation on the decode path, so the engine's CUDA-graph
  capture of decode steps works as before (pad rows use the dummy slot).
"""
from __future__ import annotations

import contextlib

import torch
import torch.nn.functional as F
from torch import nn

from . import context as _context
from . import ops
from . import parallel as _parallel
from .parallel import ColumnParallelLinear, RowParallelLinear, conv_layout_shard


class Qwen3_5RMSNormGated(nn.Module):
    """Delta-net output norm (qwen3_5.py:697-709): plain w*x RMSNorm over the
    value head dim, gated by silu(z); weight initialised to ones."""

    def __init__(self, hidden_size: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size), requires_grad=False)
        self.eps = eps

    def forward(self, hidden_states: torch.Tensor, gate: torch.Tensor) -> torch.Tensor:
        return ops.rms_norm_gated(hidden_states, gate, self.weight, self.eps)


class Qwen3_5GatedDeltaNet(nn.Module):
    """Linear-attention layer (gated delta net) over pooled recurrent state.

    ``parallel`` supplies get_tp_rank / get_tp_size / get_tp_group (this
    package's :mod:`parallel` by default, the engine's utils.parallel when
    installed); ``get_context`` returns the per-step Context.
    """

    # Decode rows through the one-launch fused core (ops.decode_fused) when the
    # shape allows; it is the faster route at every batch size measured on
    # B200 (bs 1..256).  False runs the four operators (identical results
    # wherever their recurrent kernel runs full tiles).
    fused_decode = True
    # Poll the kernels' device status word (its pinned host copy) before each
    # call and raise if a kernel flagged a fault (bad slot id, malformed
    # cu_seqlens, a wait that gave up); one layer per device, the first to run,
    # publishes the word after its kernels (one 4-byte asynchronous copy per
    # step).  See ops.poll_status for graph-replayed steps.
    report_status = True
    # Mark the layer's phases with NVTX ranges ("gdn.in_proj", "gdn.decode_core",
    # "gdn.conv_gate", "gdn.chunk", "gdn.out_proj") for nsys-style
    # timelines; off by default (a range costs a host call per phase).
    nvtx = False

    def __init__(self, config, parallel=None, get_context=None) -> None:
        super().__init__()
        P = parallel if parallel is not None else _parallel
        self._get_context = get_context if get_context is not None else _context.get_context
        tp_size, tp_rank = P.get_tp_size(), P.get_tp_rank()
        self.hidden_size = config.hidden_size
        self.total_num_k_heads = config.linear_num_key_heads
        self.total_num_v_heads = config.linear_num_value_heads
        assert self.total_num_v_heads % self.total_num_k_heads == 0, \
            "qwen3_5: v/k head replication must be integral"
        assert self.total_num_k_heads % tp_size == 0
        assert self.total_num_v_heads % tp_size == 0
        self.num_k_heads = self.total_num_k_heads // tp_size
        self.num_v_heads = self.total_num_v_heads // tp_size
        self.head_k_dim = config.linear_key_head_dim
        self.head_v_dim = config.linear_value_head_dim
        self.key_dim = self.head_k_dim * self.num_k_heads
        self.value_dim = self.head_v_dim * self.num_v_heads
        self.conv_kernel = config.linear_conv_kernel_dim
        self.conv_dim = self.key_dim * 2 + self.value_dim
        self._total_conv_dim = (self.head_k_dim * self.total_num_k_heads * 2
                                + self.head_v_dim * self.total_num_v_heads)
        self._tp_rank, self._tp_size = tp_rank, tp_size

        # Fused input-projection weight: rows [qkv | z | b | a | pad] of this
        # rank's shard; the four projection modules own views of it.
        cd, vd, hv = self.conv_dim, self.value_dim, self.num_v_heads
        self._proj_rows = (cd, cd + vd, cd + vd + hv, cd + vd + 2 * hv)
        total = (self._proj_rows[-1] + 7) // 8 * 8   # 16-byte aligned output rows
        fused = torch.zeros(total, self.hidden_size)
        r = self._proj_rows
        self.in_proj_qkv = ColumnParallelLinear(self.hidden_size, self._total_conv_dim, tp_rank,
                                                tp_size, weight=fused[:r[0]])
        self.in_proj_qkv.weight.weight_loader = self._conv_layout_loader
        self.in_proj_z = ColumnParallelLinear(self.hidden_size, vd * tp_size, tp_rank, tp_size,
                                              weight=fused[r[0]:r[1]])
        self.in_proj_b = ColumnParallelLinear(self.hidden_size, hv * tp_size, tp_rank, tp_size,
                                              weight=fused[r[1]:r[2]])
        self.in_proj_a = ColumnParallelLinear(self.hidden_size, hv * tp_size, tp_rank, tp_size,
                                              weight=fused[r[2]:r[3]])
        self._fused_w = fused
        self.conv1d = nn.Conv1d(self.conv_dim, self.conv_dim, self.conv_kernel,
                                groups=self.conv_dim, padding=0, bias=False)
        self.conv1d.weight.requires_grad_(False)
        self.conv1d.weight.weight_loader = self._conv_layout_loader
        A = torch.empty(self.total_num_v_heads).uniform_(0, 16)
        self.A_log = nn.Parameter(torch.log(A), requires_grad=False)   # full; sliced per rank
        self.dt_bias = nn.Parameter(torch.ones(self.total_num_v_heads), requires_grad=False)
        self._v_head_slice = slice(tp_rank * self.num_v_heads, (tp_rank + 1) * self.num_v_heads)
        self.norm = Qwen3_5RMSNormGated(self.head_v_dim, eps=config.rms_norm_eps)
        self.out_proj = RowParallelLinear(self.head_v_dim * self.total_num_v_heads,
                                          self.hidden_size, tp_rank, tp_size, P.get_tp_group())
        self.s_cache: torch.Tensor | None = None      # [slots, HV, DK, DV] fp32 view
        self.conv_cache: torch.Tensor | None = None   # [slots, conv_dim, K-1] view

    # -- weight loading -----------------------------------------------------

    def _conv_layout_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor):
        """Shard the [q | k | v] stacked dim at head granularity
        (qwen3_5.py:840-851)."""
        kd = self.head_k_dim * self.total_num_k_heads
        vd = self.head_v_dim * self.total_num_v_heads
        param.data.copy_(conv_layout_shard(loaded_weight, kd, vd, self._tp_size, self._tp_rank))

    def _fused_weight(self) -> torch.Tensor:
        """The fused projection weight; rebuilt (once) if the projection
        parameters stopped aliasing it, e.g. after ``module.to(...)``."""
        ws = (self.in_proj_qkv.weight, self.in_proj_z.weight, self.in_proj_b.weight,
              self.in_proj_a.weight)
        Fw = self._fused_w
        starts = (0,) + self._proj_rows[:-1]
        ok = (Fw.device == ws[0].device and Fw.dtype == ws[0].dtype and
              all(w.data_ptr() == Fw[s].data_ptr() for w, s in zip(ws, starts)))
        if ok:
            return Fw
        Fw = torch.zeros(Fw.shape[0], self.hidden_size, dtype=ws[0].dtype, device=ws[0].device)
        for w, s, e in zip(ws, starts, self._proj_rows):
            Fw[s:e].copy_(w.data)
            w.data = Fw[s:e]
        self._fused_w = Fw
        return Fw

    # -- forward --------------------------------------------------------------

    def _range(self, name: str):
        return torch.cuda.nvtx.range(name) if self.nvtx else contextlib.nullcontext()

    def forward(self, positions: torch.Tensor, hidden_states: torch.Tensor) -> torch.Tensor:
        """hidden_states [N, hidden] (varlen concatenation, decode rows
        first) -> [N, hidden]; slot states updated in place."""
        assert self.s_cache is not None and self.conv_cache is not None, \
            "state pools not bound (s_cache / conv_cache)"
        assert hidden_states.dtype == torch.bfloat16, "the GDN kernels take bf16 activations"
        if self.report_status:
            ops.poll_status(hidden_states.device)      # faults of earlier calls raise here
        ctx = self._get_context()
        ids = ctx.linear_state_ids
        N = hidden_states.shape[0]
        cd, vd, hv = self.conv_dim, self.value_dim, self.num_v_heads
        r = self._proj_rows

        with self._range("gdn.in_proj"):
            proj = F.linear(hidden_states, self._fused_weight())    # [N, total]
        mixed = proj[:, :cd]
        z = proj[:, r[0]:r[1]].view(N, hv, self.head_v_dim)
        b = proj[:, r[1]:r[2]]
        a = proj[:, r[2]:r[3]]

        T = int(ctx.max_seqlen_q)
        if T == 1:
            n1 = N
            lens_q = None
        else:
            cu_q = ctx.cu_seqlens_q
            lens_q = ctx.lens_q if ctx.lens_q is not None else (cu_q[1:] - cu_q[:-1]).tolist()
            n1 = 0
            while n1 < len(lens_q) and lens_q[n1] == 1:
                n1 += 1
        # the gated RMSNorm (self.norm) runs fused in each core's kernels; decode and
        # prefill rows write their halves of one output buffer (no concatenation)
        core = torch.empty(N, hv, self.head_v_dim, dtype=torch.bfloat16,
                           device=hidden_states.device)
        if n1:
            with self._range("gdn.decode_core"):
                self._decode_core(mixed[:n1], z[:n1], b[:n1], a[:n1], ids[:n1], out=core[:n1])
        if n1 < N:
            cu_q = ctx.cu_seqlens_q
            cu_p = cu_q[n1:] - cu_q[n1] if n1 else cu_q
            self._prefill_core(mixed[n1:], b[n1:], a[n1:], ids[n1:], cu_p, max(lens_q[n1:]),
                               z[n1:], out=core[n1:])
        if self.report_status and ops.is_status_publisher(self, hidden_states.device):
            ops.publish_status(hidden_states.device)
        with self._range("gdn.out_proj"):
            return self.out_proj(core.view(N, vd))

    def _split(self, y: torch.Tensor):
        kd = self.key_dim
        n = y.shape[0]
        q = y[:, :kd].view(n, self.num_k_heads, self.head_k_dim)
        k = y[:, kd:2 * kd].view(n, self.num_k_heads, self.head_k_dim)
        v = y[:, 2 * kd:].view(n, self.num_v_heads, self.head_v_dim)
        return q, k, v

    def _decode_core(self, mixed, z, b, a, ids, out=None):
        """T == 1 rows: conv step + gate + in-place recurrent + gated norm
        (qwen3_5.py:976-982, 1008-1026, 1083-1085), one fused kernel when the
        shape allows (``fused_decode``), else the four operators."""
        a_log = self.A_log[self._v_head_slice]
        dt_bias = self.dt_bias[self._v_head_slice]
        w = self.conv1d.weight.view(self.conv_dim, self.conv_kernel)
        if self.fused_decode and ops.decode_fused_supported(self.num_k_heads, self.num_v_heads,
                                              self.head_k_dim, self.head_v_dim, self.conv_kernel):
            return ops.decode_fused(mixed, z, b, a, self.conv_cache, w, a_log, dt_bias,
                                    self.s_cache, ids, self.norm.weight, self.norm.eps, out=out)
        g, beta = ops.fused_g_beta(b, a, a_log, dt_bias, None)
        y = ops.conv_decode_step(mixed, self.conv_cache, ids, w)
        q, k, v = self._split(y)
        o = ops.recurrent_gdn_inplace(q, k, v, g, beta, self.s_cache, ids, z=z,
                                      norm_weight=self.norm.weight, eps=self.norm.eps)
        o = o.view(-1, self.num_v_heads, self.head_v_dim)
        if out is not None:
            out.copy_(o)
            return out
        return o

    def _prefill_core(self, mixed, b, a, ids, cu_seqlens, max_seqlen, z, out=None):
        """Prefill rows: varlen conv and g / beta gate (one call) + chunked rule
        with slot states + gated norm (the composition of qwen3_5.py:922-963,
        unpadded)."""
        with self._range("gdn.conv_gate"):
            y, g, beta = ops.conv_gate_varlen(
                mixed, self.conv_cache, ids,
                self.conv1d.weight.view(self.conv_dim, self.conv_kernel), cu_seqlens, b, a,
                self.A_log[self._v_head_slice], self.dt_bias[self._v_head_slice])
        q, k, v = self._split(y)
        with self._range("gdn.chunk"):
            return ops.chunk_gated_delta_rule_varlen(
                q, k, v, g, beta, self.s_cache, ids, cu_seqlens, max_seqlen, z=z,
                norm_weight=self.norm.weight, eps=self.norm.eps, out=out)


def install(qwen3_5_module=None, parallel_module=None, context_module=None):
    """Swap the reference's GDN layer class for this one.

    Call after importing the reference package and before the model is
    built (ModelRunner constructs Qwen3_5ForCausalLM, whose decoder layers
    look the class up by its module-global name).  The installed subclass
    reads the engine's own parallel state and per-step context.  Returns
    the class that was replaced (pass it to :func:`uninstall`)."""
    if qwen3_5_module is None:
        import nanovllm.models.qwen3_5 as qwen3_5_module  # noqa: PLC0415
    if parallel_module is None:
        import nanovllm.utils.parallel as parallel_module  # noqa: PLC0415
    if context_module is None:
        import nanovllm.utils.context as context_module  # noqa: PLC0415
    P, Cx = parallel_module, context_module

    class Qwen3_5GatedDeltaNetB200(Qwen3_5GatedDeltaNet):
        def __init__(self, config):
            super().__init__(config, parallel=P, get_context=Cx.get_context)

    previous = qwen3_5_module.Qwen3_5GatedDeltaNet
    qwen3_5_module.Qwen3_5GatedDeltaNet = Qwen3_5GatedDeltaNetB200
    return previous


def uninstall(previous, qwen3_5_module=None):
    if qwen3_5_module is None:
        import nanovllm.models.qwen3_5 as qwen3_5_module  # noqa: PLC0415
    qwen3_5_module.Qwen3_5GatedDeltaNet = previous
