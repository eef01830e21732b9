"""GDN layer-path benchmark (one JSON line on rank 0).

Headline workload (config 1): a Qwen3.5-2B-shaped GatedDeltaNet decode
stack — 18 GDN layers (hidden 2048, 16 QK heads x 128, 32 V heads x 128,
conv kernel 4), batch 256, one token per sequence, bf16 activations and
fp32 recurrent states in a 1024-slot pool (+ dummy slot) addressed by a
seeded random permutation of slot ids.  A step runs every layer's forward
(fused input projection, conv step, gate, in-place recurrent, gated norm,
out projection) with a residual add between layers, captured once in a
CUDA graph as the engine captures decode.  The state pool (38.7 GB) is far
larger than L2, so no flush is needed between steps.

  value     tokens/s with the step input already in HBM
  e2e       same metric through the public layer API with the step input
            copied from pinned host memory and the step output copied back
            inside the timed region
  roofline  the dominant kernel (in-place recurrent decode), HBM-bound:
            algorithmic bytes per launch / CUDA-event launch duration
  prefill   secondary: config-2 varlen chunked prefill of one layer

``--impl reference`` times the CPU restatement of the reference path on the
host cores instead (the reference itself is Python that does not travel).
Multi-GPU (torchrun, one process per GPU): every rank decodes its own 256
sequences against its own pool (weak scaling, no data-path collective);
times are the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

C1 = dict(layers=18, bs=256, hidden=2048, HK=16, DK=128, HV=32, DV=128, K=4, slots=1024,
          eps=1e-6)
C2 = dict(n_seqs=64, len_lo=128, len_hi=8192, hidden=2048, HK=16, DK=128, HV=32, DV=128, K=4)
CHUNK_FLOPS_PER_TOKEN_HEAD = 180_224   # 4C*Dk + 2C*Dk + 4C*Dv + 6*Dk*Dv at C=64, Dk=Dv=128


class OneRank:
    """Parallel state of an unsharded layer (tp size 1), passed explicitly to
    every layer that must not pick up the package's process-wide TP state."""
    get_tp_rank = staticmethod(lambda: 0)
    get_tp_size = staticmethod(lambda: 1)
    get_tp_group = staticmethod(lambda: None)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-config4", action="store_true")
    ap.add_argument("--prefill-steps", type=int, default=3)
    ap.add_argument("--profile-case", default=None,
                    choices=["recurrent", "decode_fused", "conv_decode", "conv_varlen", "chunk",
                             "chunk_long", "gbeta", "norm"],
                    help="run a small single-kernel case for ncu (3 launches) and exit")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# distributed helpers
# ---------------------------------------------------------------------------


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    return world, rank, local


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------


class Clocks:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        fd, self.path = tempfile.mkstemp(prefix="gdn_clocks_", suffix=".csv")
        os.close(fd)

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "20"], stdout=self.f,
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.f.close()
        rows = []
        for line in open(self.path):
            p = [x.strip() for x in line.split(",")]
            if len(p) >= 8:
                rows.append(p)
        try:
            os.remove(self.path)
        except OSError:
            pass
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = max(float(r[2]) for r in rows if r[2].replace(".", "").isdigit())
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i] == "Active"})
        load = [s for s in sm if s > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(load), "sm_max_mhz": smax, "reasons": reasons,
                "samples": len(rows)}


# ---------------------------------------------------------------------------
# config-1 decode stack
# ---------------------------------------------------------------------------


class DecodeStack:
    def __init__(self, pkg, device, seed, layers=None):
        self.pkg, self.dev = pkg, device
        c = C1
        n_layers = c["layers"] if layers is None else layers
        cfg = type("Cfg", (), dict(hidden_size=c["hidden"], linear_num_key_heads=c["HK"],
                                   linear_num_value_heads=c["HV"], linear_key_head_dim=c["DK"],
                                   linear_value_head_dim=c["DV"], linear_conv_kernel_dim=c["K"],
                                   rms_norm_eps=c["eps"]))
        g = torch.Generator(device=device).manual_seed(seed)
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            with torch.device(device), torch.no_grad():
                self.layers = [pkg.layer.Qwen3_5GatedDeltaNet(cfg, parallel=OneRank)
                               for _ in range(n_layers)]
                for m in self.layers:
                    h = c["hidden"]
                    Fw = m._fused_weight()
                    Fw.normal_(0, h ** -0.5, generator=g)
                    m.conv1d.weight.uniform_(-0.5, 0.5, generator=g)
                    m.A_log.uniform_(-1.0, 0.0, generator=g)
                    m.dt_bias.zero_()
                    m.norm.weight.fill_(1.0)
                    m.out_proj.weight.normal_(0, (c["HV"] * c["DV"]) ** -0.5, generator=g)
        finally:
            torch.set_default_dtype(prev)
        self.pools = None   # a pipeline stage can own no layers (ceil split, many stages)
        if self.layers:
            self.pools = pkg.state_pool.StatePools(self.layers, c["slots"], device)
            with torch.no_grad():
                self.pools.s_pool.normal_(0, 0.02, generator=g)
                self.pools.conv_pool.normal_(0, 1.0, generator=g)
        perm = torch.randperm(c["slots"], generator=torch.Generator().manual_seed(seed))
        self.ids = perm[:c["bs"]].to(device)
        self.cu = torch.arange(c["bs"] + 1, dtype=torch.int32, device=device)
        self.x = torch.empty(c["bs"], c["hidden"], dtype=torch.bfloat16, device=device)
        self.x.normal_(0, 1.0, generator=g)
        self.graph = None

    def _step(self, h):
        for m in self.layers:
            h = h + m(None, h)
        return h

    def capture(self):
        if not self.layers:          # an empty pipeline stage passes hidden through
            self.y = self.x
            return
        ctx = self.pkg.context
        ctx.set_context(self.cu, self.cu, 1, 1, linear_state_ids=self.ids)
        with torch.inference_mode():
            for _ in range(2):
                self.y = self._step(self.x)
            torch.cuda.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.y = self._step(self.x)
        ctx.reset_context()

    def replay(self):
        if self.graph is not None:
            self.graph.replay()


C3 = dict(layers=24, attn_every=4, hidden=2048, HK=16, DK=128, HV=32, DV=128, K=4, q_heads=16,
          kv_heads=4, head_dim=128, inter=6144, vocab=151936, bs=128, ctx_lo=256, ctx_hi=4096,
          gen=256, slots=256, eps=1e-6)


def _add_rms(h, r, w, eps):
    """Fused residual add + RMSNorm of the decoder chain (models/qwen3.py's
    RMSNorm with a residual): r <- h + r, h <- rmsnorm(r) * w."""
    r = h if r is None else (h.float() + r.float()).to(h.dtype)
    x = r.float()
    x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return (x * w.float()).to(h.dtype), r


class HybridStage:
    """One pipeline stage of a config-3-shaped hybrid decoder (decode step):
    the stage's contiguous range of the 24 layers (split_layers, 3 per stage
    at 8 stages), every 4th layer full attention and the rest GatedDeltaNet
    (this package's layer), each followed by a SwiGLU MLP (6144), with the
    fused residual chain (hidden, residual) between layers; the first stage
    embeds the tokens (vocab 151,936), the last applies the final norm and the
    LM head and takes the greedy token.  Attention is GQA 16 q / 4 kv heads x
    128 through torch SDPA over a contiguous KV cache whose length is the mean
    config-3 context (prompts U[256, 4096] plus half of 256 generated tokens:
    2304): the attention layers' weights and KV bytes are config 3's, but the
    KV cache is not paged.  Weights random (seeded); the whole stage step is
    one CUDA graph."""

    def __init__(self, pkg, dev, seed, lo, hi, first, last):
        c = C3
        self.pkg, self.dev, self.first, self.last = pkg, dev, first, last
        H, bs = c["hidden"], c["bs"]
        g = torch.Generator(device=dev).manual_seed(seed)

        def nrm(*shape, std):
            return (torch.randn(*shape, generator=g, device=dev) * std).to(torch.bfloat16)

        cfg = type("Cfg", (), dict(hidden_size=H, linear_num_key_heads=c["HK"],
                                   linear_num_value_heads=c["HV"], linear_key_head_dim=c["DK"],
                                   linear_value_head_dim=c["DV"], linear_conv_kernel_dim=c["K"],
                                   rms_norm_eps=c["eps"]))
        self.ctx_len = (c["ctx_lo"] + c["ctx_hi"]) // 2 + c["gen"] // 2
        self.layers = []
        gdn = []
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            for i in range(lo, hi):
                L = {"ln1": torch.ones(H, dtype=torch.bfloat16, device=dev),
                     "ln2": torch.ones(H, dtype=torch.bfloat16, device=dev),
                     "gate_up": nrm(2 * c["inter"], H, std=H ** -0.5),
                     "down": nrm(H, c["inter"], std=c["inter"] ** -0.5)}
                if (i + 1) % c["attn_every"] == 0:
                    qd, kd = c["q_heads"] * c["head_dim"], c["kv_heads"] * c["head_dim"]
                    L["qkv"] = nrm(qd + 2 * kd, H, std=H ** -0.5)
                    L["o"] = nrm(H, qd, std=qd ** -0.5)
                    L["k_cache"] = nrm(bs, c["kv_heads"], self.ctx_len, c["head_dim"], std=1.0)
                    L["v_cache"] = nrm(bs, c["kv_heads"], self.ctx_len, c["head_dim"], std=1.0)
                else:
                    with torch.device(dev), torch.no_grad():
                        # unsharded: a pipeline stage's layers hold no collective
                        m = pkg.layer.Qwen3_5GatedDeltaNet(cfg, parallel=OneRank)
                        m._fused_weight().normal_(0, H ** -0.5, generator=g)
                        m.conv1d.weight.uniform_(-0.5, 0.5, generator=g)
                        m.A_log.uniform_(-1.0, 0.0, generator=g)
                        m.dt_bias.zero_()
                        m.out_proj.weight.normal_(0, (c["HV"] * c["DV"]) ** -0.5, generator=g)
                    L["gdn"] = m
                    gdn.append(m)
                self.layers.append(L)
        finally:
            torch.set_default_dtype(prev)
        if gdn:
            self.pools = pkg.state_pool.StatePools(gdn, c["slots"], dev)
            with torch.no_grad():
                self.pools.s_pool.normal_(0, 0.02, generator=g)
        perm = torch.randperm(c["slots"], generator=torch.Generator().manual_seed(seed))
        self.ids = perm[:bs].to(dev)
        self.cu = torch.arange(bs + 1, dtype=torch.int32, device=dev)
        self.embed = nrm(c["vocab"], H, std=1.0) if first else None
        self.lm_head = nrm(c["vocab"], H, std=H ** -0.5) if last else None
        self.final_ln = torch.ones(H, dtype=torch.bfloat16, device=dev)
        self.tokens = torch.randint(0, c["vocab"], (bs,), generator=g, device=dev)
        self.x_h = torch.randn(bs, H, generator=g, device=dev).to(torch.bfloat16)
        self.x_r = torch.randn(bs, H, generator=g, device=dev).to(torch.bfloat16)
        self.graph = None

    def _attn(self, L, h):
        c = C3
        bs, qh, kh, hd = h.shape[0], c["q_heads"], c["kv_heads"], c["head_dim"]
        qkv = torch.nn.functional.linear(h, L["qkv"])
        q = qkv[:, :qh * hd].view(bs, qh, 1, hd)
        o = torch.nn.functional.scaled_dot_product_attention(q, L["k_cache"], L["v_cache"],
                                                             enable_gqa=True)
        return torch.nn.functional.linear(o.reshape(bs, qh * hd), L["o"])

    def _step(self):
        eps = C3["eps"]
        if self.first:
            h, r = self.embed[self.tokens], None
        else:
            h, r = self.x_h, self.x_r
        for L in self.layers:
            h, r = _add_rms(h, r, L["ln1"], eps)
            h = self._attn(L, h) if "qkv" in L else L["gdn"](None, h)
            h, r = _add_rms(h, r, L["ln2"], eps)
            gu = torch.nn.functional.linear(h, L["gate_up"])
            a, b = gu.chunk(2, dim=-1)
            h = torch.nn.functional.linear(torch.nn.functional.silu(a) * b, L["down"])
        if self.last:
            h, _ = _add_rms(h, r, self.final_ln, eps)
            return torch.nn.functional.linear(h, self.lm_head).argmax(-1), None
        return h, r

    def capture(self):
        ctx = self.pkg.context
        ctx.set_context(self.cu, self.cu, 1, 1, linear_state_ids=self.ids)
        with torch.inference_mode():
            for _ in range(2):
                self.y_h, self.y_r = self._step()
            torch.cuda.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.y_h, self.y_r = self._step()
        ctx.reset_context()

    def replay(self):
        self.graph.replay()


def pp_bench(pkg, dev, world, rank, steps, warmup):
    """Config-3-shaped hybrid decoder (HybridStage) as a `world`-stage
    pipeline, decode steps of 128 sequences.  Stage r hands (hidden,
    residual) to stage r + 1 through PipelineHandoff — one packed NCCL
    message per boundary on a side stream and on that boundary's own
    two-rank process group, double-buffered and event-ordered — in place of
    the reference's two blocking send / recv calls per boundary
    (engine/model_runner.py:795-810).  Stage r starts step i + 1 as soon as
    it has queued step i, so successive steps (independent micro-batches)
    overlap across stages.

    Three timings, CUDA events, max over ranks, `steps` steps each:
      t_stage  each stage's graph alone (no handoff)
      t_local  each stage with the handoff replaced by local copies of the
               same bytes (the receive buffer copied in, the output copied out)
      t_pp     the pipeline with the NCCL handoff
    t_local and t_pp alternate three times and their medians are used.
    K steps through S stages take K + S - 1 stage steps even with a free
    handoff (the pipeline fills once), so exposed handoff = (t_pp - fill -
    t_local) / t_pp with fill = (S - 1) t_local / K."""
    c = C3
    P = pkg.parallel
    lo, hi = P.split_layers(c["layers"], world, rank)
    prev, nxt = P.pp_peers(rank, 1, world)
    stage = HybridStage(pkg, dev, seed=4321 + rank, lo=lo, hi=hi, first=prev is None,
                        last=nxt is None)
    stage.capture()
    barrier(world)
    # the boundary groups are made after every rank's capture: no NCCL communicator
    # is created or connected while a CUDA graph is being captured
    groups = P.boundary_groups(world)
    ho = P.PipelineHandoff(c["hidden"], c["bs"], torch.bfloat16, dev, prev, nxt, mode="packed",
                           recv_group=groups[rank - 1] if prev is not None else None,
                           send_group=groups[rank] if nxt is not None else None)
    rbuf = torch.empty(2, c["bs"], c["hidden"], dtype=torch.bfloat16, device=dev)
    sbuf = torch.empty_like(rbuf)

    def stage_only():
        stage.replay()

    def local_step():
        if prev is not None:
            stage.x_h.copy_(rbuf[0])
            stage.x_r.copy_(rbuf[1])
        stage.replay()
        if nxt is not None:
            sbuf[0].copy_(stage.y_h)
            sbuf[1].copy_(stage.y_r)

    def pp_step():
        if prev is not None:
            h, r = ho.recv(c["bs"])
            stage.x_h.copy_(h)
            stage.x_r.copy_(r)
            ho.consumed()        # the next receive need not wait for this step's compute
        stage.replay()
        if nxt is not None:
            ho.send(stage.y_h, stage.y_r)

    for fn in (stage_only, local_step, pp_step):
        for _ in range(warmup):
            fn()
        ho.flush()
        torch.cuda.synchronize()
    t_stage = time_region(stage_only, steps, world)
    # local-copy and pipelined timings alternate three times (medians): the GPUs'
    # power-capped clocks drift over seconds, more than the handoff costs
    t_locals, t_pps = [], []
    for _ in range(3):
        t_locals.append(time_region(local_step, steps, world))
        t_pps.append(time_region(pp_step, steps, world))
        ho.flush()
        torch.cuda.synchronize()
    barrier(world)
    t_local, t_pp = statistics.median(t_locals), statistics.median(t_pps)
    fill = (world - 1) * t_local / steps
    exposed = (t_pp - fill - t_local) / t_pp
    per_stage = [b - a for a, b in (P.split_layers(c["layers"], world, r) for r in range(world))]
    out = {"workload": "config3-shaped hybrid decoder, decode steps of 128 sequences: 24 layers "
                       "(every 4th full attention GQA 16q/4kv x 128 over a 2304-token KV cache, "
                       "the rest GDN), SwiGLU 6144, vocab 151936, bf16; embedding on the first "
                       "stage, final norm + LM head + greedy token on the last",
           "stages": world, "layers_per_stage": per_stage,
           "handoff": "PipelineHandoff packed (hidden, residual), NCCL send/recv on a side "
                      "stream, one two-rank process group per boundary",
           "bytes_per_handoff": 2 * c["bs"] * c["hidden"] * 2, "steps": steps,
           "ms_per_step_pipelined": round(t_pp / steps * 1e3, 4),
           "ms_per_step_local_copy": round(t_local / steps * 1e3, 4),
           "ms_per_step_runs": {"pipelined": [round(t / steps * 1e3, 4) for t in t_pps],
                                "local_copy": [round(t / steps * 1e3, 4) for t in t_locals]},
           "ms_per_step_slowest_stage": round(t_stage / steps * 1e3, 4),
           "pipeline_fill_ms": round(fill * 1e3, 4),
           "exposed_handoff_ms_per_step": round((t_pp - fill - t_local) / steps * 1e3, 4),
           "exposed_handoff_frac": round(exposed, 4),
           "tok_s_pipelined": round(c["bs"] * steps / t_pp, 1)}
    stage.graph = None
    return out


def hybrid_single_gpu(pkg, dev, steps, warmup):
    """The config-3-shaped hybrid decoder of pp_bench run whole on one GPU (all
    24 layers, embedding and LM head in one CUDA graph): the step the pipeline
    splits, for comparing pipelined throughput at N stages against one GPU."""
    c = C3
    stage = HybridStage(pkg, dev, seed=4321, lo=0, hi=c["layers"], first=True, last=True)
    stage.capture()
    for _ in range(warmup):
        stage.replay()
    t = time_region(stage.replay, steps, 1)
    out = {"workload": "config3-shaped hybrid decoder (as pp), all 24 layers on one GPU, "
                       "decode steps of 128 sequences",
           "steps": steps, "ms_per_step": round(t / steps * 1e3, 4),
           "tok_s": round(c["bs"] * steps / t, 1)}
    stage.graph = None
    return out


def time_region(fn, steps, world, stream=None):
    """CUDA-event time of ``steps`` calls of fn, bracketed by barrier + sync."""
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(e0.elapsed_time(e1) / 1e3, world)


def decode_kernel_roofline(pkg, stack, peaks, launches):
    """Time the fused decode-core kernel alone as the layer launches it (one
    launch per layer, each on its own layer views of the stack's 38.7 GB state
    and conv pools) with CUDA events on its stream."""
    ops = pkg.ops
    c = C1
    bs, HK, HV, D, K = c["bs"], c["HK"], c["HV"], c["DK"], c["K"]
    m0 = stack.layers[0]
    g = torch.Generator(device=stack.dev).manual_seed(7)
    C = m0.conv_dim
    W = m0._fused_weight().shape[0]
    proj = torch.randn(bs, W, generator=g, device=stack.dev).to(torch.bfloat16)
    r = m0._proj_rows
    mixed, z = proj[:, :C], proj[:, r[0]:r[1]].view(bs, HV, D)
    b, a = proj[:, r[1]:r[2]], proj[:, r[2]:r[3]]

    def launch(m):
        return ops.decode_fused(mixed, z, b, a, m.conv_cache,
                                m.conv1d.weight.view(m.conv_dim, m.conv_kernel), m.A_log,
                                m.dt_bias, m.s_cache, stack.ids, m.norm.weight, m.norm.eps)

    with torch.inference_mode():
        for m in stack.layers[:3]:
            launch(m)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = 0
        e0.record()
        for _ in range(launches):
            for m in stack.layers:
                launch(m)
                n += 1
        e1.record()
        torch.cuda.synchronize()
    dt = e0.elapsed_time(e1) / 1e3 / n
    algo = decode_algorithmic_bytes(bs, HK, HV, D, K)
    achieved = algo / dt / 1e9
    traffic = read_profile_traffic("decode_fused_c1.md")
    return {"kernel": "decode_fused_kernel", "bound": "hbm", "achieved": round(achieved, 1),
            "peak": peaks["hbm_gbs"], "peak_source": peaks["source"], "unit": "GB/s",
            "frac": round(achieved / peaks["hbm_gbs"], 4),
            "traffic": traffic, "algorithmic_bytes_per_launch": algo,
            "launch_us": round(dt * 1e6, 2), "launches_timed": n}


def decode_algorithmic_bytes(bs, HK, HV, D, K):
    """Bytes one fused decode launch must move: each (row, v-head) state read
    and written once (fp32), each conv state read and written once, the
    projection inputs read (q/k/v channels, z, a, b), the output written, the
    conv weight and slot ids read."""
    C = (2 * HK + HV) * D
    state = 2 * bs * HV * D * D * 4
    conv_state = 2 * bs * C * (K - 1) * 2
    inputs = bs * (C + HV * D + 2 * HV) * 2
    out = bs * HV * D * 2
    return state + conv_state + inputs + out + C * K * 2 + bs * 8


def read_profile_traffic(name):
    """dram bytes per launch recorded in a committed ncu summary, if any."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("dram_bytes_per_launch:"):
            try:
                return int(line.split(":")[1].strip().split()[0])
            except ValueError:
                return None
    return None


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "source": "fallback"}


# ---------------------------------------------------------------------------
# config-2 prefill (secondary)
# ---------------------------------------------------------------------------


def prefill_bench(pkg, device, steps, peaks):
    c = C2
    rng = np.random.Generator(np.random.PCG64(2))
    lens = rng.integers(c["len_lo"], c["len_hi"] + 1, size=c["n_seqs"]).tolist()
    N = int(sum(lens))
    cfg = type("Cfg", (), dict(hidden_size=c["hidden"], linear_num_key_heads=c["HK"],
                               linear_num_value_heads=c["HV"], linear_key_head_dim=c["DK"],
                               linear_value_head_dim=c["DV"], linear_conv_kernel_dim=c["K"],
                               rms_norm_eps=1e-6))
    g = torch.Generator(device=device).manual_seed(3)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(device), torch.no_grad():
            m = pkg.layer.Qwen3_5GatedDeltaNet(cfg, parallel=OneRank)
            m._fused_weight().normal_(0, c["hidden"] ** -0.5, generator=g)
            m.conv1d.weight.uniform_(-0.5, 0.5, generator=g)
            m.A_log.uniform_(-1.0, 0.0, generator=g)
            m.dt_bias.zero_()
            m.out_proj.weight.normal_(0, 4096 ** -0.5, generator=g)
    finally:
        torch.set_default_dtype(prev)
    pools = pkg.state_pool.StatePools([m], c["n_seqs"], device)
    ids = torch.randperm(c["n_seqs"], generator=torch.Generator().manual_seed(4)).to(device)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=device)
    x = torch.randn(N, c["hidden"], generator=g, device=device).to(torch.bfloat16)
    ctx = pkg.context

    def step():
        pools.reset(ids)                       # fresh prefill: zero slots
        ctx.set_context(cu, cu, max(lens), max(lens), linear_state_ids=ids, lens_q=lens)
        with torch.inference_mode():
            m(None, x)
        ctx.reset_context()

    for _ in range(2):
        step()
    torch.cuda.synchronize()
    per_step = []
    for _ in range(steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step()
        e1.record()
        torch.cuda.synchronize()
        per_step.append(e0.elapsed_time(e1) / 1e3)
    t = statistics.median(per_step)
    # Stage breakdown of one step (CUDA events), the chunk kernel alone and the
    # gated norm alone.  Every measured call runs once untimed first, so the
    # caching allocator already holds its output blocks (a fresh multi-GB
    # cudaMalloc next to the 40 GB decode stack costs ~100 ms).
    stage_runs = {}
    with torch.inference_mode():
        for rep in range(4):   # one untimed pass, then the median of three
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
            pools.reset(ids)
            ev[0].record()
            proj = torch.nn.functional.linear(x, m._fused_weight())
            ev[1].record()
            r = m._proj_rows
            y, gg, beta = pkg.ops.conv_gate_varlen(proj[:, :m.conv_dim], m.conv_cache, ids,
                                                   m.conv1d.weight, cu, proj[:, r[1]:r[2]],
                                                   proj[:, r[2]:r[3]], m.A_log, m.dt_bias)
            ev[2].record()
            q, k, v = m._split(y)
            z = proj[:, r[0]:r[1]].view(N, c["HV"], c["DV"])
            core = pkg.ops.chunk_gated_delta_rule_varlen(q, k, v, gg, beta, m.s_cache, ids, cu,
                                                         max(lens), z=z,
                                                         norm_weight=m.norm.weight)
            ev[3].record()
            m.out_proj(core.view(N, c["HV"] * c["DV"]))
            ev[4].record()
            torch.cuda.synchronize()
            for i, name in enumerate(["in_proj_gemm", "conv_and_gate", "chunk_with_norm",
                                      "out_proj_gemm"]):
                if rep > 0:
                    stage_runs.setdefault(name, []).append(ev[i].elapsed_time(ev[i + 1]))
            del core
            if rep < 3:    # free this pass's buffers before the next pass allocates
                del proj, gg, beta, y, q, k, v, z
                torch.cuda.synchronize()
        stages = {k: round(statistics.median(v), 3) for k, v in stage_runs.items()}
        pkg.ops.chunk_gated_delta_rule_varlen(q, k, v, gg, beta, m.s_cache, ids, cu, max(lens))
        torch.cuda.synchronize()
        clocks = Clocks(device.index if device.index is not None else 0)
        clocks.start()
        csteps = max(steps, 50)            # ~0.3 s: long enough for the clock sampler
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(csteps):
            pkg.ops.chunk_gated_delta_rule_varlen(q, k, v, gg, beta, m.s_cache, ids, cu,
                                                  max(lens))
        e1.record()
        torch.cuda.synchronize()
        chunk_clk = clocks.stop()
        # the one-kernel form (no workspace), for comparison
        pkg.ops.chunk_gated_delta_rule_varlen(q, k, v, gg, beta, m.s_cache, ids, cu, max(lens),
                                              split=False)
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(steps):
            pkg.ops.chunk_gated_delta_rule_varlen(q, k, v, gg, beta, m.s_cache, ids, cu,
                                                  max(lens), split=False)
        s1.record()
        torch.cuda.synchronize()
        o = pkg.ops.chunk_gated_delta_rule_varlen(q, k, v, gg, beta, m.s_cache, ids, cu,
                                                  max(lens))
        pkg.ops.rms_norm_gated(o, z, m.norm.weight, 1e-6)
        torch.cuda.synchronize()
        n0, n1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0.record()
        for _ in range(steps):
            pkg.ops.rms_norm_gated(o, z, m.norm.weight, 1e-6)
        n1.record()
        torch.cuda.synchronize()
    tn = n0.elapsed_time(n1) / 1e3 / steps
    norm_bytes = 3 * N * c["HV"] * c["DV"] * 2
    tk = e0.elapsed_time(e1) / 1e3 / csteps
    flops = CHUNK_FLOPS_PER_TOKEN_HEAD * N * c["HV"]
    achieved = flops / tk / 1e12
    return {"workload": "config2: 1 GDN layer, 64 seqs, lens U[128,8192] seed 2, "
                        f"{N} tokens, full layer forward",
            "value": round(N / t, 1), "unit": "tok/s", "tokens": N, "ms_per_step": round(t * 1e3, 3),
            "ms_per_step_min": round(min(per_step) * 1e3, 3), "stages_ms": stages,
            "norm_kernel": {"kernel": "rms_gated_kernel (config-2 core output)",
                            "ms": round(tn * 1e3, 3), "bound": "hbm",
                            "achieved": round(norm_bytes / tn / 1e9, 1), "unit": "GB/s",
                            "frac": round(norm_bytes / tn / 1e9 / peaks["hbm_gbs"], 4)},
            "chunk_kernel": {"kernel": "chunk_index_kernel + chunk_prep_kernel + "
                                       "chunk_chain_kernel (split form, one call)",
                             "bound": "tensor",
                             "ms": round(tk * 1e3, 3), "tok_s": round(N / tk, 1),
                             "one_kernel_form_ms": round(s0.elapsed_time(s1) / steps, 3),
                             "workspace_bytes": pkg.ops.chunk_prefill_workspace_bytes(
                                 N, c["n_seqs"], c["HV"], c["DK"], c["DV"]),
                             "achieved": round(achieved, 2), "unit": "TFLOP/s",
                             "peak": peaks["bf16_tflops"], "peak_source": peaks["source"],
                             "frac": round(achieved / peaks["bf16_tflops"], 5),
                             "algorithmic_flops": flops, "clocks": chunk_clk}}


# ---------------------------------------------------------------------------
# config-2 prefill with the v-heads sharded over the ranks (tensor parallel)
# ---------------------------------------------------------------------------


def config2_lens():
    c = C2
    rng = np.random.Generator(np.random.PCG64(2))
    return rng.integers(c["len_lo"], c["len_hi"] + 1, size=c["n_seqs"]).tolist()


def config2_cfg():
    c = C2
    return type("Cfg", (), dict(hidden_size=c["hidden"], linear_num_key_heads=c["HK"],
                                linear_num_value_heads=c["HV"], linear_key_head_dim=c["DK"],
                                linear_value_head_dim=c["DV"], linear_conv_kernel_dim=c["K"],
                                rms_norm_eps=1e-6))


def config2_full_weights(device, seed):
    """Full (unsharded) config-2 layer weights from a seeded device generator:
    every rank draws the same tensors."""
    c = C2
    H, HK, HV, D, K = c["hidden"], c["HK"], c["HV"], c["DK"], c["K"]
    cd = 2 * HK * D + HV * D
    g = torch.Generator(device=device).manual_seed(seed)

    def nrm(*shape, std):
        return (torch.randn(*shape, generator=g, device=device) * std).to(torch.bfloat16)

    return {"in_proj_qkv.weight": nrm(cd, H, std=H ** -0.5),
            "in_proj_z.weight": nrm(HV * D, H, std=H ** -0.5),
            "in_proj_b.weight": nrm(HV, H, std=H ** -0.5),
            "in_proj_a.weight": nrm(HV, H, std=H ** -0.5),
            "conv1d.weight": ((torch.rand(cd, 1, K, generator=g, device=device) - 0.5)
                              .to(torch.bfloat16)),
            "A_log": (-torch.rand(HV, generator=g, device=device)).to(torch.bfloat16),
            "dt_bias": torch.zeros(HV, dtype=torch.bfloat16, device=device),
            "norm.weight": torch.ones(D, dtype=torch.bfloat16, device=device),
            "out_proj.weight": nrm(H, HV * D, std=(HV * D) ** -0.5)}


def build_loaded_layer(pkg, cfg, weights, device, parallel=None):
    """A layer on `device` whose parameters are loaded from full weights through
    the layer's own weight loaders (the engine's load path), so a sharded
    layer takes its rank's heads."""
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(device):
            m = pkg.layer.Qwen3_5GatedDeltaNet(cfg, parallel=parallel)
    finally:
        torch.set_default_dtype(prev)
    with torch.no_grad():
        for name, w in weights.items():
            p = m.get_parameter(name)
            getattr(p, "weight_loader", lambda p_, w_: p_.data.copy_(w_))(p, w)
    return m


def tp_prefill_bench(pkg, dev, world, rank, steps):
    """Config-2 varlen prefill of one layer with the 32 v-heads (and the
    matching k-heads) sharded over the `world` ranks as the reference's
    tensor parallelism shards them (qwen3_5.py:796-835): each rank runs the
    projection GEMM of its heads, the conv / chunk kernels on its heads and
    the out_proj partial product, which an NCCL all-reduce sums
    (layers/linear.py:154-158).  Strong scaling: the same 282,505 tokens at
    every N.  Reports tok/s (max-over-ranks step time), the efficiency
    against the unsharded layer on one of these GPUs, the all-reduce's share,
    and tp_parity: every rank also runs the unsharded layer from the same
    seeds and compares the all-reduced output and its own heads' final
    states."""
    c = C2
    P = pkg.parallel
    P.init_parallel_state(rank, world, tp_size=world, pp_size=1)
    lens = config2_lens()
    N = int(sum(lens))
    cfg = config2_cfg()
    W = config2_full_weights(dev, seed=11)
    m = build_loaded_layer(pkg, cfg, W, dev)                      # this rank's shard
    ref = build_loaded_layer(pkg, cfg, W, dev, parallel=OneRank)  # the whole layer
    del W
    pools = pkg.state_pool.StatePools([m], c["n_seqs"], dev)
    ref_pools = pkg.state_pool.StatePools([ref], c["n_seqs"], dev)
    ids = torch.randperm(c["n_seqs"], generator=torch.Generator().manual_seed(4)).to(dev)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
    g = torch.Generator(device=dev).manual_seed(3)
    x = torch.randn(N, c["hidden"], generator=g, device=dev).to(torch.bfloat16)
    ctx = pkg.context

    def run(layer, pl):
        pl.reset(ids)                          # fresh prefill: zero slots
        ctx.set_context(cu, cu, max(lens), max(lens), linear_state_ids=ids, lens_q=lens)
        try:
            with torch.inference_mode():
                return layer(None, x)
        finally:
            ctx.reset_context()

    for _ in range(2):
        run(m, pools)
        run(ref, ref_pools)
    torch.cuda.synchronize()
    t_tp = time_region(lambda: run(m, pools), steps, world)
    t_one = time_region(lambda: run(ref, ref_pools), steps, world)
    # the out_proj all-reduce alone, on the same [N, hidden] bf16 shape
    y = torch.empty(N, c["hidden"], dtype=torch.bfloat16, device=dev)
    grp = P.get_tp_group()
    for _ in range(2):
        torch.distributed.all_reduce(y, group=grp)
    t_ar = time_region(lambda: torch.distributed.all_reduce(y, group=grp), steps, world)
    del y
    # parity: one fresh prefill through both layers
    y_tp = run(m, pools)
    y_ref = run(ref, ref_pools)
    torch.cuda.synchronize()
    out_err = (y_tp.float() - y_ref.float()).abs().max().item()
    out_mag = y_ref.float().abs().max().item()
    hv = slice(rank * m.num_v_heads, (rank + 1) * m.num_v_heads)
    a, b = m.s_cache[ids], ref.s_cache[ids][:, hv]
    state_rel = max(((a[i] - b[i]).norm() / b[i].norm().clamp_min(1e-30)).item()
                    for i in range(a.shape[0]))
    errs = torch.tensor([out_err, state_rel], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(errs, op=torch.distributed.ReduceOp.MAX)
    out_err, state_rel = errs.tolist()
    pkg.ops.check_status(dev)
    per_step = t_tp / steps
    flops = CHUNK_FLOPS_PER_TOKEN_HEAD * N * c["HV"]
    res = {"workload": f"config2 prefill, 1 GDN layer, {N} tokens (64 seqs, lens U[128,8192] "
                       f"seed 2), v-heads sharded {world} ways",
           "parallelism": f"tp{world}", "scaling": "strong",
           "v_heads_per_gpu": m.num_v_heads, "k_heads_per_gpu": m.num_k_heads,
           "value": round(N / per_step, 1), "unit": "tok/s",
           "ms_per_step": round(per_step * 1e3, 3), "steps": steps,
           "ms_per_step_unsharded_1gpu": round(t_one / steps * 1e3, 3),
           "efficiency_vs_1gpu": round((t_one / steps) / (world * per_step), 4),
           "allreduce": {"what": f"NCCL all_reduce of the out_proj output [{N}, "
                                 f"{c['hidden']}] bf16", "ms": round(t_ar / steps * 1e3, 3),
                         "share_of_step": round((t_ar / steps) / per_step, 4)},
           "chunk_tflops_per_gpu": round(flops / world / per_step / 1e12, 1),
           "tp_parity": {"vs": "the unsharded layer from the same seeds on each rank",
                         "out_max_abs": out_err, "out_ref_max_abs": round(out_mag, 3),
                         "state_rel_max": state_rel,
                         "tolerance": {"out_max_abs": 2e-2, "state_rel": 2e-2},
                         "pass": bool(out_err <= 2e-2 and state_rel <= 2e-2)}}
    del m, ref, pools, ref_pools, x, y_tp, y_ref
    torch.cuda.empty_cache()
    P.reset_parallel_state()     # later sections build unsharded layers
    return res


# ---------------------------------------------------------------------------
# config 4: long-context prefill + decode, v-heads over 8 GPUs
# ---------------------------------------------------------------------------

C4 = dict(n_seqs=8, seq_len=131072, shards=8, decode_steps=1024)


def config4_bench(pkg, dev, world, rank, peaks):
    """Config 4: 8 sequences of 131,072 tokens through one GDN layer at
    config-2 head shapes, chunked prefill then 1024 decode steps, the 32
    v-heads sharded 8 ways (4 v-heads / 2 k-heads per GPU).  At 8 ranks each
    rank runs its shard and out_proj all-reduces over NCCL; on 1 GPU the
    bench runs shard 0 of 8 (the same per-GPU kernels and bytes; the
    all-reduce across shards is not run).  Reports the prefill layer time,
    the chunk prefill kernels alone against the bf16 tensor roofline, the
    decode step (one layer forward per step, captured in a CUDA graph) and
    the fused decode core alone against HBM (state bytes 2 x 8 x 4 x 64 KiB
    per step per GPU)."""
    c, c4 = C2, C4
    shards = c4["shards"]
    assert world in (1, shards)
    tp_rank = rank if world == shards else 0
    P = pkg.parallel
    if world == shards:
        P.init_parallel_state(rank, world, tp_size=world, pp_size=1)
        par = None
    else:
        par = type("OneShardOf8", (), dict(get_tp_rank=staticmethod(lambda: 0),
                                          get_tp_size=staticmethod(lambda: shards),
                                          get_tp_group=staticmethod(lambda: None)))
    W = config2_full_weights(dev, seed=13)
    m = build_loaded_layer(pkg, config2_cfg(), W, dev, parallel=par)
    del W
    if world == 1:
        m.out_proj.tp_size = 1           # the partial sum of this shard; no peers to reduce with
    n, T = c4["n_seqs"], c4["seq_len"]
    lens = [T] * n
    N = n * T
    pools = pkg.state_pool.StatePools([m], n, dev)
    ids = torch.randperm(n, generator=torch.Generator().manual_seed(9)).to(dev)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
    g = torch.Generator(device=dev).manual_seed(21)
    x = torch.randn(N, c["hidden"], generator=g, device=dev).to(torch.bfloat16)
    ctx = pkg.context

    def prefill():
        pools.reset(ids)
        ctx.set_context(cu, cu, T, T, linear_state_ids=ids, lens_q=lens)
        try:
            with torch.inference_mode():
                return m(None, x)
        finally:
            ctx.reset_context()

    prefill()
    torch.cuda.synchronize()
    t_pre = time_region(prefill, 2, world) / 2
    # the chunk prefill kernels alone on this shard's heads (conv output of the layer's q/k/v)
    with torch.inference_mode():
        proj = torch.nn.functional.linear(x, m._fused_weight())
        r = m._proj_rows
        y, gg, beta = pkg.ops.conv_gate_varlen(proj[:, :m.conv_dim], m.conv_cache, ids,
                                               m.conv1d.weight, cu, proj[:, r[1]:r[2]],
                                               proj[:, r[2]:r[3]], m.A_log[m._v_head_slice],
                                               m.dt_bias[m._v_head_slice])
        del proj
        q, k, v = m._split(y)
        chunk = lambda: pkg.ops.chunk_gated_delta_rule_varlen(q, k, v, gg, beta, m.s_cache, ids,
                                                              cu, T)
        chunk()
        torch.cuda.synchronize()
        t_chunk = time_region(chunk, 3, world) / 3
        del q, k, v, y, gg, beta
    torch.cuda.empty_cache()
    flops = CHUNK_FLOPS_PER_TOKEN_HEAD * N * m.num_v_heads
    # decode: states from a fresh prefill, then 1024 steps of one token per sequence
    prefill()
    cu1 = torch.arange(n + 1, dtype=torch.int32, device=dev)
    h = torch.randn(n, c["hidden"], generator=g, device=dev).to(torch.bfloat16)
    # the captured step holds no NCCL call: out_proj's all-reduce of the [8, 2048]
    # partial sums is timed on its own below
    tp_size = m.out_proj.tp_size
    m.out_proj.tp_size = 1
    ctx.set_context(cu1, cu1, 1, 1, linear_state_ids=ids)
    try:
        with torch.inference_mode():
            for _ in range(2):
                yd = m(None, h)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                yd = m(None, h)
    finally:
        ctx.reset_context()
        m.out_proj.tp_size = tp_size
    steps = c4["decode_steps"]
    t_dec = time_region(graph.replay, steps, world) / steps
    del graph
    t_ar = 0.0
    if world > 1:
        yr = torch.empty(n, c["hidden"], dtype=torch.bfloat16, device=dev)
        for _ in range(5):
            torch.distributed.all_reduce(yr, group=m.out_proj.tp_group)
        t_ar = time_region(lambda: torch.distributed.all_reduce(yr, group=m.out_proj.tp_group),
                           200, world) / 200
    # the fused decode core alone (the kernel the decode step runs), CUDA events
    bs, HK, HV, D = n, m.num_k_heads, m.num_v_heads, c["DK"]
    pj = torch.randn(bs, m._fused_weight().shape[0], generator=g, device=dev).to(torch.bfloat16)
    rr = m._proj_rows
    core = lambda: pkg.ops.decode_fused(
        pj[:, :m.conv_dim], pj[:, rr[0]:rr[1]].view(bs, HV, D), pj[:, rr[1]:rr[2]],
        pj[:, rr[2]:rr[3]], m.conv_cache, m.conv1d.weight.view(m.conv_dim, m.conv_kernel),
        m.A_log[m._v_head_slice], m.dt_bias[m._v_head_slice], m.s_cache, ids, m.norm.weight,
        m.norm.eps)
    with torch.inference_mode():      # 100 launches per graph: the kernel, not the host
        for _ in range(3):
            core()
        torch.cuda.synchronize()
        cg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(cg):
            for _ in range(100):
                core()
        cg.replay()
        torch.cuda.synchronize()
        t_core = time_region(cg.replay, 3, world) / 300
        del cg
    dec_bytes = decode_algorithmic_bytes(bs, HK, HV, D, c["K"])
    state_bytes = 2 * bs * HV * D * D * 4
    pkg.ops.check_status(dev)
    res = {"workload": f"config4: {n} sequences x {T} tokens, 1 GDN layer at config-2 head "
                       f"shapes, v-heads sharded {shards} ways ({HV} v / {HK} k heads per GPU)"
                       + ("" if world == shards else "; this run: shard 0 of 8 on one GPU, "
                          "without the cross-shard all-reduce"),
           "prefill": {"ms": round(t_pre * 1e3, 3), "tok_s": round(N / t_pre, 1),
                       "chunk_kernels_ms": round(t_chunk * 1e3, 3),
                       "chunk_chain_column_parts":
                           2 if n * m.num_v_heads < 2 * torch.cuda.get_device_properties(
                               dev).multi_processor_count else 1,
                       "chunk_tflops": round(flops / t_chunk / 1e12, 2),
                       "chunk_frac_of_bf16_peak": round(flops / t_chunk / 1e12 /
                                                        peaks["bf16_tflops"], 4)},
           "decode": {"steps": steps, "ms_per_step": round((t_dec + t_ar) * 1e3, 4),
                      "tok_s": round(n / (t_dec + t_ar), 1),
                      "ms_per_step_layer_graph": round(t_dec * 1e3, 4),
                      "ms_allreduce_per_step": round(t_ar * 1e3, 4),
                      "core_kernel_us": round(t_core * 1e6, 2),
                      "core_state_gbs": round(state_bytes / t_core / 1e9, 1),
                      "core_achieved_gbs": round(dec_bytes / t_core / 1e9, 1),
                      "core_frac_of_hbm": round(dec_bytes / t_core / 1e9 / peaks["hbm_gbs"], 4),
                      "algorithmic_bytes_per_launch": dec_bytes,
                      "note": f"{bs * HV} (sequence, v-head) units per GPU, one 64 KiB state "
                              "each: a launch this small is latency-bound, far from the HBM "
                              "roofline"}}
    del m, pools, x, pj
    torch.cuda.empty_cache()
    P.reset_parallel_state()
    return res


# ---------------------------------------------------------------------------
# CPU baseline (the oracle's C restatement + numpy projections)
# ---------------------------------------------------------------------------


def cpu_decode_stack(seed=0):
    """The config-1 decode step on the host cores: all 18 GDN layers, each with
    its own 257-slot state and conv pools (256 sequences + 1), numpy BLAS
    projections, gate / conv / norm in numpy, the recurrence in the C
    restatement; residual add between layers.  Returns (step callable,
    sample description, threads)."""
    from oracle import cref
    from oracle import gdn_oracle as O
    threads = cref.use_all_cores()
    c = C1
    L, bs, H, HK, HV, D = c["layers"], c["bs"], c["hidden"], c["HK"], c["HV"], c["DK"]
    cd = 2 * HK * D + HV * D
    r = np.random.Generator(np.random.PCG64(seed))
    Wf = (r.standard_normal((cd + HV * D + 2 * HV, H), dtype=np.float32) * H ** -0.5)
    Wo = (r.standard_normal((H, HV * D), dtype=np.float32) * (HV * D) ** -0.5)
    conv_w = r.uniform(-0.5, 0.5, (cd, c["K"])).astype(np.float32)
    a_log = r.uniform(-1, 0, HV).astype(np.float32)
    dt_bias = np.zeros(HV, np.float32)
    norm_w = np.ones(D, np.float32)
    # per-layer pools; the states of the first layer are N(0, 0.02), copied to the others
    pools = np.empty((L, bs + 1, HV, D, D), np.float32)
    pools[0] = r.standard_normal((bs + 1, HV, D, D), dtype=np.float32) * 0.02
    for i in range(1, L):
        pools[i] = pools[0]
    conv_pools = np.empty((L, bs + 1, cd, c["K"] - 1), np.float32)
    conv_pools[:] = r.standard_normal((bs + 1, cd, c["K"] - 1), dtype=np.float32)
    ids = r.permutation(bs + 1)[:bs]
    x0 = r.standard_normal((bs, H), dtype=np.float32)

    def layer(x, pool, conv_pool):
        p = x @ Wf.T
        mixed, z = p[:, :cd], p[:, cd:cd + HV * D]
        b, a = p[:, cd + HV * D:cd + HV * D + HV], p[:, cd + HV * D + HV:]
        g, beta = O.fused_g_beta(b, a, a_log, dt_bias, None, None)
        # conv step (vectorised restatement of qwen3_5.py:515-558)
        st = conv_pool[ids]
        acc = mixed * conv_w[:, 3] + (st * conv_w[None, :, :3]).sum(-1)
        with np.errstate(over="ignore"):   # silu of a large negative input is 0
            y = acc / (1 + np.exp(-acc))
        conv_pool[ids] = np.concatenate([st[:, :, 1:], mixed[:, :, None]], -1)
        q = y[:, :HK * D].reshape(bs, HK, D)
        k = y[:, HK * D:2 * HK * D].reshape(bs, HK, D)
        v = y[:, 2 * HK * D:].reshape(bs, HV, D)
        o = cref.recurrent_inplace(q, k, v, g, beta, pool, ids)
        core = O.rms_norm_gated(o, z.reshape(bs, HV, D), norm_w, 1e-6, None)
        return core.reshape(bs, HV * D) @ Wo.T

    def step():
        h = x0
        for i in range(L):
            h = h + layer(h, pools[i], conv_pools[i])
        return h

    sample = (f"the whole config-1 step per step: {L} GDN layers, bs {bs}, each layer's "
              f"state in its own {bs + 1}-slot pool (256 sequences + 1), numpy BLAS "
              "projections + C/OpenMP recurrence")
    return step, sample, threads


def cpu_prefill_baseline(budget_s=8.0):
    """The chunk prefill core (config-2 heads) in the oracle's C restatement on
    the host cores: sequences of 512 tokens x 32 v-heads, as many as the
    budget allows, extrapolated per token.  Projections, conv and norm are not
    included (the GPU chunk-kernel figure excludes them too)."""
    from oracle import cref
    cref.use_all_cores()
    c = C2
    HK, HV, D, T = c["HK"], c["HV"], c["DK"], 512
    r = np.random.Generator(np.random.PCG64(5))
    q = r.standard_normal((T, HK, D), dtype=np.float32)
    k = r.standard_normal((T, HK, D), dtype=np.float32)
    v = r.standard_normal((T, HV, D), dtype=np.float32)
    g = -np.log1p(np.exp(r.standard_normal((T, HV)))).astype(np.float32) * 0.5
    beta = (1 / (1 + np.exp(-r.standard_normal((T, HV))))).astype(np.float32)
    pool = np.zeros((2, HV, D, D), np.float32)
    ids, cu = np.array([0]), np.array([0, T])
    cref.chunk_prefill(q, k, v, g, beta, pool, ids, cu)
    n, t0 = 0, time.perf_counter()
    while True:
        cref.chunk_prefill(q, k, v, g, beta, pool, ids, cu)
        n += 1
        if time.perf_counter() - t0 > budget_s or n >= 50:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": round(T / dt, 1), "unit": "tok/s", "cores": cref.num_threads(),
            "kind": "port",
            "sample": f"chunk prefill core only, {n} sequences of {T} tokens x {HV} v-heads "
                      "(head dim 128, chunk 64) in the C/OpenMP restatement, per token"}


def cpu_baseline(budget_s=20.0):
    """The CPU decode stack on a bounded number of whole steps (~budget_s)."""
    step, sample, threads = cpu_decode_stack()
    step()
    n, t0 = 0, time.perf_counter()
    while True:
        step()
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": round(C1["bs"] / dt, 2), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{sample}; {n} whole steps timed", "ms_per_step": round(dt * 1e3, 1)}


def reference_torch_recurrence(budget_s=15.0):
    """The reference's own torch decode recurrence, timed on the host cores when
    its package is installed next to this file (baseline/_ref; None otherwise):
    one config-1 layer step of its non-in-place decode path (qwen3_5.py:
    1028-1030) — gather the 256 slot states from a 257-slot fp32 pool, run
    recurrent_gated_delta_rule (the pure-torch _torch_recurrent_gated_delta_rule,
    :616-651, with fla switched off and torch.compile disabled, run eagerly) on
    q / k repeated to the v-heads as its split_qkv does (:1002-1005), scatter the
    new states back.  The recurrence only (no projections, conv or norm);
    reported per layer and scaled to the 18-layer step, labelled so."""
    root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(root, "nanovllm")):
        return None
    for k_, v_ in (("FLA_CHUNK", "0"), ("FLA_RECURRENT", "0"), ("NANOVLLM_FI_NORM", "0")):
        os.environ.setdefault(k_, v_)
    import torch._dynamo
    sys.path.insert(0, root)
    try:
        import nanovllm.models.qwen3_5 as Q
    except Exception as e:  # reported, never fatal
        return {"unavailable": repr(e)[:200]}
    finally:
        sys.path.remove(root)
    torch._dynamo.config.disable = True
    torch.set_num_threads(os.cpu_count() or 1)
    c = C1
    bs, HK, HV, D = c["bs"], c["HK"], c["HV"], c["DK"]
    g_ = torch.Generator().manual_seed(0)
    pool = torch.randn(bs + 1, HV, D, D, generator=g_) * 0.02
    ids = torch.randperm(bs + 1, generator=g_)[:bs]
    q = torch.randn(bs, 1, HK, D, generator=g_).to(torch.bfloat16).repeat_interleave(2, dim=2)
    k = torch.randn(bs, 1, HK, D, generator=g_).to(torch.bfloat16).repeat_interleave(2, dim=2)
    v = torch.randn(bs, 1, HV, D, generator=g_).to(torch.bfloat16)
    g = -torch.rand(bs, 1, HV, generator=g_)
    beta = torch.rand(bs, 1, HV, generator=g_).to(torch.bfloat16)

    def layer():
        out, new_s = Q.recurrent_gated_delta_rule(q, k, v, g, beta, pool[ids])
        pool[ids] = new_s
        return out

    with torch.inference_mode():
        layer()
        n, t0 = 0, time.perf_counter()
        while n < 3 or time.perf_counter() - t0 < budget_s:
            layer()
            n += 1
            if n >= 200:
                break
    dt = (time.perf_counter() - t0) / n
    return {"ms_per_layer_step": round(dt * 1e3, 2),
            "tok_s_18_layer_step": round(bs / (dt * c["layers"]), 2),
            "threads": torch.get_num_threads(),
            "sample": f"{n} config-1 layer steps (bs {bs}, 257-slot pool) of the reference's "
                      "own torch recurrence with its gather / scatter, recurrence only, "
                      "scaled x18 for the 18-layer step"}


def decode_config(world):
    """The config dict of the decode line (both arms print the same one)."""
    c = C1
    return {"workload": "config1 GDN decode stack", "layers": c["layers"],
            "global_batch": c["bs"] * world, "per_gpu_batch": c["bs"],
            "hidden": c["hidden"], "qk_heads": c["HK"], "v_heads": c["HV"],
            "head_dim": c["DK"], "conv_kernel": c["K"], "pool_slots": c["slots"],
            "state_dtype": "fp32", "l2": "inputs larger than L2 (38.7 GB state pool)",
            "cuda_graph": True, "parallelism": f"dp{world} (independent sequences)"}


DECODE_METRIC = "GDN decode tok/s (config 1: 18-layer stack, bs 256)"


def run_reference(args, world, rank):
    """The reference arm: the CPU restatement of the path on the host cores,
    whole 18-layer steps (rank 0 only; other ranks exit without work).  The
    timed step count is capped so the run stays within about a minute."""
    if rank != 0:
        return
    step, sample, threads = cpu_decode_stack()
    t0 = time.perf_counter()
    step()
    est = time.perf_counter() - t0
    for _ in range(min(max(0, args.warmup - 1), 2)):
        step()
    n = max(1, min(args.steps, int(45.0 / max(est, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(n):
        step()
    dt = (time.perf_counter() - t0) / n
    tok_s = C1["bs"] / dt
    line = {"metric": DECODE_METRIC, "impl": "reference",
            "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": args.gpus, "steps": n,
            "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 2), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": decode_config(world),
            "cpu_baseline": {"value": round(tok_s, 2), "unit": "tok/s", "cores": threads,
                             "kind": "port",
                             "sample": f"{sample}; {n} whole steps timed (of {args.steps} "
                                       f"asked), warm-up capped at 3"},
            "e2e": {"value": round(tok_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    ref_torch = reference_torch_recurrence()
    if ref_torch is not None:
        line["reference_torch_recurrence"] = ref_torch
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------


def profile_case(pkg, name):
    """Small cases for `ncu --set full` (a few hundred MB, 3 launches each):
    inputs exceed L2 (126 MB) so DRAM counters mean something."""
    ops = pkg.ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    bs, HK, HV, D, C = 256, 16, 32, 128, 8192
    if name == "recurrent":            # 257-slot pool, 1 layer: 540 MB of state
        pool = torch.randn(bs + 1, HV, D, D, generator=g, device=dev) * 0.02
        mixed = torch.randn(bs, C, generator=g, device=dev).to(torch.bfloat16)
        q = mixed[:, :HK * D].view(bs, HK, D)
        k = mixed[:, HK * D:2 * HK * D].view(bs, HK, D)
        v = mixed[:, 2 * HK * D:].view(bs, HV, D)
        gg = -torch.rand(bs, HV, generator=g, device=dev)
        beta = torch.rand(bs, HV, generator=g, device=dev).to(torch.bfloat16)
        ids = torch.randperm(bs + 1, generator=torch.Generator().manual_seed(0))[:bs].to(dev)
        fn = lambda: ops.recurrent_gdn_inplace(q, k, v, gg, beta, pool, ids)
    elif name == "decode_fused":       # the one-launch decode core, 257-slot pools
        W = C + HV * D + 2 * HV + 64
        pool = torch.randn(bs + 1, HV, D, D, generator=g, device=dev) * 0.02
        cpool = torch.randn(bs + 1, C, 3, generator=g, device=dev).to(torch.bfloat16)
        proj = torch.randn(bs, W, generator=g, device=dev).to(torch.bfloat16)
        w = (torch.rand(C, 4, generator=g, device=dev) - 0.5).to(torch.bfloat16)
        al = torch.rand(HV, device=dev) - 0.5
        dtb = torch.zeros(HV, device=dev)
        nw = torch.ones(D, device=dev, dtype=torch.bfloat16)
        ids = torch.randperm(bs + 1, generator=torch.Generator().manual_seed(0))[:bs].to(dev)
        mixed, z = proj[:, :C], proj[:, C:C + HV * D].view(bs, HV, D)
        b = proj[:, C + HV * D:C + HV * D + HV]
        a = proj[:, C + HV * D + HV:C + HV * D + 2 * HV]
        fn = lambda: ops.decode_fused(mixed, z, b, a, cpool, w, al, dtb, pool, ids, nw)
    elif name == "conv_decode":        # 4096 rows x 8192 channels
        n = 4096
        pool = torch.randn(n + 1, C, 3, generator=g, device=dev).to(torch.bfloat16)
        x = torch.randn(n, C, generator=g, device=dev).to(torch.bfloat16)
        w = torch.randn(C, 4, generator=g, device=dev).to(torch.bfloat16)
        ids = torch.arange(n, device=dev)
        fn = lambda: ops.conv_decode_step(x, pool, ids, w)
    elif name == "chunk_long":         # few long chains: the chain splits into column parts
        HKl, HVl, T = 2, 4, 16384
        lens = [T, T]
        N = sum(lens)
        cu = torch.tensor([0, T, N], dtype=torch.int32, device=dev)
        ids = torch.arange(2, device=dev)
        x = torch.randn(N, (2 * HKl + HVl) * D, generator=g, device=dev).to(torch.bfloat16)
        pool = torch.zeros(2, HVl, D, D, device=dev)
        q = x[:, :HKl * D].view(N, HKl, D)
        k = x[:, HKl * D:2 * HKl * D].view(N, HKl, D)
        v = x[:, 2 * HKl * D:].view(N, HVl, D)
        gg = -torch.rand(N, HVl, generator=g, device=dev)
        beta = torch.rand(N, HVl, generator=g, device=dev).to(torch.bfloat16)
        fn = lambda: ops.chunk_gated_delta_rule_varlen(q, k, v, gg, beta, pool, ids, cu, T)
    elif name in ("conv_varlen", "chunk", "gbeta", "norm"):
        lens = [4096] * 8 + [1000, 3000, 77, 130]
        N = sum(lens)
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
        ids = torch.arange(len(lens), device=dev)
        x = torch.randn(N, C, generator=g, device=dev).to(torch.bfloat16)
        if name == "conv_varlen":      # the layer's call: conv + the gate row, b / a columns
            xb = torch.randn(N, C + 2 * HV, generator=g, device=dev).to(torch.bfloat16)
            pool = torch.randn(len(lens), C, 3, generator=g, device=dev).to(torch.bfloat16)
            w = torch.randn(C, 4, generator=g, device=dev).to(torch.bfloat16)
            al = torch.rand(HV, device=dev)
            fn = lambda: ops.conv_gate_varlen(xb[:, :C], pool, ids, w, cu, xb[:, C:C + HV],
                                              xb[:, C + HV:], al, al)
        elif name == "chunk":
            pool = torch.zeros(len(lens), HV, D, D, device=dev)
            q = x[:, :HK * D].view(N, HK, D)
            k = x[:, HK * D:2 * HK * D].view(N, HK, D)
            v = x[:, 2 * HK * D:].view(N, HV, D)
            gg = -torch.rand(N, HV, generator=g, device=dev)
            beta = torch.rand(N, HV, generator=g, device=dev).to(torch.bfloat16)
            fn = lambda: ops.chunk_gated_delta_rule_varlen(q, k, v, gg, beta, pool, ids, cu,
                                                           max(lens))
        elif name == "gbeta":
            ab = torch.randn(N * 64, 2 * HV, generator=g, device=dev).to(torch.bfloat16)
            al = torch.rand(HV, device=dev)
            fn = lambda: ops.fused_g_beta(ab[:, :HV], ab[:, HV:], al, al)
        else:
            o = torch.randn(N, HV, D, generator=g, device=dev).to(torch.bfloat16)
            z = torch.randn(N, HV, D, generator=g, device=dev).to(torch.bfloat16)
            w = torch.ones(D, device=dev, dtype=torch.bfloat16)
            fn = lambda: ops.rms_norm_gated(o, z, w, 1e-6)
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    print(f"profile case {name}: 3 launches done")


def main():
    args = parse()
    world, rank, local = dist_setup()
    if args.profile_case:
        import __graft_entry__
        profile_case(__graft_entry__.load_package(), args.profile_case)
        return
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            torch.distributed.destroy_process_group()
        return
    import __graft_entry__
    pkg = __graft_entry__.load_package()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peaks = load_peaks()
    c = C1

    stack = DecodeStack(pkg, dev, seed=1234 + rank)
    stack.capture()
    for _ in range(args.warmup):
        stack.replay()
    torch.cuda.synchronize()

    clocks = Clocks(local)
    clocks.start()
    t = time_region(stack.replay, args.steps, world)
    clk = clocks.stop()
    tok = world * c["bs"] * args.steps
    value = tok / t

    # e2e: pinned host input -> HBM, graph, HBM -> pinned host output, per step
    h_in = torch.empty(c["bs"], c["hidden"], dtype=torch.bfloat16).pin_memory()
    h_in.copy_(stack.x.cpu())
    h_out = torch.empty_like(h_in).pin_memory()

    def e2e_step():
        stack.x.copy_(h_in, non_blocking=True)
        stack.replay()
        h_out.copy_(stack.y, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    te = time_region(e2e_step, args.steps, world)
    e2e = {"value": round(tok / te, 1), "unit": "tok/s",
           "h2d_bytes_per_step": h_in.numel() * h_in.element_size(),
           "d2h_bytes_per_step": h_out.numel() * h_out.element_size()}

    roof = decode_kernel_roofline(pkg, stack, peaks, launches=max(2, args.steps // 10))
    state_bytes_step = c["layers"] * 2 * c["bs"] * c["HV"] * c["DK"] * c["DV"] * 4

    line = {"metric": DECODE_METRIC,
            "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(t / args.steps * 1e3, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random weights, inputs and states)",
            "config": decode_config(world),
            "state_gbs": round(world * state_bytes_step * args.steps / t / 1e9, 1),
            "e2e": e2e, "roofline": roof,
            # per layer: the fused decode core (1 launch), or gate, conv step and
            # recurrent with the gated norm fused (3 launches)
            "gpu_launches": (1 if stack.layers[0].fused_decode else 3) * c["layers"] * args.steps,
            "clocks": clk}

    if world > 1:
        del stack.graph
        stack = None
        torch.cuda.empty_cache()
        line["tp_prefill"] = tp_prefill_bench(pkg, dev, world, rank, steps=5)
        line["pp"] = pp_bench(pkg, dev, world, rank, max(args.steps, 400), args.warmup)
        if world == C4["shards"] and not args.no_config4:
            line["config4"] = config4_bench(pkg, dev, world, rank, peaks)
    if rank == 0 and world == 1 and not args.no_prefill:
        try:
            line["prefill"] = prefill_bench(pkg, dev, args.prefill_steps, peaks)
            if not args.no_cpu:
                line["prefill"]["chunk_kernel"]["cpu_baseline"] = cpu_prefill_baseline()
        except Exception as e:  # reported, never hides the headline
            line["prefill"] = {"error": repr(e)[:300]}
    if world == 1 and not args.no_prefill:
        try:
            line["hybrid_1gpu"] = hybrid_single_gpu(pkg, dev, 100, args.warmup)
        except Exception as e:  # reported, never hides the headline
            line["hybrid_1gpu"] = {"error": repr(e)[:300]}
    if world == 1 and not args.no_config4:
        try:
            line["config4"] = config4_bench(pkg, dev, world, rank, peaks)
        except Exception as e:  # reported, never hides the headline
            line["config4"] = {"error": repr(e)[:300]}
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if stack is not None:
        del stack.graph
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
