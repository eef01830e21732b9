"""Worker bodies for the multi-GPU tests (one spawned process per GPU, NCCL).

Each worker raises on a mismatch, which makes its process exit non-zero and
the test fail.  Every rank takes the same collective steps in the same order
and tears its process group down before it exits.
"""
import os
import sys
import types
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def _init(rank, world, port, timeout_s=60):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=timeout_s),
                            device_id=torch.device("cuda", rank))
    import __graft_entry__
    return __graft_entry__.load_package()


def _cfg(hidden, HK, HV, D, K):
    return types.SimpleNamespace(hidden_size=hidden, linear_num_key_heads=HK,
                                 linear_num_value_heads=HV, linear_key_head_dim=D,
                                 linear_value_head_dim=D, linear_conv_kernel_dim=K,
                                 rms_norm_eps=1e-6)


def _build(pkg, cfg, W, dev, parallel=None):
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            m = pkg.layer.Qwen3_5GatedDeltaNet(cfg, parallel=parallel)
    finally:
        torch.set_default_dtype(prev)
    names = dict(in_proj_qkv="in_proj_qkv.weight", in_proj_z="in_proj_z.weight",
                 in_proj_b="in_proj_b.weight", in_proj_a="in_proj_a.weight",
                 conv1d="conv1d.weight", A_log="A_log", dt_bias="dt_bias", norm="norm.weight",
                 out_proj="out_proj.weight")
    with torch.no_grad():
        for k, pname in names.items():
            p = m.get_parameter(pname)
            w = torch.from_numpy(W[k]).to(torch.bfloat16)
            getattr(p, "weight_loader", lambda p_, w_: p_.data.copy_(w_))(p, w)
    return m


def _run(pkg, m, h, ids, lens):
    ctx = pkg.context
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=h.device)
    ctx.set_context(cu, cu, max(lens), max(lens),
                    linear_state_ids=torch.as_tensor(ids, dtype=torch.int64, device=h.device),
                    lens_q=list(lens))
    try:
        with torch.inference_mode():
            return m(None, h)
    finally:
        ctx.reset_context()


def tp_layer_worker(rank, world, port, D, HK=4, HV=8):
    """V-head sharded layer on `world` GPUs (TP group over NCCL): prefill of
    three sequences then decode steps; every rank's all-reduced output equals
    the unsharded layer run on the same GPU, and each rank's state slots hold
    exactly its heads of the unsharded state."""
    pkg = _init(rank, world, port)
    import inputs as I
    P = pkg.parallel
    P.init_parallel_state(rank, world, tp_size=world, pp_size=1)
    dev = torch.device("cuda", rank)
    hidden, K = 512, 4
    cfg = _cfg(hidden, HK, HV, D, K)
    W = I.layer_weights(hidden, HK, D, HV, D, K, seed=21)
    m = _build(pkg, cfg, W, dev)                                     # this rank's shard
    one = types.SimpleNamespace(get_tp_rank=lambda: 0, get_tp_size=lambda: 1,
                                get_tp_group=lambda: None)
    ref = _build(pkg, cfg, W, dev, parallel=one)                     # the whole layer
    slots = 5
    for mm in (m, ref):
        mm.s_cache = torch.zeros(slots, mm.num_v_heads, D, D, device=dev)
        mm.conv_cache = torch.zeros(slots, mm.conv_dim, K - 1, dtype=torch.bfloat16, device=dev)
    ids = [3, 0, 4]
    lens = [70, 1, 23]
    steps = [(I.layer_hidden(sum(lens), hidden, seed=31), lens)]
    steps += [(I.layer_hidden(3, hidden, seed=40 + s), [1, 1, 1]) for s in range(3)]
    for s, (hid, ls) in enumerate(steps):
        h = torch.from_numpy(hid).to(dev).to(torch.bfloat16)
        y = _run(pkg, m, h, ids, ls)
        y_ref = _run(pkg, ref, h, ids, ls)
        d = (y.float() - y_ref.float()).abs().max().item()
        assert d <= 2e-2, f"rank {rank} step {s}: max |tp - single| = {d}"
    hv = slice(rank * m.num_v_heads, (rank + 1) * m.num_v_heads)
    a, b = m.s_cache[ids], ref.s_cache[ids][:, hv]
    rel = ((a - b).norm() / b.norm()).item()
    assert rel <= 1e-2, f"rank {rank}: state rel {rel}"
    pkg.ops.check_status()
    dist.barrier()
    dist.destroy_process_group()


def nccl_handoff_worker(rank, world, port, mode):
    """PipelineHandoff between consecutive GPUs over NCCL on the side stream:
    several steps in flight (double buffers), receiver ordered on events; the
    packed mode on per-boundary process groups, presum on the default group."""
    pkg = _init(rank, world, port)
    P = pkg.parallel
    dev = torch.device("cuda", rank)
    H, N = 2048, 64
    prev, nxt = P.pp_peers(rank, 1, world)
    kw = {}
    if mode == "packed":        # one two-rank group per boundary; presum uses the default group
        groups = P.boundary_groups(world)
        kw = dict(recv_group=groups[rank - 1] if prev is not None else None,
                  send_group=groups[rank] if nxt is not None else None)
    ho = P.PipelineHandoff(H, 256, torch.bfloat16, dev, prev, nxt, mode=mode, **kw)
    g = torch.Generator(device=dev).manual_seed(0)
    steps = []
    for s in range(6):
        h = torch.randn(N + s, H, generator=g, device=dev).to(torch.bfloat16)
        r = torch.randn(N + s, H, generator=g, device=dev).to(torch.bfloat16)
        steps.append((h, r))
    if nxt is not None:
        for h, r in steps:
            ho.send(h, r)
    if prev is not None:
        # receive every step before checking any: each message is copied out and
        # marked consumed(), so a later receive into the same (double) buffer
        # waits only for that copy; an early overwrite would corrupt a copy
        got = []
        for h, r in steps:
            hh, rr = ho.recv(h.shape[0])
            got.append((hh.clone(), None if rr is None else rr.clone()))
            ho.consumed()
        for (h, r), (hh, rr) in zip(steps, got):
            if mode == "packed":
                assert torch.equal(hh, h) and torch.equal(rr, r)
            else:
                assert rr is None
                assert torch.equal(hh, (h.float() + r.float()).to(torch.bfloat16))
    ho.flush()
    torch.cuda.synchronize()
    dist.barrier()
    dist.destroy_process_group()
