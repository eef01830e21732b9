"""Worker bodies for the world_size-2 gloo tests (spawned processes).

Each worker returns nothing; failures raise, which makes the spawned process
exit non-zero and the test fail.
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


def _init(rank, world, port, timeout_s=30):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=timedelta(seconds=timeout_s))
    import __graft_entry__
    return __graft_entry__.load_package()


def gemma_add_rms(x, residual, w, eps=1e-6):
    """The torch-path fused add + Gemma RMSNorm of the reference
    (nanovllm/models/qwen3_5.py:109-118): residual = bf16(x + r), normed from it."""
    residual = (x.float() + residual.float()).to(x.dtype)
    xf = residual.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * (1.0 + w.float())).to(x.dtype), residual


def gemma_rms(x, w, eps=1e-6):
    """qwen3_5.py:99-105 (residual=None path of the decoder layer)."""
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * (1.0 + w.float())).to(x.dtype)


def handoff_worker(rank, world, port, mode):
    pkg = _init(rank, world, port)
    P = pkg.parallel
    H, N = 64, 10
    prev, nxt = P.pp_peers(rank, 1, world)
    ho = P.PipelineHandoff(H, 32, torch.bfloat16, torch.device("cpu"), prev, nxt, mode=mode)
    g = torch.Generator().manual_seed(0)
    steps = []
    for s in range(4):   # several steps in flight exercise the double buffering
        h = torch.randn(N + s, H, generator=g).to(torch.bfloat16)
        r = torch.randn(N + s, H, generator=g).to(torch.bfloat16)
        steps.append((h, r))
    w = torch.randn(H, generator=g).to(torch.bfloat16) * 0.1
    if rank == 0:
        for h, r in steps:
            ho.send(h, r)
        ho.flush()
    else:
        for h, r in steps:
            hh, rr = ho.recv(h.shape[0])
            if mode == "packed":
                assert torch.equal(hh, h) and torch.equal(rr, r)
                got_x, got_r = gemma_add_rms(hh, rr, w)
            else:
                assert rr is None
                # the receiver's first add-norm with residual=None on the sum
                got_x, got_r = gemma_rms(hh, w), hh
            ref_x, ref_r = gemma_add_rms(h, r, w)
            assert torch.equal(got_r, ref_r)
            assert torch.equal(got_x, ref_x)
    dist.barrier()
    dist.destroy_process_group()


def handoff_chain_worker(rank, world, port):
    """A pipeline of `world` stages on one two-rank process group per boundary
    (boundary_groups): every stage but the first receives, adds its rank to the
    hidden part and passes the pair on, with several steps in flight and each
    received message copied out and marked consumed(); the last stage checks
    that every step arrived intact through the middle stages."""
    pkg = _init(rank, world, port)
    P = pkg.parallel
    H, N, steps = 32, 6, 5
    prev, nxt = P.pp_peers(rank, 1, world)
    groups = P.boundary_groups(world)
    ho = P.PipelineHandoff(H, 16, torch.float32, torch.device("cpu"), prev, nxt, mode="packed",
                           recv_group=groups[rank - 1] if prev is not None else None,
                           send_group=groups[rank] if nxt is not None else None)
    g = torch.Generator().manual_seed(0)
    data = [(torch.randn(N, H, generator=g), torch.randn(N, H, generator=g))
            for _ in range(steps)]
    got = []
    for s in range(steps):
        if prev is None:
            h, r = data[s]
        else:
            hh, rr = ho.recv(N)
            h, r = hh.clone() + rank, rr.clone()
            ho.consumed()
        if nxt is not None:
            ho.send(h, r)
        else:
            got.append((h, r))
    ho.flush()
    if nxt is None:
        for (h, r), (h0, r0) in zip(got, data):
            want = h0
            for stage in range(1, world):      # the stages' additions, in their order
                want = want + stage
            assert torch.equal(h, want) and torch.equal(r, r0)
    dist.barrier()
    dist.destroy_process_group()


def handoff_peer_dies_worker(rank, world, port):
    """Rank 0 leaves before sending; rank 1's receive must end with an error
    (never hang) within the short process-group timeout."""
    pkg = _init(rank, world, port, timeout_s=5)
    P = pkg.parallel
    if rank == 0:
        os._exit(0)                       # the peer disappears between steps
    prev, nxt = P.pp_peers(rank, 1, world)
    ho = P.PipelineHandoff(16, 8, torch.bfloat16, torch.device("cpu"), prev, nxt)
    try:
        ho.recv(4)
    except Exception:
        os._exit(0)                       # detected on the host
    os._exit(3)                           # received data from a dead peer: wrong


def row_parallel_worker(rank, world, port):
    pkg = _init(rank, world, port)
    P = pkg.parallel
    g = torch.Generator().manual_seed(1)
    W = torch.randn(24, 32, generator=g)
    x = torch.randn(5, 32, generator=g)
    m = P.RowParallelLinear(32, 24, rank, world, tp_group=None)
    m.weight.weight_loader(m.weight, W)
    y = m(x[:, rank * 16:(rank + 1) * 16])
    torch.testing.assert_close(y, x @ W.T, rtol=1e-5, atol=1e-5)
    dist.destroy_process_group()


def head_sharded_layer_worker(rank, world, port):
    """Each rank loads its V-head shard of a full config-0 layer through the
    layer's own weight loaders, runs the oracle core on its shard, and the
    partial out_proj outputs all-reduce to the single-process layer output."""
    pkg = _init(rank, world, port)
    import inputs as I
    from oracle import gdn_oracle as O
    c = I.C0
    cfg = types.SimpleNamespace(hidden_size=c["hidden"], linear_num_key_heads=c["HK"],
                                linear_num_value_heads=c["HV"], linear_key_head_dim=c["DK"],
                                linear_value_head_dim=c["DV"], linear_conv_kernel_dim=c["K"],
                                rms_norm_eps=c["eps"])
    Pv = types.SimpleNamespace(get_tp_rank=lambda: rank, get_tp_size=lambda: world,
                               get_tp_group=lambda: None)
    m = pkg.layer.Qwen3_5GatedDeltaNet(cfg, parallel=Pv)
    W = I.layer_weights(c["hidden"], c["HK"], c["DK"], c["HV"], c["DV"], c["K"])
    names = dict(in_proj_qkv="in_proj_qkv.weight", in_proj_z="in_proj_z.weight",
                 in_proj_b="in_proj_b.weight", in_proj_a="in_proj_a.weight",
                 conv1d="conv1d.weight", A_log="A_log", dt_bias="dt_bias", norm="norm.weight",
                 out_proj="out_proj.weight")
    with torch.no_grad():
        for kname, pname in names.items():
            p = m.get_parameter(pname)
            getattr(p, "weight_loader", lambda p_, w_: p_.data.copy_(w_))(p, torch.from_numpy(W[kname]))
    shard = {k: m.get_parameter(pn).detach().numpy().copy() for k, pn in names.items()}
    shard["A_log"] = shard["A_log"][m._v_head_slice]
    shard["dt_bias"] = shard["dt_bias"][m._v_head_slice]
    HK, HV = m.num_k_heads, m.num_v_heads
    lens = [40, 1, 23]
    N = sum(lens)
    hid = I.layer_hidden(N, c["hidden"], seed=9)
    conv_dim = m.conv_dim
    s_pool = np.zeros((4, HV, c["DK"], c["DV"]), np.float32)
    conv_pool = np.zeros((4, conv_dim, c["K"] - 1), np.float32)
    ids = np.array([2, 0, 3])
    # this rank's partial: projections of its shard, core, partial out_proj (no round to
    # bf16: fp32 model, as config 0)
    part = O.gdn_layer_forward(hid, shard, conv_pool, s_pool, ids, lens, HK, c["DK"], HV,
                               c["DV"], c["eps"], None)
    t = torch.from_numpy(part.copy())
    dist.all_reduce(t)
    full_s = np.zeros((4, c["HV"], c["DK"], c["DV"]), np.float32)
    full_c = np.zeros((4, 2 * c["HK"] * c["DK"] + c["HV"] * c["DV"], c["K"] - 1), np.float32)
    ref = O.gdn_layer_forward(hid, W, full_c, full_s, ids, lens, c["HK"], c["DK"], c["HV"],
                              c["DV"], c["eps"], None)
    np.testing.assert_allclose(t.numpy(), ref, rtol=2e-4, atol=2e-5)
    # the rank's state rows are exactly its heads of the full state
    hv = slice(rank * HV, (rank + 1) * HV)
    np.testing.assert_allclose(s_pool, full_s[:, hv], rtol=2e-4, atol=1e-6)
    dist.destroy_process_group()
