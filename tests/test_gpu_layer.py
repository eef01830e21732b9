"""The drop-in Qwen3_5GatedDeltaNet on the GPU: the reference's own layer
output (golden, config 0, bf16) through forward(positions, hidden_states),
mixed decode/prefill batches, CUDA-graph decode with dummy-slot pad rows,
and the module swap into a reference-shaped namespace."""
import os
import types

import numpy as np
import pytest
import torch

import inputs as I

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def L(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    return pkg


def cfg_c0():
    c = I.C0
    return types.SimpleNamespace(hidden_size=c["hidden"], linear_num_key_heads=c["HK"],
                                 linear_num_value_heads=c["HV"], linear_key_head_dim=c["DK"],
                                 linear_value_head_dim=c["DV"], linear_conv_kernel_dim=c["K"],
                                 rms_norm_eps=c["eps"])


def build_layer(pkg, cfg, weights):
    prev_dtype = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(DEV):
            m = pkg.layer.Qwen3_5GatedDeltaNet(cfg)
    finally:
        torch.set_default_dtype(prev_dtype)
    names = dict(in_proj_qkv="in_proj_qkv.weight", in_proj_z="in_proj_z.weight",
                 in_proj_b="in_proj_b.weight", in_proj_a="in_proj_a.weight",
                 conv1d="conv1d.weight", A_log="A_log", dt_bias="dt_bias", norm="norm.weight",
                 out_proj="out_proj.weight")
    with torch.no_grad():
        for k, pname in names.items():
            p = m.get_parameter(pname)
            w = torch.from_numpy(weights[k]).to(torch.bfloat16)
            getattr(p, "weight_loader", lambda p_, w_: p_.data.copy_(w_))(p, w)
    return m


def run(pkg, m, hidden_np, ids, lens):
    ctx = pkg.context
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=DEV)
    ctx.set_context(cu, cu, max(lens), max(lens),
                    linear_state_ids=torch.as_tensor(ids, dtype=torch.int64, device=DEV),
                    lens_q=list(lens))
    try:
        with torch.inference_mode():
            h = torch.from_numpy(np.ascontiguousarray(hidden_np)).to(DEV).to(torch.bfloat16)
            return m(None, h)
    finally:
        ctx.reset_context()


def test_layer_c0_bf16_golden(L, golden_dir):
    """Prefill of 4 sequences then 16 decode steps vs the reference layer."""
    d = dict(np.load(os.path.join(golden_dir, "layer_c0_bf16.npz")))
    c = I.C0
    W = I.layer_weights(c["hidden"], c["HK"], c["DK"], c["HV"], c["DV"], c["K"])
    m = build_layer(L, cfg_c0(), W)
    s_np, conv_np = I.layer_pools(7, c["HV"], c["DK"], c["DV"], m.conv_dim, c["K"])
    hid = I.layer_hidden(sum(c["lens"]), c["hidden"])
    assert I.digest(hid, s_np, conv_np) == str(d["digest"])
    ids = d["ids"]
    s_pool = torch.from_numpy(s_np).to(DEV)
    conv_pool = torch.from_numpy(conv_np).to(DEV).to(torch.bfloat16)
    s_pool[torch.from_numpy(ids).to(DEV)] = 0          # fresh-prefill zeroing
    conv_pool[torch.from_numpy(ids).to(DEV)] = 0
    m.s_cache, m.conv_cache = s_pool[:, 0], conv_pool[:, 0]
    y = run(L, m, hid, ids, list(c["lens"])).float().cpu().numpy()
    assert np.abs(y - d["y_prefill"]).max() <= 2e-2
    for s in range(c["n_decode"]):
        h = I.layer_hidden(4, c["hidden"], seed=200 + s)
        y = run(L, m, h, ids, [1, 1, 1, 1]).float().cpu().numpy()
        assert np.abs(y - d["y_decode"][s]).max() <= 2e-2, f"decode step {s}"
    s_out = s_pool.cpu().numpy()
    rel = np.linalg.norm(s_out[ids] - d["s_rows"]) / np.linalg.norm(d["s_rows"])
    assert rel <= 2e-2     # bf16 projections: one rounding apart from the reference's GEMMs
    conv_out = conv_pool.float().cpu().numpy()
    diff = np.abs(conv_out[ids] - d["conv_rows"])
    assert diff.max() <= 2 ** -6 * np.abs(d["conv_rows"]).max()
    untouched = np.setdiff1d(np.arange(7), ids)
    assert np.array_equal(s_out[untouched], s_np[untouched])
    assert np.array_equal(conv_out[untouched], conv_np[untouched])
    L.ops.check_status()


def test_layer_mixed_batch_equals_split(L):
    """A mixed step (decode rows first, then prefill chunks) equals running the
    decode rows and the prefill rows as two separate steps."""
    c = I.C0
    W = I.layer_weights(c["hidden"], c["HK"], c["DK"], c["HV"], c["DV"], c["K"], seed=3)
    m = build_layer(L, cfg_c0(), W)
    pools = []
    for _ in range(2):
        s = torch.zeros(6, 1, c["HV"], c["DK"], c["DV"], device=DEV)
        cv = torch.zeros(6, 1, m.conv_dim, c["K"] - 1, dtype=torch.bfloat16, device=DEV)
        pools.append((s, cv))
    warm = I.layer_hidden(90, c["hidden"], seed=4)
    mixed_h = I.layer_hidden(2 + 50 + 70, c["hidden"], seed=5)
    outs = []
    for s, cv in pools:
        m.s_cache, m.conv_cache = s[:, 0], cv[:, 0]
        run(L, m, warm, [0, 1], [40, 50])                       # two sequences prefill
        outs.append(s)
    m.s_cache, m.conv_cache = pools[0][0][:, 0], pools[0][1][:, 0]
    y_mixed = run(L, m, mixed_h, [0, 1, 2, 3], [1, 1, 50, 70])
    m.s_cache, m.conv_cache = pools[1][0][:, 0], pools[1][1][:, 0]
    y_a = run(L, m, mixed_h[:2], [0, 1], [1, 1])
    y_b = run(L, m, mixed_h[2:], [2, 3], [50, 70])
    # cuBLAS may pick different kernels for different row counts, so the two
    # routes agree to bf16 rounding, not bit for bit
    assert (y_mixed.float() - torch.cat([y_a, y_b]).float()).abs().max().item() <= 2e-2
    s0, s1 = pools[0][0], pools[1][0]
    assert ((s0 - s1).norm() / s1.norm()).item() <= 1e-2


def test_layer_cuda_graph_decode_with_dummy_slot(L):
    """Decode captured in a CUDA graph at bs=8 with 5 pad rows on the dummy
    slot equals eager decode of the 3 real rows; no other slot moves."""
    c = I.C0
    W = I.layer_weights(c["hidden"], c["HK"], c["DK"], c["HV"], c["DV"], c["K"], seed=6)
    m = build_layer(L, cfg_c0(), W)
    nslots = 10
    dummy = nslots
    s = (torch.randn(nslots + 1, 1, c["HV"], c["DK"], c["DV"], device=DEV) * 0.02)
    cv = torch.randn(nslots + 1, 1, m.conv_dim, c["K"] - 1, device=DEV).to(torch.bfloat16)
    s2, cv2 = s.clone(), cv.clone()
    s_init, cv_init = s.clone(), cv.clone()
    real = [7, 2, 4]
    ctx = L.context
    gb = 8
    ids_buf = torch.full((gb,), dummy, dtype=torch.int64, device=DEV)
    h_buf = torch.zeros(gb, c["hidden"], dtype=torch.bfloat16, device=DEV)
    cu = torch.arange(gb + 1, dtype=torch.int32, device=DEV)
    m.s_cache, m.conv_cache = s[:, 0], cv[:, 0]
    ctx.set_context(cu, cu, 1, 1, linear_state_ids=ids_buf)
    with torch.inference_mode():
        for _ in range(2):                                   # warm-up (allocations)
            m(None, h_buf)
        s.copy_(s2); cv.copy_(cv2)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            y_buf = m(None, h_buf)
    ctx.reset_context()
    for step in range(3):
        h = torch.from_numpy(I.layer_hidden(3, c["hidden"], seed=300 + step)).to(DEV)
        ids_buf.fill_(dummy)
        ids_buf[:3] = torch.tensor(real, device=DEV)
        h_buf.zero_()
        h_buf[:3] = h.to(torch.bfloat16)
        graph.replay()
        # eager twin on a copy of the pools, same shapes (pad rows included)
        m.s_cache, m.conv_cache = s2[:, 0], cv2[:, 0]
        y_eager = run(L, m, h_buf.float().cpu().numpy(), ids_buf.cpu().numpy(), [1] * gb)
        m.s_cache, m.conv_cache = s[:, 0], cv[:, 0]
        torch.cuda.synchronize()
        assert torch.equal(y_buf[:3], y_eager[:3])
    # pad rows all hit the dummy slot concurrently, so only real slots compare
    assert torch.equal(s[:nslots], s2[:nslots]) and torch.equal(cv[:nslots], cv2[:nslots])
    keep = [i for i in range(nslots) if i not in real]
    assert torch.equal(s[keep], s_init[keep]) and torch.equal(cv[keep], cv_init[keep])
    assert not torch.equal(s[real], s_init[real])
    del graph


def test_install_swaps_the_class(L):
    """install() replaces the class in a reference-shaped module namespace and
    the swapped class reads that namespace's parallel state and context."""
    Q = types.SimpleNamespace(Qwen3_5GatedDeltaNet=object)
    P = types.SimpleNamespace(get_tp_rank=lambda: 0, get_tp_size=lambda: 1,
                              get_tp_group=lambda: None)
    seen = {}

    def get_context():
        seen["called"] = True
        return L.context.get_context()

    Cx = types.SimpleNamespace(get_context=get_context)
    prev = L.layer.install(Q, P, Cx)
    assert prev is object
    cls = Q.Qwen3_5GatedDeltaNet
    assert issubclass(cls, L.layer.Qwen3_5GatedDeltaNet)
    c = I.C0
    W = I.layer_weights(c["hidden"], c["HK"], c["DK"], c["HV"], c["DV"], c["K"], seed=8)
    prev_dtype = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(DEV):
            m = cls(cfg_c0())
    finally:
        torch.set_default_dtype(prev_dtype)
    m.s_cache = torch.zeros(3, c["HV"], c["DK"], c["DV"], device=DEV)
    m.conv_cache = torch.zeros(3, m.conv_dim, 3, dtype=torch.bfloat16, device=DEV)
    run(L, m, I.layer_hidden(10, c["hidden"]), [1], [10])
    assert seen.get("called")
    L.layer.uninstall(prev, Q)
    assert Q.Qwen3_5GatedDeltaNet is object


def test_layer_bad_slot_raises_at_the_next_call(L):
    """A bad slot id in one forward call is flagged on the device, published
    to pinned host memory after the call by the device's publishing layer (this
    one), and raised (IndexError) by the next forward call once the first has
    run; the call after that is clean.  A second layer neither publishes nor
    takes the role while the first is alive."""
    c = I.C0
    W = I.layer_weights(c["hidden"], c["HK"], c["DK"], c["HV"], c["DV"], c["K"], seed=12)
    L.ops.reset_status_publisher()
    m = build_layer(L, cfg_c0(), W)
    other = build_layer(L, cfg_c0(), W)
    assert L.ops.is_status_publisher(m, DEV) and not L.ops.is_status_publisher(other, DEV)
    m.s_cache = torch.zeros(4, c["HV"], c["DK"], c["DV"], device=DEV)
    m.conv_cache = torch.zeros(4, m.conv_dim, c["K"] - 1, dtype=torch.bfloat16, device=DEV)
    L.ops.check_status()
    run(L, m, I.layer_hidden(2, c["hidden"], seed=1), [0, 9], [1, 1])    # slot 9 is outside
    torch.cuda.synchronize()            # the step has run (an engine syncs to sample)
    with pytest.raises(IndexError):
        run(L, m, I.layer_hidden(2, c["hidden"], seed=2), [0, 1], [1, 1])
    run(L, m, I.layer_hidden(2, c["hidden"], seed=3), [0, 1], [1, 1])
    torch.cuda.synchronize()
    assert L.ops.poll_status() == 0
    L.ops.check_status()


def test_layer_nvtx_ranges_leave_results_unchanged(L):
    """With the NVTX ranges on, a prefill + decode gives the same bits."""
    c = I.C0
    W = I.layer_weights(c["hidden"], c["HK"], c["DK"], c["HV"], c["DV"], c["K"], seed=14)
    outs = []
    for nv in (False, True):
        m = build_layer(L, cfg_c0(), W)
        m.nvtx = nv
        m.s_cache = torch.zeros(4, c["HV"], c["DK"], c["DV"], device=DEV)
        m.conv_cache = torch.zeros(4, m.conv_dim, c["K"] - 1, dtype=torch.bfloat16, device=DEV)
        y0 = run(L, m, I.layer_hidden(70, c["hidden"], seed=5), [2, 0], [40, 30])
        y1 = run(L, m, I.layer_hidden(2, c["hidden"], seed=6), [2, 0], [1, 1])
        outs.append((y0, y1, m.s_cache.clone()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


def test_debug_checks_raise_before_any_launch(L):
    """With the host-side checks on, a slot id outside the pool raises
    IndexError and a repeated one ValueError in the call itself, before any
    GDN kernel launches, so the device status word stays clear; repeats of the
    pool's last slot (the dummy slot of graph pad rows) pass."""
    c = I.C0
    W = I.layer_weights(c["hidden"], c["HK"], c["DK"], c["HV"], c["DV"], c["K"], seed=15)
    m = build_layer(L, cfg_c0(), W)
    m.s_cache = torch.zeros(4, c["HV"], c["DK"], c["DV"], device=DEV)
    m.conv_cache = torch.zeros(4, m.conv_dim, c["K"] - 1, dtype=torch.bfloat16, device=DEV)
    L.ops.check_status()
    L.ops.set_debug_checks(True)
    try:
        with pytest.raises(IndexError):
            run(L, m, I.layer_hidden(2, c["hidden"], seed=1), [0, 9], [1, 1])
        with pytest.raises(ValueError):
            run(L, m, I.layer_hidden(5, c["hidden"], seed=2), [1, 1], [2, 3])   # prefill rows
        run(L, m, I.layer_hidden(3, c["hidden"], seed=3), [0, 3, 3], [1, 1, 1])   # dummy slot 3
        torch.cuda.synchronize()
        assert L.ops.check_status() == 0
    finally:
        L.ops.set_debug_checks(False)
