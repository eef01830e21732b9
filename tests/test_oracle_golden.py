"""Pin the CPU oracle against golden vectors produced by the reference itself.

The fixtures under tests/golden/ were written by make_golden.py, which runs
the reference's own torch functions and Triton kernels (interpreted) on the
CPU.  Inputs are regenerated here from the same seeds; a digest stored in each
fixture proves they are the same inputs.
"""
import os

import numpy as np
import pytest

import inputs as I
from oracle import gdn_oracle as O


def load(golden_dir, name):
    return dict(np.load(os.path.join(golden_dir, name)))


def bf16_ulp(x):
    """Spacing of bf16 numbers at |x| (8 significant bits)."""
    ax = np.maximum(np.abs(x), 1e-30)
    return 2.0 ** (np.floor(np.log2(ax)) - 7)


def assert_bf16_close(a, b, ulps=1, atol=1e-6):
    a = np.asarray(a, np.float32); b = np.asarray(b, np.float32)
    tol = ulps * bf16_ulp(np.maximum(np.abs(a), np.abs(b))) + atol
    bad = np.abs(a - b) > tol
    assert not bad.any(), f"{bad.sum()} of {bad.size} differ; max |d| {np.abs(a - b).max()}"


def test_round_bf16_matches_torch():
    torch = pytest.importorskip("torch")
    x = I.rng(3).standard_normal(10000).astype(np.float32) * 100
    x[:4] = [0.0, -0.0, 1e-38, 3.4e38]
    ref = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(O.round_bf16(x), ref)


def test_gbeta_golden(golden_dir):
    d = load(golden_dir, "gbeta.npz")
    g, beta = O.fused_g_beta(d["b"], d["a"], d["a_log"], d["dt_bias"], d["mask"])
    np.testing.assert_allclose(g, d["g_mask"], rtol=2e-6, atol=1e-7)
    assert_bf16_close(beta, d["beta_mask"])
    assert np.all(g[~d["mask"]] == 0)
    g, beta = O.fused_g_beta(d["b"], d["a"], d["a_log"], d["dt_bias"], None)
    np.testing.assert_allclose(g, d["g"], rtol=2e-6, atol=1e-7)
    assert_bf16_close(beta, d["beta"])


def test_conv_decode_golden(golden_dir):
    d = load(golden_dir, "conv_decode.npz")
    pool = d["pool_in"].copy()
    y = O.conv_decode_step(d["x"], pool[:, int(d["layer"])], d["ids"], d["w"])
    assert_bf16_close(y, d["y"])
    assert np.array_equal(pool, d["pool_out"])        # state roll is bit-exact


def test_conv_padded_golden(golden_dir):
    d = load(golden_dir, "conv_padded.npz")
    st = d["state_in"].copy()
    y = O.causal_conv_silu_padded(d["x"], st, d["w"], d["endp"])
    assert_bf16_close(y, d["y"])
    assert np.array_equal(st, d["state_out"])


def test_conv_varlen_equals_padded_rows(golden_dir):
    """The varlen restatement gives the padded kernel's values on real rows
    and the same state roll (rows with ENDP == T in the padded fixture)."""
    d = load(golden_dir, "conv_padded.npz")
    T = d["x"].shape[2]
    full = [r for r in range(d["x"].shape[0]) if d["endp"][r] == T]
    for r in full:
        pool = d["state_in"][r][None].copy()
        y = O.causal_conv_silu_varlen(d["x"][r].T, pool, [0], [0, T], d["w"])
        assert_bf16_close(y.T, d["y"][r])
        assert np.array_equal(pool[0], d["state_out"][r])


def test_recurrent_inplace_golden(golden_dir):
    d = load(golden_dir, "recurrent_inplace.npz")
    HK, HV, D = int(d["HK"]), int(d["HV"]), int(d["D"])
    slots, L, bs = 9, 2, 5
    pool = I.recurrent_pool(slots, L, HV, D)
    assert I.digest(pool) == str(d["pool_digest"])
    layer = int(d["layer"])
    kd = HK * D
    for s in range(3):
        mixed, g, beta = I.recurrent_step_inputs(bs, HK, HV, D, s)
        q = mixed[:, :kd].reshape(bs, HK, D)
        k = mixed[:, kd:2 * kd].reshape(bs, HK, D)
        v = mixed[:, 2 * kd:].reshape(bs, HV, D)
        out = O.recurrent_inplace(q, k, v, g, beta, pool[:, layer], d["ids"])
        assert_bf16_close(O.round_bf16(out), d[f"out{s}"], ulps=1, atol=1e-5)
    np.testing.assert_allclose(pool[d["ids"], layer], d["rows_out"], rtol=1e-5, atol=1e-6)


def test_chunk_and_recurrent_c0_golden(golden_dir):
    d = load(golden_dir, "chunk_c0.npz")
    c = I.C0
    lens = c["lens"]
    q, k, v, g, beta = I.core_inputs(sum(lens), c["HK"], c["DK"], c["HV"], c["DV"], seed=0)
    init = I.chunk_init_state(len(lens), c["HV"], c["DK"], c["DV"])
    assert I.digest(q, k, v, g, beta, init) == str(d["digest"])
    pool = init.copy()
    out = O.chunk_prefill_varlen(q, k, v, g, beta, pool, np.arange(len(lens)),
                                 I.cu_from_lens(lens))
    np.testing.assert_allclose(out, d["out"], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(pool, d["state"], rtol=1e-4, atol=2e-6)
    S = d["state"].copy()
    for s in range(c["n_decode"]):
        dq, dk, dv, dg, db = I.core_inputs(len(lens), c["HK"], c["DK"], c["HV"], c["DV"],
                                           seed=1000 + s)
        o, S = O.recurrent_step(dq, dk, dv, dg, db, S)
        np.testing.assert_allclose(o, d["dec_out"][s], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(S, d["dec_state"], rtol=1e-4, atol=2e-6)


def test_chunk_equals_token_recurrence():
    """Chunked and token-by-token forms are the same recurrence (fp64)."""
    q, k, v, g, beta = I.core_inputs(150, 2, 16, 4, 16, seed=5)
    o_c, S_c = O.chunk_gated_delta_rule(q, k, v, g, beta, None, 64, np.float64)
    S = np.zeros((1, 4, 16, 16))
    outs = []
    for t in range(150):
        o, S = O.recurrent_step(q[t:t + 1], k[t:t + 1], v[t:t + 1], g[t:t + 1],
                                beta[t:t + 1], S, np.float64)
        outs.append(o[0])
    np.testing.assert_allclose(o_c, np.stack(outs), rtol=1e-9, atol=1e-11)
    np.testing.assert_allclose(S_c, S[0], rtol=1e-9, atol=1e-11)


def test_rms_gated_golden(golden_dir):
    d = load(golden_dir, "rms_gated.npz")
    y = O.rms_norm_gated(d["x"], d["z"], d["w"], 1e-6)
    assert_bf16_close(y, d["y"])


@pytest.mark.parametrize("dtype_name", ["fp32", "bf16"])
def test_layer_c0_golden(golden_dir, dtype_name):
    d = load(golden_dir, f"layer_c0_{dtype_name}.npz")
    c = I.C0
    act = O.round_bf16 if dtype_name == "bf16" else None
    lens = list(c["lens"])
    W = I.layer_weights(c["hidden"], c["HK"], c["DK"], c["HV"], c["DV"], c["K"])
    conv_dim = 2 * c["HK"] * c["DK"] + c["HV"] * c["DV"]
    s_pool, conv_pool = I.layer_pools(7, c["HV"], c["DK"], c["DV"], conv_dim, c["K"])
    hid = I.layer_hidden(sum(lens), c["hidden"])
    assert I.digest(hid, s_pool, conv_pool) == str(d["digest"])
    ids = d["ids"]
    s_pool[ids] = 0
    conv_pool[ids] = 0
    y = O.gdn_layer_forward(hid, W, conv_pool[:, 0], s_pool[:, 0], ids, lens,
                            c["HK"], c["DK"], c["HV"], c["DV"], c["eps"], act)
    if act is None:
        np.testing.assert_allclose(y, d["y_prefill"], rtol=1e-3, atol=1e-5)
    else:
        assert np.abs(y - d["y_prefill"]).max() <= 2e-2
        assert np.mean(np.abs(y - d["y_prefill"])) < 1e-3
    for s in range(c["n_decode"]):
        h = I.layer_hidden(len(lens), c["hidden"], seed=200 + s)
        y = O.gdn_layer_forward(h, W, conv_pool[:, 0], s_pool[:, 0], ids, [1] * len(lens),
                                c["HK"], c["DK"], c["HV"], c["DV"], c["eps"], act)
        if act is None:
            np.testing.assert_allclose(y, d["y_decode"][s], rtol=1e-3, atol=1e-5)
        else:
            assert np.abs(y - d["y_decode"][s]).max() <= 2e-2
    if act is None:
        np.testing.assert_allclose(s_pool[ids], d["s_rows"], rtol=1e-3, atol=1e-6)
        np.testing.assert_allclose(conv_pool[ids], d["conv_rows"], rtol=1e-5, atol=1e-6)
    else:
        num = np.linalg.norm(s_pool[ids] - d["s_rows"])
        assert num / np.linalg.norm(d["s_rows"]) <= 1e-2
        # the conv state holds raw projection values: bf16, one rounding apart
        assert_bf16_close(conv_pool[ids], d["conv_rows"], ulps=1)
