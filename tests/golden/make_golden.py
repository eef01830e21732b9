"""Generate the GDN golden vectors from the reference implementation itself.

Run in a container where the reference checkout is present (its path is the
first argument, or $GDN_REFERENCE_ROOT); it is NOT needed to run the tests.
The reference's own functions and Triton kernels are imported from that
checkout and executed on the CPU (Triton through its interpreter), with the
environment switches that force its pure-torch paths:

    FLA_CHUNK=0 FLA_RECURRENT=0 NANOVLLM_FI_NORM=0 TORCHDYNAMO_DISABLE=1
    TRITON_INTERPRET=1 PYTHONDONTWRITEBYTECODE=1

Outputs are written as compressed .npz files next to this script.  Inputs
come from ``inputs.py`` (seeded numpy); each fixture stores the digest of its
inputs so the tests can prove they regenerate the same ones.

    python tests/golden/make_golden.py <reference-root>
"""
from __future__ import annotations

import os
import sys

for _k, _v in dict(FLA_CHUNK="0", FLA_RECURRENT="0", NANOVLLM_FI_NORM="0",
                   TORCHDYNAMO_DISABLE="1", TRITON_INTERPRET="1",
                   PYTHONDONTWRITEBYTECODE="1").items():
    os.environ[_k] = _v

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs as I  # noqa: E402


def _ref_root():
    if len(sys.argv) > 1:
        return sys.argv[1]
    return os.environ["GDN_REFERENCE_ROOT"]


def t(x, dtype=torch.float32):
    """A torch copy of x (never aliasing the numpy buffer: several kernels
    under test update their state arguments in place)."""
    return torch.from_numpy(np.array(x, copy=True)).to(dtype)


def n(x):
    return x.detach().to(torch.float32).numpy().copy()


def bf(x):
    """float32 array rounded through bf16 (what the fixture stores)."""
    return n(t(x, torch.bfloat16))


def save(name, **arrays):
    path = os.path.join(HERE, name)
    np.savez_compressed(path, **arrays)
    print(f"wrote {name}: " + ", ".join(f"{k}{tuple(v.shape)}" for k, v in arrays.items()
                                         if hasattr(v, "shape")))


def main():
    sys.path.insert(0, _ref_root())
    import nanovllm.models.qwen3_5 as Q
    from nanovllm.utils.context import set_context, reset_context

    # ---------------- (b) fused g / beta (Triton kernel, interpreted) -----
    r = I.rng(10)
    a = bf(r.standard_normal((3, 5, 8)).astype(np.float32) * 4)
    a[0, 0, :] = 30.0                      # softplus threshold branch (z > 20)
    b = bf(r.standard_normal((3, 5, 8)).astype(np.float32) * 3)
    a_log = bf(r.uniform(-1, 1, 8).astype(np.float32))
    dt_bias = bf(r.standard_normal(8).astype(np.float32))
    mask = np.arange(5)[None, :] < np.array([5, 2, 0])[:, None]
    g_m, beta_m = Q.fused_g_beta(t(b, torch.bfloat16), t(a, torch.bfloat16),
                                 t(a_log, torch.bfloat16), t(dt_bias, torch.bfloat16),
                                 torch.from_numpy(mask))
    g_n, beta_n = Q.fused_g_beta(t(b, torch.bfloat16), t(a, torch.bfloat16),
                                 t(a_log, torch.bfloat16), t(dt_bias, torch.bfloat16), None)
    save("gbeta.npz", a=a, b=b, a_log=a_log, dt_bias=dt_bias, mask=mask,
         g_mask=n(g_m), beta_mask=n(beta_m), g=n(g_n), beta=n(beta_n))

    # ---------------- (a) conv decode step (in place by slot) -------------
    r = I.rng(11)
    nseq, C, K, slots, L = 5, 96, 4, 9, 2
    x = bf(r.standard_normal((nseq, C)).astype(np.float32))
    pool = bf(r.standard_normal((slots, L, C, K - 1)).astype(np.float32))
    w = bf(r.uniform(-0.6, 0.6, (C, K)).astype(np.float32))
    ids = np.array([7, 2, 5, 0, 8], np.int64)
    pool_t = t(pool, torch.bfloat16)
    y = Q.conv_decode_step(t(x, torch.bfloat16), pool_t[:, 1], torch.from_numpy(ids),
                           t(w, torch.bfloat16))
    save("conv_decode.npz", x=x, pool_in=pool, w=w, ids=ids, layer=np.int64(1),
         y=n(y), pool_out=n(pool_t))

    # ---------------- (a) padded causal conv with ENDP writeback ----------
    r = I.rng(12)
    nrow, C, T = 4, 72, 70
    x = bf(r.standard_normal((nrow, C, T)).astype(np.float32))
    st = bf(r.standard_normal((nrow, C, K - 1)).astype(np.float32))
    w = bf(r.uniform(-0.6, 0.6, (C, K)).astype(np.float32))
    endp = np.array([70, 10, -1, 1], np.int32)
    st_t = t(st, torch.bfloat16)
    y = Q.causal_conv_silu(t(x, torch.bfloat16), st_t, t(w, torch.bfloat16),
                           torch.from_numpy(endp))
    save("conv_padded.npz", x=x, state_in=st, w=w, endp=endp, y=n(y), state_out=n(st_t))

    # ---------------- (d) in-place recurrent decode (Triton kernel) -------
    r = I.rng(13)
    bs, HK, HV, D, slots, L = 5, 2, 4, 64, 9, 2
    kd, vd = HK * D, HV * D
    conv_dim = 2 * kd + vd
    pool = I.recurrent_pool(slots, L, HV, D)
    ids = np.array([3, 8, 0, 6, 1], np.int64)
    pool_t = t(pool)
    steps = []
    for s in range(3):
        mixed, g, beta = I.recurrent_step_inputs(bs, HK, HV, D, s)
        mt = t(mixed, torch.bfloat16)
        qv = mt[:, :kd].reshape(bs, 1, HK, D).repeat_interleave(HV // HK, dim=2)
        kv = mt[:, kd:2 * kd].reshape(bs, 1, HK, D).repeat_interleave(HV // HK, dim=2)
        vv = mt[:, 2 * kd:].view(bs, 1, HV, D)
        o = Q.recurrent_gdn_inplace(qv, kv, vv, t(g).view(bs, 1, HV),
                                    t(beta, torch.bfloat16).view(bs, 1, HV),
                                    pool_t[:, 1], torch.from_numpy(ids))
        steps.append(dict(mixed=mixed, g=g, beta=beta, out=n(o).reshape(bs, HV, D)))
    pool_out = n(pool_t)
    untouched = np.ones(slots, bool); untouched[ids] = False
    assert np.array_equal(pool_out[untouched], pool[untouched])
    assert np.array_equal(pool_out[:, 0], pool[:, 0])
    save("recurrent_inplace.npz", ids=ids, layer=np.int64(1),
         HK=np.int64(HK), HV=np.int64(HV), D=np.int64(D),
         pool_digest=np.array(I.digest(pool)),
         **{f"{k}{i}": v for i, s in enumerate(steps) for k, v in s.items()
            if k in ("out",)},
         rows_out=pool_out[ids, 1])

    # ---------------- (c)+(d) chunk prefill then recurrent, config 0, fp32 -
    c = I.C0
    lens = c["lens"]
    Ntok = sum(lens)
    q, k, v, g, beta = I.core_inputs(Ntok, c["HK"], c["DK"], c["HV"], c["DV"], seed=0)
    rep = c["HV"] // c["HK"]
    cu = I.cu_from_lens(lens)
    init = I.chunk_init_state(len(lens), c["HV"], c["DK"], c["DV"])
    outs, finals = [], []
    for i in range(len(lens)):
        a0, a1 = cu[i], cu[i + 1]
        o, S = Q._torch_chunk_gated_delta_rule(
            t(q[a0:a1][None]).repeat_interleave(rep, dim=2),
            t(k[a0:a1][None]).repeat_interleave(rep, dim=2),
            t(v[a0:a1][None]), t(g[a0:a1][None]), t(beta[a0:a1][None]),
            chunk_size=64, initial_state=t(init[i][None]))
        outs.append(n(o[0])); finals.append(n(S[0]))
    chunk_out = np.concatenate(outs, 0)
    chunk_state = np.stack(finals)
    # 16 recurrent decode steps from the prefill states (torch recurrence)
    S = t(chunk_state)
    dec_in, dec_out = [], []
    for s in range(c["n_decode"]):
        dq, dk, dv, dg, db = I.core_inputs(len(lens), c["HK"], c["DK"], c["HV"], c["DV"],
                                           seed=1000 + s)
        o, S = Q._torch_recurrent_gated_delta_rule(
            t(dq[:, None]).repeat_interleave(rep, dim=2),
            t(dk[:, None]).repeat_interleave(rep, dim=2),
            t(dv[:, None]), t(dg[:, None]), t(db[:, None]), initial_state=S)
        dec_out.append(n(o[:, 0]))
    save("chunk_c0.npz", digest=np.array(I.digest(q, k, v, g, beta, init)),
         out=chunk_out, state=chunk_state, dec_out=np.stack(dec_out), dec_state=n(S))

    # ---------------- gated RMSNorm (bf16 rounding order) -----------------
    r = I.rng(15)
    x = bf(r.standard_normal((6, 8, 64)).astype(np.float32) * 2)
    z = bf(r.standard_normal((6, 8, 64)).astype(np.float32) * 2)
    w = bf((1 + 0.1 * r.standard_normal(64)).astype(np.float32))
    y = Q._rms_gated_forward(t(x, torch.bfloat16), t(z, torch.bfloat16),
                             t(w, torch.bfloat16), 1e-6)
    save("rms_gated.npz", x=x, z=z, w=w, y=n(y))

    # ---------------- full layer at config 0 (prefill + 16 decode) --------
    for dtype_name, dtype in (("fp32", torch.float32), ("bf16", torch.bfloat16)):
        _layer_case(Q, set_context, reset_context, dtype_name, dtype)


class _Cfg:
    def __init__(self, c):
        self.hidden_size = c["hidden"]
        self.linear_num_key_heads = c["HK"]
        self.linear_num_value_heads = c["HV"]
        self.linear_key_head_dim = c["DK"]
        self.linear_value_head_dim = c["DV"]
        self.linear_conv_kernel_dim = c["K"]
        self.rms_norm_eps = c["eps"]


def _layer_case(Q, set_context, reset_context, dtype_name, dtype):
    c = I.C0
    torch.set_default_dtype(dtype)
    try:
        m = Q.Qwen3_5GatedDeltaNet(_Cfg(c))
        W = I.layer_weights(c["hidden"], c["HK"], c["DK"], c["HV"], c["DV"], c["K"])
        with torch.no_grad():
            m.in_proj_qkv.weight.copy_(t(W["in_proj_qkv"]))
            m.in_proj_z.weight.copy_(t(W["in_proj_z"]))
            m.in_proj_b.weight.copy_(t(W["in_proj_b"]))
            m.in_proj_a.weight.copy_(t(W["in_proj_a"]))
            m.conv1d.weight.copy_(t(W["conv1d"]))
            m.A_log.copy_(t(W["A_log"]))
            m.dt_bias.copy_(t(W["dt_bias"]))
            m.norm.weight.copy_(t(W["norm"]))
            m.out_proj.weight.copy_(t(W["out_proj"]))
        slots = 6                                   # + 1 dummy slot (index 6)
        s_np, conv_np = I.layer_pools(slots + 1, c["HV"], c["DK"], c["DV"], m.conv_dim,
                                      c["K"])
        s_pool = t(s_np)
        conv_pool = t(conv_np, dtype)
        s_in, conv_in = n(s_pool), n(conv_pool)
        ids = np.array([5, 1, 3, 0], np.int64)
        lens = list(c["lens"])
        # fresh prefill: the engine zeroes the slots before the first chunk
        s_pool[torch.from_numpy(ids)] = 0
        conv_pool[torch.from_numpy(ids)] = 0
        m.s_cache = s_pool[:, 0]
        m.conv_cache = conv_pool[:, 0]
        hid = I.layer_hidden(sum(lens), c["hidden"])
        cu = torch.from_numpy(I.cu_from_lens(lens))
        set_context(cu, cu, max(lens), max(lens), linear_state_ids=torch.from_numpy(ids),
                    lens_q=lens)
        with torch.inference_mode():
            y_pre = m(None, t(hid, dtype))
        reset_context()
        dec_hid, dec_y = [], []
        for s in range(c["n_decode"]):
            h = I.layer_hidden(len(lens), c["hidden"], seed=200 + s)
            cu1 = torch.arange(len(lens) + 1, dtype=torch.int32)
            set_context(cu1, cu1, 1, 1, linear_state_ids=torch.from_numpy(ids),
                        lens_q=[1] * len(lens))
            with torch.inference_mode():
                yd = m(None, t(h, dtype))
            reset_context()
            dec_y.append(n(yd))
        s_out, conv_out = n(s_pool), n(conv_pool)
        untouched = np.ones(slots + 1, bool); untouched[ids] = False
        assert np.array_equal(s_out[untouched], s_in[untouched])
        assert np.array_equal(conv_out[untouched], conv_in[untouched])
        save(f"layer_c0_{dtype_name}.npz", ids=ids,
             y_prefill=n(y_pre), y_decode=np.stack(dec_y),
             s_rows=s_out[ids], conv_rows=conv_out[ids],
             digest=np.array(I.digest(hid, s_np, conv_np)))
    finally:
        torch.set_default_dtype(torch.float32)


if __name__ == "__main__":
    main()
