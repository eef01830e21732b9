"""GPU parity of each GDN kernel (through the C ABI) against the CPU oracle
and the reference's golden vectors.

Tolerances (from the path's spec): bf16 outputs max-abs <= 2e-2; fp32 states
relative error <= 1e-3 (Frobenius norm of the difference over the norm of the
oracle state); slot indexing, untouched slots and sequence boundaries
bit-exact.  Inputs are bf16-representable, so the oracle and the GPU see
identical values.
"""
import os

import numpy as np
import pytest
import torch

import inputs as I
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

OUT_ATOL = 2e-2
STATE_RTOL = 1e-3


@pytest.fixture(scope="module")
def ops(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    return pkg.ops


DEV = "cuda:0"


def bf(a):
    return torch.from_numpy(np.array(a, np.float32, order="C", copy=True)).to(DEV).to(
        torch.bfloat16)


def f32(a):
    return torch.from_numpy(np.array(a, np.float32, order="C", copy=True)).to(DEV)


def i64(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.int64)).to(DEV)


def i32(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.int32)).to(DEV)


def host(t):
    return t.float().cpu().numpy()


def bf16_ulp(x):
    ax = np.maximum(np.abs(x), 1e-30)
    return 2.0 ** (np.floor(np.log2(ax)) - 7)


def assert_bf16_close(a, b, ulps=1, atol=1e-6):
    a = np.asarray(a, np.float32); b = np.asarray(b, np.float32)
    tol = ulps * bf16_ulp(np.maximum(np.abs(a), np.abs(b))) + atol
    bad = np.abs(a - b) > tol
    assert not bad.any(), f"{bad.sum()}/{bad.size} differ, max |d| {np.abs(a - b).max()}"


def state_rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def load(golden_dir, name):
    return dict(np.load(os.path.join(golden_dir, name)))


# ---------------------------------------------------------------------------
# (b) gate
# ---------------------------------------------------------------------------


def test_gbeta_golden(ops, golden_dir):
    d = load(golden_dir, "gbeta.npz")
    for mask, gk, bk in ((d["mask"], "g_mask", "beta_mask"), (None, "g", "beta")):
        m = None if mask is None else torch.from_numpy(mask).to(DEV)
        g, beta = ops.fused_g_beta(bf(d["b"]), bf(d["a"]), bf(d["a_log"]), bf(d["dt_bias"]), m)
        np.testing.assert_allclose(host(g), d[gk], rtol=2e-6, atol=1e-6)
        assert_bf16_close(host(beta), d[bk])
    # fp32 parameters and strided row views
    big = bf(np.concatenate([d["b"].reshape(15, 8), d["a"].reshape(15, 8)], 1))
    g, beta = ops.fused_g_beta(big[:, :8], big[:, 8:], f32(d["a_log"]), f32(d["dt_bias"]))
    np.testing.assert_allclose(host(g), d["g"].reshape(15, 8), rtol=2e-6, atol=1e-6)


# ---------------------------------------------------------------------------
# (a) conv
# ---------------------------------------------------------------------------


def test_conv_decode_golden(ops, golden_dir):
    d = load(golden_dir, "conv_decode.npz")
    pool = bf(d["pool_in"])
    y = ops.conv_decode_step(bf(d["x"]), pool[:, int(d["layer"])], i64(d["ids"]), bf(d["w"]))
    assert_bf16_close(host(y), d["y"])
    assert np.array_equal(host(pool), d["pool_out"])   # roll is bit-exact, other slots untouched
    ops.check_status()


@pytest.mark.parametrize("C", [1024, 96, 100])
def test_conv_decode_vs_oracle(ops, C):
    r = I.rng(31)
    n, K, slots, L = 7, 4, 12, 3
    x = O.round_bf16(r.standard_normal((n, C + 16)).astype(np.float32))   # strided rows
    pool = O.round_bf16(r.standard_normal((slots, L, C, K - 1)).astype(np.float32))
    w = O.round_bf16(r.uniform(-0.6, 0.6, (C, K)).astype(np.float32))
    ids = r.permutation(slots)[:n]
    pool_d = bf(pool)
    y = ops.conv_decode_step(bf(x)[:, :C], pool_d[:, 2], i64(ids), bf(w))
    ref_pool = pool.copy()
    ref = O.conv_decode_step(x[:, :C], ref_pool[:, 2], ids, w)
    assert_bf16_close(host(y), ref)
    assert np.array_equal(host(pool_d), ref_pool)


@pytest.mark.parametrize("C", [1024, 96, 100])
def test_conv_varlen_vs_oracle(ops, C):
    r = I.rng(32)
    lens = [0, 1, 2, 3, 31, 32, 33, 100, 0, 5]
    N = sum(lens)
    K, slots, L = 4, 14, 2
    x = O.round_bf16(r.standard_normal((N, C)).astype(np.float32))
    pool = O.round_bf16(r.standard_normal((slots, L, C, K - 1)).astype(np.float32))
    w = O.round_bf16(r.uniform(-0.6, 0.6, (C, K)).astype(np.float32))
    ids = r.permutation(slots)[:len(lens)]
    cu = I.cu_from_lens(lens)
    pool_d = bf(pool)
    y = ops.causal_conv_silu_varlen(bf(x), pool_d[:, 1], i64(ids), bf(w), i32(cu))
    ref_pool = pool.copy()
    ref = O.causal_conv_silu_varlen(x, ref_pool[:, 1], ids, cu, w)
    assert_bf16_close(host(y), ref)
    # sequence boundaries and the state roll are bit-exact; empty sequences
    # and every other slot / layer are untouched
    assert np.array_equal(host(pool_d), ref_pool)
    ops.check_status()


@pytest.mark.parametrize("C,pdt", [(1024, torch.bfloat16), (100, torch.float32)])
def test_conv_gate_varlen_equals_separate_calls(ops, C, pdt):
    """The combined conv + gate call gives the bits of causal_conv_silu_varlen
    and fused_g_beta run separately: y, g, beta and the rolled states, on
    ragged sequences (empty ones included), b / a as strided column views of
    one projection row (the layer's layout), vector and scalar conv paths."""
    r = I.rng(33)
    lens = [0, 1, 2, 3, 31, 32, 33, 100, 0, 5, 700]
    N, K, slots, HV = sum(lens), 4, 14, 16
    proj = bf(r.standard_normal((N, C + 2 * HV + 8)).astype(np.float32))
    x, b, a = proj[:, :C], proj[:, C:C + HV], proj[:, C + HV:C + 2 * HV]
    w = bf(r.uniform(-0.6, 0.6, (C, K)).astype(np.float32))
    a_log = torch.from_numpy(r.uniform(-1, 0, HV).astype(np.float32)).to(DEV).to(pdt)
    dt_bias = torch.from_numpy(r.standard_normal(HV).astype(np.float32)).to(DEV).to(pdt)
    pool = bf(r.standard_normal((slots, C, K - 1)).astype(np.float32))
    ids = i64(r.permutation(slots)[:len(lens)])
    cu = i32(I.cu_from_lens(lens))
    p1, p2 = pool.clone(), pool.clone()
    y1 = ops.causal_conv_silu_varlen(x, p1, ids, w, cu)
    g1, b1 = ops.fused_g_beta(b, a, a_log, dt_bias)
    y2, g2, b2 = ops.conv_gate_varlen(x, p2, ids, w, cu, b, a, a_log, dt_bias)
    ops.check_status()
    for u, v in ((y1, y2), (g1, g2), (b1, b2), (p1, p2)):
        assert u.shape == v.shape and torch.equal(u, v)


def test_conv_padded_golden_rows(ops, golden_dir):
    """Rows of the reference's padded conv whose writeback is at T match the
    varlen kernel (values and state)."""
    d = load(golden_dir, "conv_padded.npz")
    T = d["x"].shape[2]
    for row in [r for r in range(d["x"].shape[0]) if d["endp"][r] == T]:
        pool = bf(d["state_in"][row][None])
        y = ops.causal_conv_silu_varlen(bf(d["x"][row].T), pool, i64([0]), bf(d["w"]),
                                        i32([0, T]))
        assert_bf16_close(host(y).T, d["y"][row])
        assert np.array_equal(host(pool)[0], d["state_out"][row])


def test_conv_split_equals_one_shot(ops):
    """Chunked prefill continuation: two calls over a split sequence equal one
    call (the conv state threads across calls)."""
    r = I.rng(33)
    C, K = 512, 4
    x = O.round_bf16(r.standard_normal((150, C)).astype(np.float32))
    w = O.round_bf16(r.uniform(-0.6, 0.6, (C, K)).astype(np.float32))
    p1 = torch.zeros(2, C, K - 1, dtype=torch.bfloat16, device=DEV)
    p2 = p1.clone()
    y1 = ops.causal_conv_silu_varlen(bf(x), p1, i64([1]), bf(w), i32([0, 150]))
    ya = ops.causal_conv_silu_varlen(bf(x[:61]), p2, i64([1]), bf(w), i32([0, 61]))
    yb = ops.causal_conv_silu_varlen(bf(x[61:62]), p2, i64([1]), bf(w), i32([0, 1]))
    yc = ops.causal_conv_silu_varlen(bf(x[62:]), p2, i64([1]), bf(w), i32([0, 88]))
    assert torch.equal(y1, torch.cat([ya, yb, yc]))
    assert torch.equal(p1, p2)


# ---------------------------------------------------------------------------
# (d) recurrent decode
# ---------------------------------------------------------------------------


def test_recurrent_golden(ops, golden_dir):
    d = load(golden_dir, "recurrent_inplace.npz")
    HK, HV, D = int(d["HK"]), int(d["HV"]), int(d["D"])
    slots, L, bs = 9, 2, 5
    pool = I.recurrent_pool(slots, L, HV, D)
    layer = int(d["layer"])
    pool_d = f32(pool)
    kd = HK * D
    for s in range(3):
        mixed, g, beta = I.recurrent_step_inputs(bs, HK, HV, D, s)
        m = bf(mixed)
        q = m[:, :kd].view(bs, 1, HK, D)
        k = m[:, kd:2 * kd].view(bs, 1, HK, D)
        v = m[:, 2 * kd:].view(bs, 1, HV, D)
        out = ops.recurrent_gdn_inplace(q, k, v, f32(g).view(bs, 1, HV), bf(beta).view(bs, 1, HV),
                                        pool_d[:, layer], i64(d["ids"]))
        assert np.abs(host(out)[:, 0] - d[f"out{s}"]).max() <= OUT_ATOL
        assert_bf16_close(host(out)[:, 0], d[f"out{s}"], ulps=2, atol=1e-4)
    got = host(pool_d)
    assert state_rel(got[d["ids"], layer], d["rows_out"]) <= 1e-5
    untouched = np.setdiff1d(np.arange(slots), d["ids"])
    assert np.array_equal(got[untouched], pool[untouched])
    assert np.array_equal(got[:, 0], pool[:, 0])


@pytest.mark.parametrize("bs", [64, 2])   # full-tile and column-split launches
def test_recurrent_d128_vs_oracle(ops, bs):
    HK, HV, D, slots, L = 16, 32, 128, 97, 2
    r = I.rng(40 + bs)
    q, k, v, g, beta = I.core_inputs(bs, HK, D, HV, D, seed=41 + bs)
    q, k, v, beta = (O.round_bf16(t) for t in (q, k, v, beta))
    pool = (r.standard_normal((slots, L, HV, D, D)) * 0.02).astype(np.float32)
    ids = r.permutation(slots - 1)[:bs]
    pool_d = f32(pool)
    out = ops.recurrent_gdn_inplace(bf(q), bf(k), bf(v), f32(g), bf(beta), pool_d[:, 1], i64(ids))
    ref_pool = pool.copy()
    ref = O.recurrent_inplace(q, k, v, g, beta, ref_pool[:, 1], ids)
    assert np.abs(host(out)[:, 0] - ref).max() <= OUT_ATOL
    got = host(pool_d)
    assert state_rel(got[ids, 1], ref_pool[ids, 1]) <= 1e-5
    mask = np.ones(slots, bool); mask[ids] = False
    assert np.array_equal(got[mask], pool[mask])
    assert np.array_equal(got[:, 0], pool[:, 0])


def test_recurrent_bad_slot_is_flagged_not_touched(ops):
    HK, HV, D, slots = 1, 2, 64, 4
    q, k, v, g, beta = I.core_inputs(3, HK, D, HV, D, seed=5)
    pool = (I.rng(6).standard_normal((slots, HV, D, D)) * 0.02).astype(np.float32)
    pool_d = f32(pool)
    ops.check_status()
    ops.recurrent_gdn_inplace(bf(q), bf(k), bf(v), f32(g), bf(beta), pool_d,
                              i64([1, slots, -1]))
    with pytest.raises(IndexError):
        ops.check_status()
    got = host(pool_d)
    assert np.array_equal(np.delete(got, 1, 0), np.delete(pool, 1, 0))


# ---------------------------------------------------------------------------
# (c) chunked prefill
# ---------------------------------------------------------------------------


def _chunk_case(ops, lens, HK, HV, D, seed, init_scale=0.02):
    N = sum(lens)
    q, k, v, g, beta = I.core_inputs(N, HK, D, HV, D, seed=seed)
    q, k, v, beta = (O.round_bf16(t) for t in (q, k, v, beta))
    r = I.rng(seed + 1)
    slots = len(lens) + 3
    pool = (r.standard_normal((slots, HV, D, D)) * init_scale).astype(np.float32)
    ids = r.permutation(slots)[:len(lens)]
    cu = I.cu_from_lens(lens)
    pool_d = f32(pool)
    out = ops.chunk_gated_delta_rule_varlen(bf(q), bf(k), bf(v), f32(g), bf(beta), pool_d,
                                            i64(ids), i32(cu), max(lens))
    ref_pool = pool.copy()
    ref = O.chunk_prefill_varlen(q, k, v, g, beta, ref_pool, ids, cu, dtype=np.float64)
    got_out, got_pool = host(out), host(pool_d)
    assert np.abs(got_out - ref).max() <= OUT_ATOL
    for i, sl in enumerate(ids):
        if lens[i]:
            assert state_rel(got_pool[sl], ref_pool[sl]) <= STATE_RTOL, f"slot {sl}"
    untouched = np.setdiff1d(np.arange(slots), [s for s, n in zip(ids, lens) if n])
    assert np.array_equal(got_pool[untouched], pool[untouched])
    ops.check_status()
    return got_out, got_pool


def test_chunk_c0_vs_oracle(ops):
    c = I.C0
    _chunk_case(ops, list(c["lens"]), c["HK"], c["HV"], c["DK"], seed=0)


def test_chunk_ragged_d128(ops):
    _chunk_case(ops, [1, 2, 63, 64, 65, 130, 0, 200], 2, 4, 128, seed=7)


def test_chunk_split_equals_one_shot(ops):
    """Two varlen calls over a split sequence (the chunked-prefill budget
    splitting a prompt) give the one-shot state and outputs."""
    HK, HV, D = 2, 4, 128
    q, k, v, g, beta = I.core_inputs(300, HK, D, HV, D, seed=9)
    q, k, v, beta = (O.round_bf16(t) for t in (q, k, v, beta))
    p1 = torch.zeros(2, HV, D, D, device=DEV)
    p2 = p1.clone()
    o1 = ops.chunk_gated_delta_rule_varlen(bf(q), bf(k), bf(v), f32(g), bf(beta), p1, i64([1]),
                                           i32([0, 300]), 300)
    parts = []
    for a, b in ((0, 100), (100, 300)):
        parts.append(ops.chunk_gated_delta_rule_varlen(
            bf(q[a:b]), bf(k[a:b]), bf(v[a:b]), f32(g[a:b]), bf(beta[a:b]), p2, i64([1]),
            i32([0, b - a]), b - a))
    assert np.abs(host(o1) - host(torch.cat(parts))).max() <= OUT_ATOL
    assert state_rel(host(p2), host(p1)) <= STATE_RTOL


@pytest.mark.parametrize("lens,HK,HV", [
    ([1, 2, 63, 64, 65, 130, 0, 200, 1000], 2, 4),    # ragged; two v-heads per k-head
    ([300, 5], 4, 4),                                 # one v-head per k-head
    ([129], 1, 4),                                    # four v-heads per k-head
    (list(I.rng(33).integers(0, 150, 300)), 1, 2),    # > 256 sequences: launch-order chains
    ([100, 64, 7], 1, 3),                             # odd v-head count: a half-empty last pair
    ([129, 40], 2, 6),                                # three v-heads per k-head: a pair across two
])
def test_chunk_split_form_equals_one_kernel_form(ops, lens, HK, HV):
    """Head dim 128: the split form (per-chunk prep pass + chain) and the
    one-kernel form compute the same steps with the same roundings, so the
    outputs and the states agree bit for bit."""
    D = 128
    lens = [int(x) for x in lens]
    N = sum(lens)
    q, k, v, g, beta = I.core_inputs(N, HK, D, HV, D, seed=31 + len(lens))
    q, k, v, beta = (O.round_bf16(t) for t in (q, k, v, beta))
    slots = len(lens) + 2
    pool = (I.rng(32).standard_normal((slots, HV, D, D)) * 0.02).astype(np.float32)
    ids = I.rng(34).permutation(slots)[:len(lens)]
    cu = I.cu_from_lens(lens)
    res = []
    for split in (True, False):
        pool_d = f32(pool)
        out = ops.chunk_gated_delta_rule_varlen(bf(q), bf(k), bf(v), f32(g), bf(beta), pool_d,
                                                i64(ids), i32(cu), max(lens), split=split)
        res.append((out, pool_d))
    ops.check_status()
    assert torch.equal(res[0][0], res[1][0])
    assert torch.equal(res[0][1], res[1][1])


def test_chunk_split_overlapping_cu_is_flagged(ops):
    """Overlapping (malformed) cu_seqlens can ask for more chunks than the
    workspace holds for n_tokens rows: the sequence cut short is flagged and
    skipped (its slot untouched); the well-formed first sequence is exact."""
    HK, HV, D, N = 1, 2, 128, 160
    q, k, v, g, beta = I.core_inputs(N, HK, D, HV, D, seed=73)
    q, k, v, beta = (O.round_bf16(t) for t in (q, k, v, beta))
    pool = (I.rng(74).standard_normal((4, HV, D, D)) * 0.02).astype(np.float32)
    pool_d = f32(pool)
    ops.check_status()
    # (0, 150): 3 chunks; (150, 10): negative length; (10, 160): 3 chunks > capacity 5
    ops.chunk_gated_delta_rule_varlen(bf(q), bf(k), bf(v), f32(g), bf(beta), pool_d,
                                      i64([0, 1, 2]), i32([0, 150, 10, 160]), 150)
    with pytest.raises(ValueError):
        ops.check_status()
    got = host(pool_d)
    assert np.array_equal(got[[1, 2, 3]], pool[[1, 2, 3]])
    ref_pool = pool.copy()
    O.chunk_prefill_varlen(q[:150], k[:150], v[:150], g[:150], beta[:150], ref_pool,
                           np.array([0]), np.array([0, 150]), dtype=np.float64)
    assert state_rel(got[0], ref_pool[0]) <= STATE_RTOL


def test_chunk_then_decode_c0(ops):
    """Config 0 end to end on the core: prefill, then 16 decode steps."""
    c = I.C0
    lens = list(c["lens"])
    HK, HV, D = c["HK"], c["HV"], c["DK"]
    N = sum(lens)
    q, k, v, g, beta = I.core_inputs(N, HK, D, HV, D, seed=0)
    q, k, v, beta = (O.round_bf16(t) for t in (q, k, v, beta))
    ids = np.array([5, 1, 3, 0])
    pool = np.zeros((7, HV, D, D), np.float32)
    pool_d = f32(pool)
    ops.chunk_gated_delta_rule_varlen(bf(q), bf(k), bf(v), f32(g), bf(beta), pool_d, i64(ids),
                                      i32(I.cu_from_lens(lens)), max(lens))
    O.chunk_prefill_varlen(q, k, v, g, beta, pool, ids, I.cu_from_lens(lens), dtype=np.float64)
    for s in range(c["n_decode"]):
        dq, dk, dv, dg, db = I.core_inputs(4, HK, D, HV, D, seed=1000 + s)
        dq, dk, dv, db = (O.round_bf16(t) for t in (dq, dk, dv, db))
        o = ops.recurrent_gdn_inplace(bf(dq), bf(dk), bf(dv), f32(dg), bf(db), pool_d, i64(ids))
        ref = O.recurrent_inplace(dq, dk, dv, dg, db, pool, ids, dtype=np.float64)
        assert np.abs(host(o)[:, 0] - ref).max() <= OUT_ATOL
    got = host(pool_d)
    for sl in ids:
        assert state_rel(got[sl], pool[sl]) <= STATE_RTOL


# ---------------------------------------------------------------------------
# gated norm
# ---------------------------------------------------------------------------


def test_rms_gated_golden(ops, golden_dir):
    d = load(golden_dir, "rms_gated.npz")
    y = ops.rms_norm_gated(bf(d["x"]), bf(d["z"]), bf(d["w"]), 1e-6)
    assert_bf16_close(host(y), d["y"], ulps=2)
    # gate as a strided column slice of a wider buffer
    zz = bf(np.concatenate([d["z"].reshape(6, 512), np.zeros((6, 40), np.float32)], 1))
    y2 = ops.rms_norm_gated(bf(d["x"]), zz[:, :512].view(6, 8, 64), bf(d["w"]), 1e-6)
    assert torch.equal(y, y2)


# ---------------------------------------------------------------------------
# fused gated-RMSNorm epilogues
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("bs", [64, 2])   # full-tile (fused) and column-split (norm after)
def test_recurrent_fused_norm(ops, bs):
    HK, HV, D = 16, 32, 128
    q, k, v, g, beta = I.core_inputs(bs, HK, D, HV, D, seed=61)
    q, k, v, beta = (O.round_bf16(t) for t in (q, k, v, beta))
    r = I.rng(62)
    pool = (r.standard_normal((bs + 1, HV, D, D)) * 0.02).astype(np.float32)
    zbig = O.round_bf16(r.standard_normal((bs, HV * D + 24)).astype(np.float32))
    w = O.round_bf16((1 + 0.1 * r.standard_normal(D)).astype(np.float32))
    ids = np.arange(bs)
    p1, p2 = f32(pool), f32(pool)
    zd = bf(zbig)[:, :HV * D].view(bs, HV, D)           # strided rows, as a projection slice
    fused = ops.recurrent_gdn_inplace(bf(q), bf(k), bf(v), f32(g), bf(beta), p1, i64(ids),
                                      z=zd, norm_weight=bf(w), eps=1e-6)
    plain = ops.recurrent_gdn_inplace(bf(q), bf(k), bf(v), f32(g), bf(beta), p2, i64(ids))
    ref = ops.rms_norm_gated(plain[:, 0], zd, bf(w), 1e-6)
    assert torch.equal(p1, p2)
    assert_bf16_close(host(fused)[:, 0], host(ref), ulps=1, atol=1e-3)


def test_chunk_fused_norm(ops):
    for D, HK, HV in ((128, 2, 4), (64, 2, 4)):          # tensor-core and fp32 kernels
        lens = [70, 1, 130]
        N = sum(lens)
        q, k, v, g, beta = I.core_inputs(N, HK, D, HV, D, seed=63)
        q, k, v, beta = (O.round_bf16(t) for t in (q, k, v, beta))
        r = I.rng(64)
        zbig = O.round_bf16(r.standard_normal((N, HV * D + 8)).astype(np.float32))
        w = O.round_bf16((1 + 0.1 * r.standard_normal(D)).astype(np.float32))
        cu = I.cu_from_lens(lens)
        p1 = torch.zeros(3, HV, D, D, device=DEV)
        p2 = p1.clone()
        zd = bf(zbig)[:, :HV * D].view(N, HV, D)
        fused = ops.chunk_gated_delta_rule_varlen(bf(q), bf(k), bf(v), f32(g), bf(beta), p1,
                                                  i64([0, 1, 2]), i32(cu), max(lens), z=zd,
                                                  norm_weight=bf(w), eps=1e-6)
        plain = ops.chunk_gated_delta_rule_varlen(bf(q), bf(k), bf(v), f32(g), bf(beta), p2,
                                                  i64([0, 1, 2]), i32(cu), max(lens))
        ref = ops.rms_norm_gated(plain, zd, bf(w), 1e-6)
        assert torch.equal(p1, p2)
        assert_bf16_close(host(fused), host(ref), ulps=1, atol=1e-3)


def test_chunk_fused_norm_whole_state_chains(ops):
    """The z / norm_weight arguments on the whole-state chain form (at least
    two chains per SM), full and partial last chunks: the result equals the
    chunk output followed by the standalone gated norm, bit for bit."""
    D, HK, HV = 128, 2, 4
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    n_seqs = (2 * sms) // HV + 5
    lens = [int(x) for x in I.rng(65).integers(1, 200, n_seqs)]
    lens[:3] = [64, 128, 65]
    N = sum(lens)
    q, k, v, g, beta = I.core_inputs(N, HK, D, HV, D, seed=66)
    q, k, v, beta = (O.round_bf16(t) for t in (q, k, v, beta))
    r = I.rng(67)
    zbig = O.round_bf16(r.standard_normal((N, HV * D + 8)).astype(np.float32))
    w = O.round_bf16((1 + 0.1 * r.standard_normal(D)).astype(np.float32))
    cu = I.cu_from_lens(lens)
    ids = i64(np.arange(n_seqs))
    p1 = f32((I.rng(68).standard_normal((n_seqs, HV, D, D)) * 0.02).astype(np.float32))
    p2 = p1.clone()
    zd = bf(zbig)[:, :HV * D].view(N, HV, D)
    fused = ops.chunk_gated_delta_rule_varlen(bf(q), bf(k), bf(v), f32(g), bf(beta), p1, ids,
                                              i32(cu), max(lens), z=zd, norm_weight=bf(w),
                                              eps=1e-6)
    plain = ops.chunk_gated_delta_rule_varlen(bf(q), bf(k), bf(v), f32(g), bf(beta), p2, ids,
                                              i32(cu), max(lens))
    ref = ops.rms_norm_gated(plain, zd, bf(w), 1e-6)
    ops.check_status()
    assert torch.equal(p1, p2)
    assert torch.equal(fused, ref)


# ---------------------------------------------------------------------------
# malformed cu_seqlens: flagged on the device, never read out of bounds
# ---------------------------------------------------------------------------


def test_conv_varlen_malformed_cu_is_flagged(ops):
    """Sequence 1 ends before it starts: GDN_STATUS_BAD_SEQLEN is raised and its
    slot is not touched (the other sequences run)."""
    r = I.rng(70)
    C, K, slots = 256, 4, 5
    x = O.round_bf16(r.standard_normal((100, C)).astype(np.float32))
    pool = O.round_bf16(r.standard_normal((slots, C, K - 1)).astype(np.float32))
    w = O.round_bf16(r.uniform(-0.6, 0.6, (C, K)).astype(np.float32))
    pool_d = bf(pool)
    ops.check_status()
    ops.causal_conv_silu_varlen(bf(x), pool_d, i64([0, 3, 1]), bf(w), i32([0, 50, 30, 100]))
    with pytest.raises(ValueError):
        ops.check_status()
    assert np.array_equal(host(pool_d)[3], pool[3])


@pytest.mark.parametrize("D", [128, 64])    # tensor-core and fp32 kernels
def test_chunk_malformed_cu_is_flagged(ops, D):
    """A sequence past the end of the rows and one longer than max_seqlen: both
    flagged; the first is skipped (slot untouched), the second truncated."""
    HK, HV = 1, 2
    N = 150
    q, k, v, g, beta = I.core_inputs(N, HK, D, HV, D, seed=71)
    q, k, v, beta = (O.round_bf16(t) for t in (q, k, v, beta))
    pool = (I.rng(72).standard_normal((4, HV, D, D)) * 0.02).astype(np.float32)
    pool_d = f32(pool)
    ops.check_status()
    ops.chunk_gated_delta_rule_varlen(bf(q), bf(k), bf(v), f32(g), bf(beta), pool_d,
                                      i64([0, 2]), i32([0, 100, 180]), 80)
    with pytest.raises(ValueError):
        ops.check_status()
    got = host(pool_d)
    assert np.array_equal(got[2], pool[2])            # [100, 180) runs past 150 rows: skipped
    assert np.array_equal(got[[1, 3]], pool[[1, 3]])  # unused slots
    # the over-long sequence is truncated to max_seqlen = 80 tokens
    ref_pool = pool.copy()
    O.chunk_prefill_varlen(q[:80], k[:80], v[:80], g[:80], beta[:80], ref_pool, np.array([0]),
                           np.array([0, 80]), dtype=np.float64)
    assert state_rel(got[0], ref_pool[0]) <= STATE_RTOL


# ---------------------------------------------------------------------------
# integer-exact probes: bit-exact slots, heads and sequence boundaries
# ---------------------------------------------------------------------------
#
# g = 0 (no decay), beta = 1, k and q one-hot with magnitude 2^10 (their l2 norms
# are exact: rsqrt(2^20 + 1e-6) = 2^-10 in fp32), v and the states small integers:
# every product and sum of the delta rule is then exact in fp32 (and in the
# tensor-core kernel's bf16 hi/lo operands), so the new states must equal the
# sequential recurrence bit for bit, and each output element is one state value
# times Dk^-1/2 (rounded once by the recurrent kernel; the chunk kernels add an
# inter- and an intra-chunk fp32 term first, see the chunk test).  The one-hot positions differ per token and head,
# so a wrong slot, head (GQA mapping) or sequence boundary changes the bits.


def _exact_recurrence(q_pos, k_pos, v, S, scale):
    """Sequential delta rule for one-hot q/k (positions) on an integer state S
    [D, D] (fp32, updated in place); returns the outputs [T, D] (fp32 products
    S[j] * scale as the kernels form them, before the bf16 rounding)."""
    outs = []
    for t in range(len(k_pos)):
        i, j = int(k_pos[t]), int(q_pos[t])
        S[i, :] = v[t]                       # S[i] + (v - S[i]) with exact integers
        outs.append(S[j, :] * np.float32(scale))
    return np.array(outs, np.float32)


def _onehot(pos, D):
    x = np.zeros((len(pos), D), np.float32)
    x[np.arange(len(pos)), pos] = 1024.0
    return x


def test_recurrent_integer_exact(ops):
    HK, HV, D, slots = 2, 4, 128, 7
    rep = HV // HK
    r = I.rng(80)
    bs = 3
    ids = np.array([5, 0, 3])
    pool = r.integers(-8, 9, (slots, HV, D, D)).astype(np.float32)    # canaries everywhere
    qp = r.integers(0, D, (bs, HK))
    kp = r.integers(0, D, (bs, HK))
    q = np.stack([_onehot(qp[:, hk], D) for hk in range(HK)], 1)       # [bs, HK, D]
    k = np.stack([_onehot(kp[:, hk], D) for hk in range(HK)], 1)
    v = r.integers(-8, 9, (bs, HV, D)).astype(np.float32)
    g = np.zeros((bs, HV), np.float32)
    beta = np.ones((bs, HV), np.float32)
    pool_d = f32(pool)
    out = ops.recurrent_gdn_inplace(bf(q), bf(k), bf(v), f32(g), bf(beta), pool_d, i64(ids))
    ref_pool = pool.copy()
    ref_out = np.zeros((bs, HV, D), np.float32)
    for b in range(bs):
        for h in range(HV):
            hk = h // rep
            ref_out[b, h] = _exact_recurrence([qp[b, hk]], [kp[b, hk]], v[b, h][None],
                                              ref_pool[ids[b], h], D ** -0.5)[0]
    assert np.array_equal(host(pool_d), ref_pool)          # every slot, bit for bit
    assert np.array_equal(host(out)[:, 0], O.round_bf16(ref_out))
    ops.check_status()


@pytest.mark.parametrize("D", [128, 64])    # tensor-core and fp32 kernels
def test_chunk_integer_exact(ops, D):
    HK, HV = 2, 4
    rep = HV // HK
    lens = [70, 1, 0, 130, 64]
    N = sum(lens)
    slots = len(lens) + 3
    r = I.rng(81 + D)
    ids = r.permutation(slots)[:len(lens)]
    pool = r.integers(-8, 9, (slots, HV, D, D)).astype(np.float32)
    qp = r.integers(0, D, (N, HK))
    kp = r.integers(0, D, (N, HK))
    q = np.stack([_onehot(qp[:, hk], D) for hk in range(HK)], 1)
    k = np.stack([_onehot(kp[:, hk], D) for hk in range(HK)], 1)
    v = r.integers(-8, 9, (N, HV, D)).astype(np.float32)
    g = np.zeros((N, HV), np.float32)
    beta = np.ones((N, HV), np.float32)
    cu = I.cu_from_lens(lens)
    pool_d = f32(pool)
    out = ops.chunk_gated_delta_rule_varlen(bf(q), bf(k), bf(v), f32(g), bf(beta), pool_d,
                                            i64(ids), i32(cu), max(lens))
    ref_pool = pool.copy()
    ref_out = np.zeros((N, HV, D), np.float32)
    for s, sl in enumerate(ids):
        t0, t1 = int(cu[s]), int(cu[s + 1])
        for h in range(HV):
            hk = h // rep
            ref_out[t0:t1, h] = _exact_recurrence(qp[t0:t1, hk], kp[t0:t1, hk], v[t0:t1, h],
                                                  ref_pool[sl, h], D ** -0.5).reshape(-1, D)
    assert np.array_equal(host(pool_d), ref_pool)          # every slot, bit for bit
    # the chunk kernels add the inter-chunk term (fp32 scale) and the intra-chunk
    # term (through the bf16 M2 = QKm T) before the bf16 rounding, so outputs
    # whose terms cancel keep a residual of ~1e-4 of a term: within one bf16 ulp
    # plus that residual of the single-rounding value
    assert_bf16_close(host(out), O.round_bf16(ref_out), ulps=1, atol=2e-4)
    ops.check_status()
