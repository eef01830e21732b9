"""The one-launch decode core (gdn_decode_fused: conv step + g/beta gate +
in-place recurrence + gated RMSNorm) against the oracle's decode core
(gdn_core_decode, qwen3_5.py:974-1026, 1083-1085) and against the
four-operator sequence it replaces, through the C ABI.

Tolerances: bf16 outputs max-abs <= 2e-2 vs the oracle; fp32 states relative
<= 1e-3; conv-state rolls, slot indexing and untouched slots bit-exact.  Where
the four-operator sequence runs its full-tile recurrent kernel (>= 4 units per
SM) the fused kernel must reproduce it bit for bit.
"""
import numpy as np
import pytest
import torch

import inputs as I
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
OUT_ATOL = 2e-2
STATE_RTOL = 1e-3


@pytest.fixture(scope="module")
def ops(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    return pkg.ops


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.array(a, np.float32, order="C", copy=True)).to(DEV).to(dtype)


def host(t):
    return t.float().cpu().numpy()


def state_rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def make_case(HK, HV, D, K, bs, seed, slots_extra=5, layers=2):
    r = I.rng(seed)
    C = (2 * HK + HV) * D
    W = C + HV * D + 2 * HV + 8                    # projection row [qkv | z | b | a | pad]
    proj = O.round_bf16(r.standard_normal((bs, W)).astype(np.float32))
    slots = bs + slots_extra
    s_pool = (r.standard_normal((slots, layers, HV, D, D)) * 0.02).astype(np.float32)
    conv_pool = O.round_bf16(r.standard_normal((slots, layers, C, K - 1)).astype(np.float32))
    conv_w = O.round_bf16(r.uniform(-0.6, 0.6, (C, K)).astype(np.float32))
    a_log = O.round_bf16(r.uniform(-1.0, 1.0, HV).astype(np.float32))
    dt_bias = O.round_bf16(r.uniform(-0.5, 0.5, HV).astype(np.float32))
    norm_w = O.round_bf16((1 + 0.1 * r.standard_normal(D)).astype(np.float32))
    ids = r.permutation(slots)[:bs]
    return dict(HK=HK, HV=HV, D=D, K=K, bs=bs, C=C, proj=proj, s_pool=s_pool,
                conv_pool=conv_pool, conv_w=conv_w, a_log=a_log, dt_bias=dt_bias,
                norm_w=norm_w, ids=ids, layer=1)


def views(c, proj_d):
    """mixed / z / b / a as column views of the projection rows."""
    C, HV, D, bs = c["C"], c["HV"], c["D"], c["bs"]
    mixed = proj_d[:, :C]
    z = proj_d[:, C:C + HV * D].view(bs, HV, D)
    b = proj_d[:, C + HV * D:C + HV * D + HV]
    a = proj_d[:, C + HV * D + HV:C + HV * D + 2 * HV]
    return mixed, z, b, a


def run_fused(ops, c, pdt, counters=True):
    proj_d = dev(c["proj"], torch.bfloat16)
    mixed, z, b, a = views(c, proj_d)
    s_d = dev(c["s_pool"])
    cv_d = dev(c["conv_pool"], torch.bfloat16)
    L = c["layer"]
    out = ops.decode_fused(mixed, z, b, a, cv_d[:, L], dev(c["conv_w"], torch.bfloat16),
                           dev(c["a_log"], pdt), dev(c["dt_bias"], pdt), s_d[:, L],
                           torch.as_tensor(c["ids"], device=DEV), dev(c["norm_w"], torch.bfloat16),
                           1e-6, counters=counters)
    return out, s_d, cv_d


def run_four_ops(ops, c, pdt):
    proj_d = dev(c["proj"], torch.bfloat16)
    mixed, z, b, a = views(c, proj_d)
    s_d = dev(c["s_pool"])
    cv_d = dev(c["conv_pool"], torch.bfloat16)
    L = c["layer"]
    ids = torch.as_tensor(c["ids"], device=DEV)
    HK, HV, D, bs = c["HK"], c["HV"], c["D"], c["bs"]
    g, beta = ops.fused_g_beta(b, a, dev(c["a_log"], pdt), dev(c["dt_bias"], pdt))
    y = ops.conv_decode_step(mixed, cv_d[:, L], ids, dev(c["conv_w"], torch.bfloat16))
    kd = HK * D
    q = y[:, :kd].view(bs, 1, HK, D)
    k = y[:, kd:2 * kd].view(bs, 1, HK, D)
    v = y[:, 2 * kd:].view(bs, 1, HV, D)
    o = ops.recurrent_gdn_inplace(q, k, v, g, beta, s_d[:, L], ids, z=z,
                                  norm_weight=dev(c["norm_w"], torch.bfloat16), eps=1e-6)
    return o.view(bs, HV, D), s_d, cv_d


CASES = [
    # HK, HV, D, K, bs, param dtype
    (2, 4, 128, 4, 7, torch.float32),
    (16, 32, 128, 4, 300, torch.float32),   # 4800 groups: many per CTA, the stage ring wraps
    (1, 4, 64, 4, 5, torch.bfloat16),
    (4, 4, 64, 3, 33, torch.float32),       # one v-head per k-head
    (4, 4, 64, 3, 1200, torch.bfloat16),    # one unit per group, 8 groups per CTA
    (2, 8, 128, 2, 3, torch.bfloat16),      # four v-heads per k-head
]


def counters_zero(ops):
    t = ops._COUNTERS.get(0)
    return t is None or int(t.abs().sum().item()) == 0


@pytest.mark.parametrize("counters", [True, False])   # head-per-CTA / persistent form
@pytest.mark.parametrize("HK,HV,D,K,bs,pdt", CASES)
def test_decode_fused_vs_oracle(ops, HK, HV, D, K, bs, pdt, counters):
    c = make_case(HK, HV, D, K, bs, seed=500 + bs + D)
    out, s_d, cv_d = run_fused(ops, c, pdt, counters)
    ops.check_status()
    assert counters_zero(ops)
    L, ids = c["layer"], c["ids"]
    C = c["C"]
    p = c["proj"]
    s_ref = c["s_pool"].copy()
    cv_ref = c["conv_pool"].copy()
    ref = O.gdn_core_decode(p[:, :C], p[:, C + HV * D + HV:C + HV * D + 2 * HV],
                            p[:, C + HV * D:C + HV * D + HV], p[:, C:C + HV * D],
                            cv_ref[:, L], s_ref[:, L], ids, c["conv_w"], c["a_log"],
                            c["dt_bias"], c["norm_w"], HK, D, HV, D)
    got = host(out).reshape(bs, HV * D)
    assert np.abs(got - ref).max() <= OUT_ATOL
    s_got, cv_got = host(s_d), host(cv_d)
    assert state_rel(s_got[ids, L], s_ref[ids, L]) <= STATE_RTOL
    assert np.array_equal(cv_got, cv_ref)                  # the roll is a bit copy
    mask = np.ones(s_got.shape[0], bool)
    mask[ids] = False
    assert np.array_equal(s_got[mask], c["s_pool"][mask])
    assert np.array_equal(s_got[:, 0], c["s_pool"][:, 0])


@pytest.mark.parametrize("counters", [True, False])
@pytest.mark.parametrize("HK,HV,D,K,bs,pdt", CASES)
def test_decode_fused_equals_four_operators(ops, HK, HV, D, K, bs, pdt, counters):
    c = make_case(HK, HV, D, K, bs, seed=700 + bs + D)
    f_out, f_s, f_cv = run_fused(ops, c, pdt, counters)
    u_out, u_s, u_cv = run_four_ops(ops, c, pdt)
    torch.cuda.synchronize()
    assert torch.equal(f_cv, u_cv)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    if bs * HV >= 4 * sms:        # the sequence ran the full-tile recurrent kernel
        assert torch.equal(f_out, u_out)
        assert torch.equal(f_s, u_s)
    else:                         # column-split recurrent + separate norm: other sum order
        d = (f_out.float() - u_out.float()).abs()
        ulp = torch.maximum(f_out.float().abs(), u_out.float().abs()) * 2.0 ** -7 + 1e-3
        assert bool((d <= ulp).all())
        assert state_rel(host(f_s), host(u_s)) <= 1e-6


def test_decode_fused_two_steps_in_a_row(ops):
    """Two consecutive steps thread the conv state and the recurrent state."""
    HK, HV, D, K, bs = 4, 8, 128, 4, 40
    c1 = make_case(HK, HV, D, K, bs, seed=901)
    c2 = make_case(HK, HV, D, K, bs, seed=902)
    c2.update(s_pool=c1["s_pool"], conv_pool=c1["conv_pool"], ids=c1["ids"])
    for k in ("conv_w", "a_log", "dt_bias", "norm_w"):
        c2[k] = c1[k]
    proj1, proj2 = dev(c1["proj"], torch.bfloat16), dev(c2["proj"], torch.bfloat16)
    s_d, cv_d = dev(c1["s_pool"]), dev(c1["conv_pool"], torch.bfloat16)
    L, ids = 1, torch.as_tensor(c1["ids"], device=DEV)
    args = (cv_d[:, L], dev(c1["conv_w"], torch.bfloat16), dev(c1["a_log"]), dev(c1["dt_bias"]),
            s_d[:, L], ids, dev(c1["norm_w"], torch.bfloat16), 1e-6)
    outs = []
    for cc, pd in ((c1, proj1), (c2, proj2)):
        mixed, z, b, a = views(cc, pd)
        outs.append(host(ops.decode_fused(mixed, z, b, a, *args)))
    s_ref, cv_ref = c1["s_pool"].copy(), c1["conv_pool"].copy()
    C = c1["C"]
    for cc, got in zip((c1, c2), outs):
        p = cc["proj"]
        ref = O.gdn_core_decode(p[:, :C], p[:, C + HV * D + HV:C + HV * D + 2 * HV],
                                p[:, C + HV * D:C + HV * D + HV], p[:, C:C + HV * D],
                                cv_ref[:, L], s_ref[:, L], c1["ids"], c1["conv_w"],
                                c1["a_log"], c1["dt_bias"], c1["norm_w"], HK, D, HV, D)
        assert np.abs(got.reshape(bs, -1) - ref).max() <= OUT_ATOL
    assert np.array_equal(host(cv_d), cv_ref)
    assert state_rel(host(s_d)[c1["ids"], L], s_ref[c1["ids"], L]) <= STATE_RTOL


@pytest.mark.parametrize("counters", [True, False])
def test_decode_fused_bad_slot_is_flagged_not_touched(ops, counters):
    HK, HV, D, K, bs = 2, 4, 128, 4, 4
    c = make_case(HK, HV, D, K, bs, seed=950, slots_extra=0)
    slots = c["s_pool"].shape[0]
    c["ids"] = np.array([1, slots, -1, 2])             # rows 1 and 2 out of range
    ops.check_status()
    out, s_d, cv_d = run_fused(ops, c, torch.float32, counters)
    with pytest.raises(IndexError):
        ops.check_status()
    assert counters_zero(ops)
    s_got, cv_got = host(s_d), host(cv_d)
    keep = [0, 3]                                      # slots no valid row names
    assert np.array_equal(s_got[keep], c["s_pool"][keep])
    assert np.array_equal(cv_got[keep], c["conv_pool"][keep])
    assert not np.array_equal(s_got[1], c["s_pool"][1])


def test_decode_wait_that_runs_out_sets_timeout_and_returns(ops):
    """A bounded device wait that runs out: with the poll limit of the
    head-per-CTA form's wait for its state copy lowered to 0 (the test hook
    gdn_set_wait_limit), every CTA gives up at once, ORs GDN_STATUS_TIMEOUT,
    waits (normal limit) for the copy it has in flight and returns without
    writing any recurrent state.  The group counters stay zero, the context
    stays usable, and the next call with the normal limit matches the oracle
    (from the conv state the timed-out call left: its conv step had run)."""
    HK, HV, D, K, bs = 2, 4, 128, 4, 5
    c = make_case(HK, HV, D, K, bs, seed=971)
    ops.check_status()
    proj_d = dev(c["proj"], torch.bfloat16)
    mixed, z, b, a = views(c, proj_d)
    s_d, cv_d = dev(c["s_pool"]), dev(c["conv_pool"], torch.bfloat16)
    L, ids = c["layer"], torch.as_tensor(c["ids"], device=DEV)
    args = (cv_d[:, L], dev(c["conv_w"], torch.bfloat16), dev(c["a_log"]), dev(c["dt_bias"]),
            s_d[:, L], ids, dev(c["norm_w"], torch.bfloat16), 1e-6)
    ops.set_wait_limit(0)
    try:
        ops.decode_fused(mixed, z, b, a, *args, counters=True)
        torch.cuda.synchronize()
    finally:
        ops.set_wait_limit(None)
    with pytest.raises(ops._lib.GdnError):
        ops.check_status()
    assert counters_zero(ops)
    assert np.array_equal(host(s_d), c["s_pool"])          # no state was written
    cv_after = host(cv_d)
    out = ops.decode_fused(mixed, z, b, a, *args, counters=True)
    ops.check_status()
    s_ref, cv_ref = c["s_pool"].copy(), cv_after.copy()
    C, p = c["C"], c["proj"]
    ref = O.gdn_core_decode(p[:, :C], p[:, C + HV * D + HV:C + HV * D + 2 * HV],
                            p[:, C + HV * D:C + HV * D + HV], p[:, C:C + HV * D],
                            cv_ref[:, L], s_ref[:, L], c["ids"], c["conv_w"], c["a_log"],
                            c["dt_bias"], c["norm_w"], HK, D, HV, D)
    assert np.abs(host(out).reshape(bs, -1) - ref).max() <= OUT_ATOL
    assert state_rel(host(s_d)[c["ids"], L], s_ref[c["ids"], L]) <= STATE_RTOL
