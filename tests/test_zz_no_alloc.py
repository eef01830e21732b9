"""gdn_decode_fused_static — the fused decode core with its group counters in a
static device array instead of caller scratch — against gdn_decode_fused with
caller scratch, both through the C ABI: three calls in a row on the same
pools, each with a different permutation of slot ids, so a counter left
non-zero by one call would change which CTA rolls the shared q/k conv taps of
the next.  Both entry points run the same kernels, so outputs, states and
conv-state rolls must agree bit for bit (which also meets the path's bf16 and
fp32 tolerances).  Batches that fit one wave use the counters; the larger one
runs the persistent form.  Self-contained, so it passes alone and after every
other test (the static counters start and end at zero)."""
import ctypes

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
def lib(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    return pkg


def _dev(a, dtype=torch.float32):
    return torch.from_numpy(np.array(a, np.float32, order="C", copy=True)).to(DEV).to(dtype)


def _case(HK, HV, D, K, bs, seed, calls=3):
    r = I.rng(seed)
    C = (2 * HK + HV) * D
    W = C + HV * D + 2 * HV + 8
    projs = [O.round_bf16(r.standard_normal((bs, W)).astype(np.float32)) for _ in range(calls)]
    slots = bs + 3
    s_pool = (r.standard_normal((slots, 2, HV, D, D)) * 0.02).astype(np.float32)
    conv_pool = O.round_bf16(r.standard_normal((slots, 2, C, K - 1)).astype(np.float32))
    conv_w = O.round_bf16(r.uniform(-0.6, 0.6, (C, K)).astype(np.float32))
    a_log = r.uniform(-1.0, 1.0, HV).astype(np.float32)
    dt_bias = r.uniform(-0.5, 0.5, HV).astype(np.float32)
    norm_w = O.round_bf16((1 + 0.1 * r.standard_normal(D)).astype(np.float32))
    ids = [r.permutation(slots)[:bs] for _ in range(calls)]   # new slot ids every call
    return C, projs, s_pool, conv_pool, conv_w, a_log, dt_bias, norm_w, ids


def _run_static(pkg, proj, C, HK, HV, D, K, cv, w, al, dt, sp, ids, nw, out):
    L = pkg._lib
    bs = proj.shape[0]
    mixed = proj[:, :C]
    z = proj[:, C:C + HV * D]
    b = proj[:, C + HV * D:C + HV * D + HV]
    a = proj[:, C + HV * D + HV:C + HV * D + 2 * HV]
    status = pkg.ops.status_word(proj.device)
    rc = L.load().gdn_decode_fused_static(
        mixed.data_ptr(), mixed.stride(0), z.data_ptr(), z.stride(0), b.data_ptr(), a.data_ptr(),
        b.stride(0), cv.data_ptr(), cv.stride(0), w.data_ptr(), K, al.data_ptr(), dt.data_ptr(),
        L.GDN_DTYPE_F32, sp.data_ptr(), sp.stride(0), sp.shape[0], ids.data_ptr(), nw.data_ptr(),
        ctypes.c_float(1e-6), out.data_ptr(), bs, HK, HV, D, ctypes.c_float(D ** -0.5),
        status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == L.GDN_OK, L.load().gdn_last_error().decode()


@pytest.mark.parametrize("HK,HV,D,K,bs", [
    (16, 32, 128, 4, 8),     # 256 units: one wave, the static counters are used
    (2, 8, 64, 3, 20),       # four v-heads per k-head share the counters, head dim 64
    (16, 32, 128, 4, 64),    # 2048 units: several waves, the persistent form
])
def test_static_scratch_equals_caller_scratch_three_calls(lib, HK, HV, D, K, bs):
    C, projs, s_pool, conv_pool, conv_w, a_log, dt_bias, norm_w, ids = _case(HK, HV, D, K, bs,
                                                                             seed=1200 + bs)
    ops = lib.ops
    w = _dev(conv_w, torch.bfloat16)
    al, dt = _dev(a_log), _dev(dt_bias)
    nw = _dev(norm_w, torch.bfloat16)
    s_a, s_b = _dev(s_pool), _dev(s_pool)
    c_a, c_b = _dev(conv_pool, torch.bfloat16), _dev(conv_pool, torch.bfloat16)
    for step in range(len(projs)):              # calls in a row thread both states
        proj = _dev(projs[step], torch.bfloat16)
        ids_d = torch.as_tensor(ids[step], device=DEV, dtype=torch.int64)
        ref = ops.decode_fused(proj[:, :C], proj[:, C:C + HV * D].view(bs, HV, D),
                               proj[:, C + HV * D:C + HV * D + HV],
                               proj[:, C + HV * D + HV:C + HV * D + 2 * HV], c_a[:, 1], w, al,
                               dt, s_a[:, 1], ids_d, nw, 1e-6, counters=True)
        got = torch.empty(bs, HV, D, dtype=torch.bfloat16, device=DEV)
        _run_static(lib, proj, C, HK, HV, D, K, c_b[:, 1], w, al, dt, s_b[:, 1], ids_d, nw, got)
        torch.cuda.synchronize()
        assert (got.float() - ref.float()).abs().max().item() <= OUT_ATOL, f"call {step}"
        rel = ((s_a - s_b).norm() / s_a.norm()).item()
        assert rel <= STATE_RTOL, f"call {step}: state rel {rel}"
        assert torch.equal(got, ref), f"call {step}: outputs differ"
        assert torch.equal(s_a, s_b), f"call {step}: states differ"
        assert torch.equal(c_a, c_b), f"call {step}: conv state"
    ops.check_status()


def test_static_scratch_rejects_batches_beyond_its_size(lib):
    L = lib._lib
    lib_ = L.load()
    rc = lib_.gdn_decode_fused_static(
        None, 8192, None, 4096, None, None, 64, None, 8192 * 3, None, 4, None, None, 0, None,
        32 * 128 * 128, 2049, None, None, ctypes.c_float(1e-6), None, 2048, 16, 32, 128,
        ctypes.c_float(0.1), None, None)
    assert rc == L.GDN_ERR_UNSUPPORTED
    assert "static scratch" in lib_.gdn_last_error().decode()
