"""GPU parity of the tensor-core chunk prefill at the shapes it is benchmarked
on, against the C restatement of the reference's chunk rule
(oracle/gdn_ref.c, fp32; it agrees with the fp64 numpy oracle to ~5e-7 on
long sequences, tests/test_cref.py).

Config-2 head shapes (16 QK heads x 128, 32 V heads x 128, chunk 64) with
sequences of 8192, 4097, 1000 and 65 tokens — 128 serial chunks through the
bf16 S / T operands on the longest chain — and one 32768-token sequence
(512 chunks) at 2 v-heads as a stand-in for the long-context config.  Both
tensor-core forms (split: per-chunk prep pass + chain; one-kernel) are
checked.  Tolerances from the path's spec: bf16 outputs max-abs <= 2e-2,
fp32 final states relative (Frobenius) error <= 1e-3 per slot, untouched
slots bit-exact.
"""
import numpy as np
import pytest
import torch

import inputs as I
from oracle import cref
from oracle import gdn_oracle as O

pytestmark = pytest.mark.gpu

OUT_ATOL = 2e-2
STATE_RTOL = 1e-3
DEV = "cuda:0"


@pytest.fixture(scope="module")
def ops(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    return pkg.ops


def _dev(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV).to(dtype)


def _long_case(lens, HK, HV, seed, fresh):
    """Seeded inputs (config-0 distributions, bf16-representable activations),
    a pool with canaries in every slot, the oracle's outputs and states."""
    D = 128
    N = sum(lens)
    q, k, v, g, beta = I.core_inputs(N, HK, D, HV, D, seed=seed)
    q, k, v, beta = (O.round_bf16(t) for t in (q, k, v, beta))
    r = I.rng(seed + 1)
    slots = len(lens) + 2
    pool = (r.standard_normal((slots, HV, D, D)) * 0.02).astype(np.float32)
    ids = r.permutation(slots)[:len(lens)]
    for i in fresh:                       # fresh prefills start from a zero state
        pool[ids[i]] = 0.0
    cu = I.cu_from_lens(lens)
    ref_pool = pool.copy()
    ref = cref.chunk_prefill(q, k, v, g, beta, ref_pool, ids, cu)
    return dict(q=q, k=k, v=v, g=g, beta=beta, pool=pool, ids=ids, cu=cu, ref=ref,
                ref_pool=ref_pool, lens=lens)


def _check(ops, c, split):
    pool_d = _dev(c["pool"], torch.float32)
    out = ops.chunk_gated_delta_rule_varlen(
        _dev(c["q"], torch.bfloat16), _dev(c["k"], torch.bfloat16),
        _dev(c["v"], torch.bfloat16), _dev(c["g"], torch.float32),
        _dev(c["beta"], torch.bfloat16), pool_d, _dev(c["ids"], torch.int64),
        _dev(c["cu"], torch.int32), max(c["lens"]), split=split)
    ops.check_status()
    got_out = out.float().cpu().numpy()
    got_pool = pool_d.cpu().numpy()
    err = float(np.abs(got_out - c["ref"]).max())
    rels = []
    for i, sl in enumerate(c["ids"]):
        if c["lens"][i]:
            d = got_pool[sl] - c["ref_pool"][sl]
            rels.append(float(np.linalg.norm(d) / max(np.linalg.norm(c["ref_pool"][sl]), 1e-30)))
    print(f"split={split} lens={c['lens'][:6]} out max-abs {err:.3e} "
          f"state rel max {max(rels):.3e}")
    assert err <= OUT_ATOL, f"output max-abs {err}"
    assert max(rels) <= STATE_RTOL, f"state relative errors {rels}"
    touched = [s for s, n in zip(c["ids"], c["lens"]) if n]
    untouched = np.setdiff1d(np.arange(c["pool"].shape[0]), touched)
    assert np.array_equal(got_pool[untouched], c["pool"][untouched])
    return got_out, got_pool


@pytest.fixture(scope="module")
def config2_case():
    # config-2 head shapes; the longest config-2 sequence, an odd length, a
    # mid length and a 65-token tail (one full chunk + one row); two fresh slots
    return _long_case([8192, 4097, 1000, 65], HK=16, HV=32, seed=2024, fresh=(0, 3))


@pytest.mark.parametrize("split", [True, False])
def test_chunk_config2_heads_long_sequences_vs_c_oracle(ops, config2_case, split):
    _check(ops, config2_case, split)


@pytest.mark.parametrize("split", [True, False])
def test_chunk_32k_sequence_vs_c_oracle(ops, split):
    """512 serial chunks on one chain (long-context stand-in), GQA pair."""
    c = _long_case([32768], HK=1, HV=2, seed=77, fresh=(0,))
    _check(ops, c, split)


def test_chunk_config2_split_and_one_kernel_forms_agree(ops, config2_case):
    """The two forms share every step's arithmetic: bit-identical at the
    config-2 shapes too."""
    a = _check(ops, config2_case, True)
    b = _check(ops, config2_case, False)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
