"""The C restatement (oracle/gdn_ref.c) against the reference's golden
vectors and the numpy restatement."""
import os

import numpy as np
import pytest

import inputs as I
from oracle import cref
from oracle import gdn_oracle as O


@pytest.fixture(scope="module", autouse=True)
def _built():
    if not os.path.exists(cref.LIB_PATH):
        import subprocess
        subprocess.run(["make", "-s", "-C", os.path.dirname(cref.LIB_PATH) + "/.."], check=True)


def test_cref_chunk_and_decode_c0_golden(golden_dir):
    d = dict(np.load(os.path.join(golden_dir, "chunk_c0.npz")))
    c = I.C0
    lens = c["lens"]
    q, k, v, g, beta = I.core_inputs(sum(lens), c["HK"], c["DK"], c["HV"], c["DV"], seed=0)
    pool = I.chunk_init_state(len(lens), c["HV"], c["DK"], c["DV"])
    out = cref.chunk_prefill(q, k, v, g, beta, pool, np.arange(len(lens)), I.cu_from_lens(lens))
    np.testing.assert_allclose(out, d["out"], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(pool, d["state"], rtol=1e-4, atol=2e-6)
    S = d["state"].copy()
    for s in range(c["n_decode"]):
        dq, dk, dv, dg, db = I.core_inputs(len(lens), c["HK"], c["DK"], c["HV"], c["DV"],
                                           seed=1000 + s)
        o = cref.recurrent_inplace(dq, dk, dv, dg, db, S, np.arange(len(lens)))
        np.testing.assert_allclose(o, d["dec_out"][s], rtol=1e-4, atol=2e-5)
    np.testing.assert_allclose(S, d["dec_state"], rtol=1e-4, atol=2e-6)


def test_cref_matches_numpy_with_slots_and_d128():
    """HK 2 -> HV 4 at head dim 128, permuted slots, ragged lengths incl. 1."""
    lens = [1, 2, 63, 64, 65, 130]
    N = sum(lens)
    q, k, v, g, beta = I.core_inputs(N, 2, 128, 4, 128, seed=21)
    pool = (I.rng(22).standard_normal((9, 4, 128, 128)) * 0.02).astype(np.float32)
    ids = np.array([8, 3, 0, 5, 1, 7])
    cu = I.cu_from_lens(lens)
    p1, p2 = pool.copy(), pool.copy()
    o1 = cref.chunk_prefill(q, k, v, g, beta, p1, ids, cu)
    o2 = O.chunk_prefill_varlen(q, k, v, g, beta, p2, ids, cu)
    np.testing.assert_allclose(o1, o2, rtol=2e-4, atol=2e-5)
    np.testing.assert_allclose(p1, p2, rtol=2e-4, atol=2e-6)
    untouched = np.setdiff1d(np.arange(9), ids)
    assert np.array_equal(p1[untouched], pool[untouched])
