"""The C-ABI library loads, exports every symbol include/gdn_b200.h declares,
and rejects contract violations on the host before any CUDA call (so these
run without a GPU)."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gdn_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(gdn_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_path():
    syms = declared_symbols()
    for s in ("gdn_fused_g_beta", "gdn_conv_decode_step", "gdn_causal_conv_silu_varlen",
              "gdn_recurrent_inplace", "gdn_chunk_prefill_varlen", "gdn_rms_norm_gated",
              "gdn_abi_version", "gdn_last_error"):
        assert s in syms


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._lib.load()
    for s in declared_symbols():
        assert hasattr(lib, s), f"{s} declared in gdn_b200.h but not exported"
        assert s in pkg._lib.SIGNATURES, f"{s} has no ctypes signature"


def test_abi_version(pkg):
    lib = pkg._lib.load()
    m = re.search(r"#define GDN_ABI_VERSION (\d+)", open(HEADER).read())
    assert lib.gdn_abi_version() == int(m.group(1))


def _call(pkg, name, *args):
    lib = pkg._lib.load()
    rc = getattr(lib, name)(*args)
    return rc, lib.gdn_last_error().decode()


def test_host_validation_errors(pkg):
    L = pkg._lib
    # recurrent: unsupported head dims -> GDN_ERR_UNSUPPORTED
    rc, msg = _call(pkg, "gdn_recurrent_inplace", None, 96, None, 96, None, 96, None, None, None,
                    0, 1, None, None, 1, 1, 1, 96, 96, 0.1, None, 0, None, 1e-6, None, None)
    assert rc == L.GDN_ERR_UNSUPPORTED and "head dims" in msg
    # recurrent: HV not a multiple of HK -> invalid argument
    rc, msg = _call(pkg, "gdn_recurrent_inplace", None, 1024, None, 1024, None, 1024, None, None,
                    None, 1 << 20, 1, None, None, 1, 3, 4, 128, 128, 0.1, None, 0, None, 1e-6,
                    None, None)
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "multiple" in msg
    # recurrent: slot stride smaller than one slot
    rc, msg = _call(pkg, "gdn_recurrent_inplace", None, 512, None, 512, None, 512, None, None,
                    None, 100, 1, None, None, 1, 4, 4, 128, 128, 0.1, None, 0, None, 1e-6,
                    None, None)
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "slot_stride" in msg
    # conv: unsupported kernel width
    rc, msg = _call(pkg, "gdn_conv_decode_step", None, 64, None, 1000, 2, None, 1, 64, 5, None,
                    None, 64, None, None)
    assert rc == L.GDN_ERR_UNSUPPORTED
    # varlen conv: tokens without sequences
    rc, msg = _call(pkg, "gdn_causal_conv_silu_varlen", None, 64, None, 1000, 2, None, None, 0,
                    10, 64, 4, None, None, 64, None, None)
    assert rc == L.GDN_ERR_INVALID_ARGUMENT
    # gate: bad param dtype
    rc, msg = _call(pkg, "gdn_fused_g_beta", None, None, 8, 4, 8, None, None, 7, None, None,
                    None, None)
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "param_dtype" in msg
    # norm: unsupported dim
    rc, msg = _call(pkg, "gdn_rms_norm_gated", None, None, 96, 1, None, None, 4, 96, 1e-6, None)
    assert rc == L.GDN_ERR_UNSUPPORTED
    # chunk: unsupported dims
    rc, msg = _call(pkg, "gdn_chunk_prefill_varlen", None, 64, None, 64, None, 64, None, None,
                    None, 1 << 20, 2, None, None, 1, 1, 1, None, 1, 1, 32, 32, 0.1, None, 0, None,
                    1e-6, None, None)
    assert rc == L.GDN_ERR_UNSUPPORTED


def test_empty_calls_are_noops(pkg):
    L = pkg._lib
    assert _call(pkg, "gdn_recurrent_inplace", None, 512, None, 512, None, 1024, None, None, None,
                 1 << 20, 2, None, None, 0, 4, 8, 128, 128, 0.1, None, 0, None, 1e-6, None,
                 None)[0] == L.GDN_OK
    # fused norm without a weight is rejected on the host
    rc, msg = _call(pkg, "gdn_recurrent_inplace", None, 512, None, 512, None, 1024, None, None,
                    None, 1 << 20, 2, None, None, 0, 4, 8, 128, 128, 0.1, 1, 1024, None, 1e-6,
                    None, None)
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "norm" in msg
    assert _call(pkg, "gdn_fused_g_beta", None, None, 8, 0, 8, None, None, 0, None, None, None,
                 None)[0] == L.GDN_OK


def test_python_errors_map_from_codes(pkg):
    L = pkg._lib
    with pytest.raises(ValueError):
        L.check(L.GDN_ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(NotImplementedError):
        L.check(L.GDN_ERR_UNSUPPORTED, "x")
    with pytest.raises(RuntimeError):
        L.check(L.GDN_ERR_CUDA, "x")
