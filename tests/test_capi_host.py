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
              "gdn_conv_gate_varlen", "gdn_recurrent_inplace", "gdn_chunk_prefill_varlen",
              "gdn_rms_norm_gated", "gdn_decode_fused", "gdn_abi_version", "gdn_last_error"):
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
    # conv + gate: the gate's checks, then the conv's (named after the combined call)
    fake = 1 << 20                                   # aligned, never dereferenced
    conv = (fake, 64, fake, 1000, 2, fake, fake, 1, 10, 64, 4, fake, fake, 64)
    rc, msg = _call(pkg, "gdn_conv_gate_varlen", *conv, fake, fake, 8, 8, fake, fake, 7, fake,
                    fake, None, None)
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "param_dtype" in msg
    rc, msg = _call(pkg, "gdn_conv_gate_varlen", *conv, fake, fake, 4, 8, fake, fake, 0, fake,
                    fake, None, None)
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "row stride" in msg
    rc, msg = _call(pkg, "gdn_conv_gate_varlen", *conv, None, fake, 8, 8, fake, fake, 0, fake,
                    fake, None, None)
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "null pointer" in msg
    rc, msg = _call(pkg, "gdn_conv_gate_varlen", fake, 64, fake, 1000, 2, fake, fake, 0, 10, 64,
                    4, fake, fake, 64, fake, fake, 8, 8, fake, fake, 0, fake, fake, None, None)
    assert rc == L.GDN_ERR_INVALID_ARGUMENT
    assert msg.startswith("gdn_conv_gate_varlen:") and "without sequences" in msg
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
                    1e-6, None, 0, None, None)
    assert rc == L.GDN_ERR_UNSUPPORTED


def test_chunk_workspace_size_and_too_small_workspace(pkg):
    """The split chunk prefill's scratch: one 17,664-byte block per (chunk, v-head) for up
    to cap = (n_tokens + 63 n_seqs) / 64 chunks, after the int32 chunk starts and the
    int2 per-chunk rows (each part 256-byte padded); none for head dim 64.  A workspace
    below that size is rejected before any launch."""
    L = pkg._lib
    lib = L.load()
    n, seqs, hv = 282505, 64, 32
    cap = (n + 63 * seqs) // 64
    a256 = lambda x: (x + 255) // 256 * 256
    want = a256((seqs + 1) * 4) + a256(cap * 8) + cap * hv * 17664
    assert lib.gdn_chunk_prefill_workspace_bytes(n, seqs, hv, 128, 128) == want
    assert lib.gdn_chunk_prefill_workspace_bytes(n, seqs, hv, 64, 64) == 0
    assert lib.gdn_chunk_prefill_workspace_bytes(0, seqs, hv, 128, 128) == 0
    fake = 1 << 20                                   # aligned, never dereferenced
    rc, msg = _call(pkg, "gdn_chunk_prefill_varlen", fake, 512, fake, 512, fake, 1024, fake,
                    fake, fake, 8 * 128 * 128, 4, fake, fake, 2, 300, 200, fake, 4, 8, 128, 128,
                    0.1, None, 0, None, 1e-6, fake, 1000, None, None)
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "workspace" in msg


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
    # conv + gate with no sequences and no tokens: nothing to launch
    assert _call(pkg, "gdn_conv_gate_varlen", None, 64, None, 1000, 2, None, None, 0, 0, 64, 4,
                 None, None, 64, None, None, 8, 8, None, None, 0, None, None, None,
                 None)[0] == L.GDN_OK


def test_python_errors_map_from_codes(pkg):
    L = pkg._lib
    with pytest.raises(ValueError):
        L.check(L.GDN_ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(NotImplementedError):
        L.check(L.GDN_ERR_UNSUPPORTED, "x")
    with pytest.raises(RuntimeError):
        L.check(L.GDN_ERR_CUDA, "x")


def _decode_fused_args(**kw):
    """gdn_decode_fused arguments for a bs-1 call of HK=2, HV=4, D=128, K=4
    with null pointers (host checks only), overridable by name."""
    a = dict(mixed=None, ms=8192, z=None, zs=4096, b=None, a=None, abs_=8, conv_pool=None,
             conv_ss=8192 * 3, conv_w=None, K=4, a_log=None, dt_bias=None, pdt=0, s_pool=None,
             slot_stride=4 * 128 * 128, num_slots=2, ids=None, nw=None, eps=1e-6, out=None, bs=1,
             HK=2, HV=4, D=128, scale=0.1, counters=None, status=None, stream=None)
    a.update(kw)
    return list(a.values())


def test_decode_fused_host_validation(pkg):
    L = pkg._lib
    rc, msg = _call(pkg, "gdn_decode_fused", *_decode_fused_args(D=96))
    assert rc == L.GDN_ERR_UNSUPPORTED and "head dim" in msg
    rc, msg = _call(pkg, "gdn_decode_fused", *_decode_fused_args(HK=1, HV=8, zs=8192,
                                                                  ms=10 * 128,
                                                                  conv_ss=10 * 128 * 3,
                                                                  slot_stride=8 * 128 * 128))
    assert rc == L.GDN_ERR_UNSUPPORTED and "v-heads per k-head" in msg
    rc, msg = _call(pkg, "gdn_decode_fused", *_decode_fused_args(HV=3))
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "multiple" in msg
    rc, msg = _call(pkg, "gdn_decode_fused", *_decode_fused_args(K=5))
    assert rc == L.GDN_ERR_UNSUPPORTED and "conv kernel" in msg
    rc, msg = _call(pkg, "gdn_decode_fused", *_decode_fused_args(pdt=7))
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "param_dtype" in msg
    rc, msg = _call(pkg, "gdn_decode_fused", *_decode_fused_args(slot_stride=1000))
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "slot_stride" in msg
    rc, msg = _call(pkg, "gdn_decode_fused", *_decode_fused_args(conv_ss=100))
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "conv_slot_stride" in msg
    rc, msg = _call(pkg, "gdn_decode_fused", *_decode_fused_args(ms=100))
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "row stride" in msg
    # zero rows: nothing to do, no pointer is touched
    rc, msg = _call(pkg, "gdn_decode_fused", *_decode_fused_args(bs=0))
    assert rc == L.GDN_OK
    # rows with null pointers are rejected before any launch
    rc, msg = _call(pkg, "gdn_decode_fused", *_decode_fused_args())
    assert rc == L.GDN_ERR_INVALID_ARGUMENT and "null" in msg


def test_integration_ctypes_stubs_match_the_signature_table(pkg):
    """The ctypes bindings printed in INTEGRATION.md (what a maintainer of the
    reference would paste) list the same argument types as the package's own
    table, which the symbol test above ties to the header."""
    L = pkg._lib
    names = {L.vp: "vp", L.i32: "i32", L.i64: "i64", L.f32: "f32"}
    doc = re.sub(r"#[^\n]*", "", open(os.path.join(ROOT, "INTEGRATION.md")).read())
    stubs = re.findall(r"lib\.(gdn_\w+)\.argtypes = \[(.*?)\]", doc, flags=re.S)
    assert len(stubs) >= 4
    for name, body in stubs:
        assert re.findall(r"\b(vp|i32|i64|f32)\b", body) == [names[t] for t in L.SIGNATURES[name]], \
            name
