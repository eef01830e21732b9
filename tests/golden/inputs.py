"""Seeded synthetic inputs for the GDN parity cases (numpy only).

Shared by ``make_golden.py`` (which feeds them to the reference) and the
tests (which feed them to the oracle and the CUDA path).  Distributions follow
the workload description of config 0: q, k, v ~ N(0, 1); log-decay
g = -softplus(N(0,1)) * exp(A) with A ~ U(-1, 0) per v-head; beta =
sigmoid(N(0,1)).  Every generator takes an explicit seed and uses numpy's
PCG64 bit generator; the fixtures store a digest of the regenerated inputs so
a change of numpy's streams is caught instead of silently comparing against
different inputs.
"""
from __future__ import annotations

import hashlib

import numpy as np

# config 0: hidden 512, 4 QK heads x 64, 8 V heads x 64, conv kernel 4
C0 = dict(hidden=512, HK=4, DK=64, HV=8, DV=64, K=4, lens=(64, 97, 180, 256),
          n_decode=16, eps=1e-6)


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode()); h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()[:16]


def _round_bf16(x):
    """float32 -> nearest bf16 (ties to even), returned as float32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).reshape(np.shape(x))


def softplus(x):
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20))))


def core_inputs(N, HK, DK, HV, DV, seed=0):
    """q, k [N, HK, DK]; v [N, HV, DV]; g, beta [N, HV] (float32)."""
    r = rng(seed)
    q = r.standard_normal((N, HK, DK), dtype=np.float32)
    k = r.standard_normal((N, HK, DK), dtype=np.float32)
    v = r.standard_normal((N, HV, DV), dtype=np.float32)
    A = r.uniform(-1.0, 0.0, size=HV).astype(np.float32)
    g = (-softplus(r.standard_normal((N, HV), dtype=np.float32)) * np.exp(A)).astype(np.float32)
    beta = (1.0 / (1.0 + np.exp(-r.standard_normal((N, HV), dtype=np.float32)))).astype(np.float32)
    return q, k, v, g, beta


def cu_from_lens(lens):
    return np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)


def layer_weights(hidden, HK, DK, HV, DV, K, seed=1):
    """Random parameters of one GDN layer (tp = 1 layout)."""
    r = rng(seed)
    key_dim, value_dim = HK * DK, HV * DV
    conv_dim = 2 * key_dim + value_dim
    std = 0.02
    return dict(
        in_proj_qkv=(r.standard_normal((conv_dim, hidden), dtype=np.float32) * std),
        in_proj_z=(r.standard_normal((value_dim, hidden), dtype=np.float32) * std),
        in_proj_b=(r.standard_normal((HV, hidden), dtype=np.float32) * std),
        in_proj_a=(r.standard_normal((HV, hidden), dtype=np.float32) * std),
        conv1d=r.uniform(-0.5, 0.5, size=(conv_dim, 1, K)).astype(np.float32),
        A_log=r.uniform(-1.0, 0.0, size=HV).astype(np.float32),
        dt_bias=(r.standard_normal(HV, dtype=np.float32) * 0.5),
        norm=(1.0 + 0.1 * r.standard_normal(DV, dtype=np.float32)),
        out_proj=(r.standard_normal((hidden, value_dim), dtype=np.float32) * std),
    )


def layer_hidden(N, hidden, seed=2):
    return rng(seed).standard_normal((N, hidden), dtype=np.float32)


def recurrent_pool(slots, L, HV, D, seed=13):
    """State pool [slots, L, HV, D, D] ~ N(0, 0.02) for the in-place case."""
    return (rng(seed).standard_normal((slots, L, HV, D, D)) * 0.02).astype(np.float32)


def recurrent_step_inputs(bs, HK, HV, D, step):
    """(mixed [bs, 2*HK*D + HV*D], g [bs, HV], beta [bs, HV]) for one decode
    step; mixed and beta are bf16-representable."""
    q, k, v, g, beta = core_inputs(bs, HK, D, HV, D, seed=100 + step)
    mixed = np.concatenate([q.reshape(bs, -1), k.reshape(bs, -1), v.reshape(bs, -1)], 1)
    return _round_bf16(mixed), g, _round_bf16(beta)


def chunk_init_state(n, HV, DK, DV, seed=14):
    """Initial states for the chunk case; sequence 0 starts fresh (zero)."""
    init = (rng(seed).standard_normal((n, HV, DK, DV)) * 0.02).astype(np.float32)
    init[0] = 0.0
    return init


def layer_pools(slots, HV, DK, DV, conv_dim, K, seed=16):
    """s_pool [slots, 1, HV, DK, DV] fp32 and conv_pool [slots, 1, conv_dim,
    K-1] (bf16-representable) filled with canary values."""
    r = rng(seed)
    s = (r.standard_normal((slots, 1, HV, DK, DV)) * 0.02).astype(np.float32)
    conv = _round_bf16(r.standard_normal((slots, 1, conv_dim, K - 1)).astype(np.float32))
    return s, conv


# a two-layer decoder stack at config-0 shapes (both layers linear attention)
DEC = dict(layers=2, inter=1024, slots=6, ids=(5, 1, 3, 0))


def decoder_weights(hidden, inter, HK, DK, HV, DV, K, layers=2, seed=60):
    """Parameters of a stack of Qwen3.5 decoder layers whose token mixer is the
    GDN layer: {"<layer>.<parameter name>": array}, names as the reference's
    Qwen3_5DecoderLayer (linear_attn.*, mlp.*, *_layernorm.weight)."""
    out = {}
    gdn_names = dict(in_proj_qkv="linear_attn.in_proj_qkv.weight",
                     in_proj_z="linear_attn.in_proj_z.weight",
                     in_proj_b="linear_attn.in_proj_b.weight",
                     in_proj_a="linear_attn.in_proj_a.weight",
                     conv1d="linear_attn.conv1d.weight", A_log="linear_attn.A_log",
                     dt_bias="linear_attn.dt_bias", norm="linear_attn.norm.weight",
                     out_proj="linear_attn.out_proj.weight")
    for i in range(layers):
        W = layer_weights(hidden, HK, DK, HV, DV, K, seed=seed + i)
        for k, name in gdn_names.items():
            out[f"{i}.{name}"] = W[k]
        r = rng(seed + 100 + i)
        out[f"{i}.mlp.gate_up_proj.weight"] = (
            r.standard_normal((2 * inter, hidden), dtype=np.float32) * hidden ** -0.5)
        out[f"{i}.mlp.down_proj.weight"] = (
            r.standard_normal((hidden, inter), dtype=np.float32) * inter ** -0.5)
        # Gemma-style norms: the weight is applied as (1 + w)
        out[f"{i}.input_layernorm.weight"] = r.standard_normal(hidden, dtype=np.float32) * 0.1
        out[f"{i}.post_attention_layernorm.weight"] = (
            r.standard_normal(hidden, dtype=np.float32) * 0.1)
    return out
