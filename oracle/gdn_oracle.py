"""CPU oracle for the GatedDeltaNet (GDN) layer path — TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it.
The CUDA path in ``nano-vllm-extend_b200/`` never routes through it.

It restates, in numpy, the algorithms of the reference's GDN layer
(sileaver/nano-vllm-extend, ``nanovllm/models/qwen3_5.py``).  Every function
cites the reference lines it follows.  Arithmetic is carried in the dtype of
the inputs' float view (``np.float32`` mirrors the reference's fp32 maths;
``np.float64`` gives a higher-precision yardstick).  Activations in "model
dtype" are emulated with :func:`round_bf16` where the reference rounds to
bf16.

Parity of this restatement is pinned against golden vectors produced by the
reference itself (``tests/golden/make_golden.py`` imports the reference's own
functions and kernels on CPU); ``tests/test_oracle_golden.py`` checks it.
"""
from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# bf16 emulation
# ---------------------------------------------------------------------------


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 (round-half-to-even), returned
    as float32.  This is what ``tensor.to(torch.bfloat16)`` does on finite
    values."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    bias = 0x7FFF + ((u >> 16) & 1)
    r = ((u + bias) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32).reshape(x.shape)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 array (already bf16-representable) -> uint16 bit patterns."""
    x = np.ascontiguousarray(round_bf16(x), dtype=np.float32)
    return (x.view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def _silu(x):
    return x * _sigmoid(x)


# ---------------------------------------------------------------------------
# (b) fused g / beta gate — qwen3_5.py:320-360 (_gdn_g_beta_kernel, fused_g_beta)
# ---------------------------------------------------------------------------


def fused_g_beta(b, a, a_log, dt_bias, mask=None, act_round=round_bf16):
    """g = -exp(A_log[h]) * softplus(a + dt_bias[h]) in fp32 (softplus is
    ``log(1 + exp(z))`` with threshold 20, as the kernel at qwen3_5.py:336-338
    writes it), zero where ``mask`` is False; beta = sigmoid(b) rounded to the
    activation dtype (qwen3_5.py:340-343).

    b, a: [..., Vh]; a_log, dt_bias: [Vh]; mask: [...] bool or None.
    Returns (g float32 [..., Vh], beta [..., Vh])."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    al = np.asarray(a_log, np.float32)
    dt = np.asarray(dt_bias, np.float32)
    z = a + dt
    with np.errstate(over="ignore"):
        sp = np.where(z > 20.0, z, np.log(np.float32(1.0) + np.exp(z)))
    g = (-np.exp(al) * sp).astype(np.float32)
    if mask is not None:
        g = np.where(np.asarray(mask)[..., None], g, np.float32(0.0))
    beta = _sigmoid(b).astype(np.float32)
    if act_round is not None:
        beta = act_round(beta)
    return g.astype(np.float32), beta


# ---------------------------------------------------------------------------
# (a) causal conv1d + SiLU
# ---------------------------------------------------------------------------


def conv_decode_step(x, conv_pool, ids, weight, act_round=round_bf16):
    """Single-token depthwise causal conv + SiLU with in-place state roll —
    qwen3_5.py:515-558 (_conv_decode_step_kernel / conv_decode_step).

    acc = x*w[K-1] + sum_{i<K-1} s[i]*w[i] (fp32, that order, :538-542);
    y = silu(acc); the slot's state then rolls to [s1, .., s_{K-2}, x]
    (:545-547).  x [n, C]; conv_pool [slots, C, K-1] (mutated at rows ids);
    weight [C, K].  Returns y [n, C]."""
    x = np.asarray(x, np.float32)
    w = np.asarray(weight, np.float32)
    K = w.shape[-1]
    y = np.empty_like(x)
    for n, slot in enumerate(np.asarray(ids, np.int64)):
        s = conv_pool[slot].astype(np.float32)          # [C, K-1]
        acc = x[n] * w[:, K - 1]
        for i in range(K - 1):
            acc = acc + s[:, i] * w[:, i]
        y[n] = _silu(acc)
        new = np.concatenate([s[:, 1:], x[n][:, None]], axis=1)
        conv_pool[slot] = new.astype(conv_pool.dtype)
    if act_round is not None:
        y = act_round(y)
    return y


def causal_conv_silu_varlen(x, conv_pool, ids, cu_seqlens, weight,
                            act_round=round_bf16):
    """Varlen depthwise causal conv + SiLU over flat rows, state rolled in
    place by slot — qwen3_5.py:402-473 (_causal_conv_silu_varlen_kernel),
    restated for any channel count (the reference's [3, N, C/3] output slab
    is a layout choice; the values are those of y [N, C] here).

    Sequence r owns rows [cu[r], cu[r+1]).  For its token t:
    acc = sum_{i<K} w[c,i] * win[t-K+1+i] in that order (:438-446), where win
    is [state | x] and the state supplies positions < 0.  After the tokens,
    the slot's state becomes the last K-1 entries of [state | x] (:450-456).
    x [N, C]; conv_pool [slots, C, K-1] (mutated at rows ids); weight [C, K].
    Returns y [N, C]."""
    x = np.asarray(x, np.float32)
    w = np.asarray(weight, np.float32)
    K = w.shape[-1]
    cu = np.asarray(cu_seqlens, np.int64)
    y = np.zeros_like(x)
    for r, slot in enumerate(np.asarray(ids, np.int64)):
        t0, t1 = int(cu[r]), int(cu[r + 1])
        st = conv_pool[slot].astype(np.float32)           # [C, K-1]
        win = np.concatenate([st.T, x[t0:t1]], axis=0)    # [K-1+T, C]
        T = t1 - t0
        acc = np.zeros((T, x.shape[1]), np.float32)
        for i in range(K):
            acc = acc + win[i:i + T] * w[:, i]
        y[t0:t1] = _silu(acc)
        conv_pool[slot] = win[-(K - 1):].T.astype(conv_pool.dtype)
    if act_round is not None:
        y = act_round(y)
    return y


def causal_conv_silu_padded(x, state, weight, endp, act_round=round_bf16):
    """Padded conv over x [n, C, T] with per-row ENDP writeback —
    qwen3_5.py:249-317 (_causal_conv_silu_kernel).  state [n, C, K-1] is
    rolled in place at the row's ENDP (last real position, -1 = skip)."""
    x = np.asarray(x, np.float32)
    w = np.asarray(weight, np.float32)
    n, C, T = x.shape
    K = w.shape[-1]
    y = np.zeros_like(x)
    for r in range(n):
        st = state[r].astype(np.float32)                  # [C, K-1]
        win = np.concatenate([st, x[r]], axis=1)          # [C, K-1+T]
        acc = np.zeros((C, T), np.float32)
        for i in range(K):
            acc = acc + win[:, i:i + T] * w[:, i:i + 1]
        y[r] = _silu(acc)
        e = int(endp[r])
        if e >= 0:
            state[r] = win[:, e:e + K - 1].astype(state.dtype)
    if act_round is not None:
        y = act_round(y)
    return y


# ---------------------------------------------------------------------------
# l2norm, recurrent decode, chunked prefill
# ---------------------------------------------------------------------------


def l2norm(x, eps=1e-6):
    """x * rsqrt(sum(x*x) + eps) over the last dim — qwen3_5.py:134-137."""
    x = np.asarray(x)
    return x * (1.0 / np.sqrt((x * x).sum(-1, keepdims=True) + x.dtype.type(eps)))


def recurrent_step(q, k, v, g, beta, state, dtype=np.float32):
    """One gated-delta-rule step — qwen3_5.py:616-651
    (_torch_recurrent_gated_delta_rule), head-mapped as the reference's
    repeat_interleave does (qwen3_5.py:1002-1005: v-head h reads k-head
    h // (HV/HK)).

    q, k [B, HK, DK]; v [B, HV, DV]; g, beta [B, HV]; state [B, HV, DK, DV].
    Returns (out [B, HV, DV], new_state) in ``dtype``."""
    q = np.asarray(q, dtype); k = np.asarray(k, dtype); v = np.asarray(v, dtype)
    g = np.asarray(g, dtype); beta = np.asarray(beta, dtype)
    S = np.asarray(state, dtype)
    HV, HK = v.shape[1], k.shape[1]
    rep = HV // HK
    q = np.repeat(l2norm(q), rep, axis=1)
    k = np.repeat(l2norm(k), rep, axis=1)
    q = q * dtype(k.shape[-1] ** -0.5)
    S = S * np.exp(g)[..., None, None]
    kv = (S * k[..., :, None]).sum(-2)
    delta = (v - kv) * beta[..., None]
    S = S + k[..., :, None] * delta[..., None, :]
    out = (S * q[..., :, None]).sum(-2)
    return out, S


def recurrent_inplace(q, k, v, g, beta, s_pool, ids, dtype=np.float32):
    """In-place decode by pool slot — qwen3_5.py:561-613
    (_recurrent_inplace_kernel): state rows s_pool[ids[b]] are read, updated
    and written back; other slots are untouched.  Returns out [B, HV, DV]."""
    ids = np.asarray(ids, np.int64)
    out, new = recurrent_step(q, k, v, g, beta, s_pool[ids], dtype)
    s_pool[ids] = new.astype(s_pool.dtype)
    return out


def _solve_unit_lower(attn):
    """Row-by-row forward substitution of the chunk's strictly-lower matrix,
    exactly as qwen3_5.py:196-200: for i: attn[i,:i] += attn[i,:i] @ attn[:i,:i];
    then attn += I.  attn [..., C, C]."""
    attn = attn.copy()
    C = attn.shape[-1]
    for i in range(1, C):
        row = attn[..., i, :i].copy()
        sub = attn[..., :i, :i].copy()
        attn[..., i, :i] = row + (row[..., :, None] * sub).sum(-2)
    return attn + np.eye(C, dtype=attn.dtype)


def chunk_gated_delta_rule(q, k, v, g, beta, initial_state=None,
                           chunk_size=64, dtype=np.float32):
    """Chunked gated delta rule for ONE sequence — qwen3_5.py:152-227
    (_torch_chunk_gated_delta_rule), head-mapped by h_k = h_v // (HV/HK).

    q, k [T, HK, DK]; v [T, HV, DV]; g, beta [T, HV]; initial_state
    [HV, DK, DV] or None.  Returns (out [T, HV, DV], final_state
    [HV, DK, DV]) in ``dtype``.  Steps: l2norm q/k (:165-166), pad T to the
    chunk (:173-178), q *= DK^-0.5 (:181-182), beta-scaled k/v (:183-184),
    in-chunk cumsum of g (:193), decay mask (:194), strictly-lower
    -(k_beta k^T * decay) (:195), forward substitution (:196-200),
    U = attn @ v_beta and W = attn @ (k_beta * exp(g)) (:201-202), then the
    sequential chunk loop (:211-222)."""
    dt = dtype
    T, HK, DK = k.shape
    HV, DV = v.shape[1], v.shape[2]
    rep = HV // HK
    q = np.repeat(l2norm(np.asarray(q, dt)), rep, axis=1).transpose(1, 0, 2)
    k = np.repeat(l2norm(np.asarray(k, dt)), rep, axis=1).transpose(1, 0, 2)
    v = np.asarray(v, dt).transpose(1, 0, 2)
    beta = np.asarray(beta, dt).T
    g = np.asarray(g, dt).T
    C = chunk_size
    pad = (C - T % C) % C
    if pad:
        q = np.pad(q, ((0, 0), (0, pad), (0, 0)))
        k = np.pad(k, ((0, 0), (0, pad), (0, 0)))
        v = np.pad(v, ((0, 0), (0, pad), (0, 0)))
        beta = np.pad(beta, ((0, 0), (0, pad)))
        g = np.pad(g, ((0, 0), (0, pad)))
    Tp = T + pad
    nc = Tp // C
    q = q * dt(DK ** -0.5)
    v_beta = v * beta[..., None]
    k_beta = k * beta[..., None]
    q, k, v, k_beta, v_beta = [x.reshape(HV, nc, C, x.shape[-1])
                               for x in (q, k, v, k_beta, v_beta)]
    g = g.reshape(HV, nc, C).cumsum(-1)
    diff = g[..., :, None] - g[..., None, :]
    tril = np.tril(np.ones((C, C), bool))
    decay = np.where(tril, np.exp(np.where(tril, diff, 0)), 0).astype(dt)
    strict = np.tril(np.ones((C, C), bool), -1)
    attn = np.where(strict, -((k_beta @ k.swapaxes(-1, -2)) * decay), 0).astype(dt)
    attn = _solve_unit_lower(attn)
    u = attn @ v_beta
    w = attn @ (k_beta * np.exp(g)[..., None])
    S = (np.zeros((HV, DK, DV), dt) if initial_state is None
         else np.asarray(initial_state, dt).copy())
    out = np.zeros((HV, nc, C, DV), dt)
    for i in range(nc):
        qi, ki = q[:, i], k[:, i]
        a = (qi @ ki.swapaxes(-1, -2)) * decay[:, i]
        v_new = u[:, i] - w[:, i] @ S
        inter = (qi * np.exp(g[:, i])[..., None]) @ S
        out[:, i] = inter + a @ v_new
        gl = g[:, i, -1]
        S = (S * np.exp(gl)[:, None, None]
             + (ki * np.exp(gl[:, None] - g[:, i])[..., None]).swapaxes(-1, -2) @ v_new)
    out = out.reshape(HV, Tp, DV)[:, :T].transpose(1, 0, 2)
    return out, S


def chunk_prefill_varlen(q, k, v, g, beta, s_pool, ids, cu_seqlens,
                         chunk_size=64, dtype=np.float32):
    """Varlen chunked prefill with the state read from and written back to
    pool slots: the composition the reference performs at
    qwen3_5.py:1039-1077 (gather s_cache[ids], chunk rule per sequence,
    scatter) and :956-961 (varlen form).  q, k [N, HK, DK]; v [N, HV, DV];
    g, beta [N, HV].  Returns out [N, HV, DV]; s_pool rows ids are updated."""
    cu = np.asarray(cu_seqlens, np.int64)
    out = np.zeros((q.shape[0], v.shape[1], v.shape[2]), dtype)
    for r, slot in enumerate(np.asarray(ids, np.int64)):
        a, b = int(cu[r]), int(cu[r + 1])
        if b == a:
            continue
        o, S = chunk_gated_delta_rule(q[a:b], k[a:b], v[a:b], g[a:b], beta[a:b],
                                      s_pool[slot], chunk_size, dtype)
        out[a:b] = o
        s_pool[slot] = S.astype(s_pool.dtype)
    return out


# ---------------------------------------------------------------------------
# gated RMSNorm — qwen3_5.py:121-131 (_rms_gated_forward), :697-709
# ---------------------------------------------------------------------------


def rms_norm_gated(x, gate, weight, eps=1e-6, act_round=round_bf16):
    """y = (w * to_act(x * rsqrt(mean(x^2) + eps))) * silu(gate), rounded to
    the activation dtype at the points the reference rounds (:127-131):
    the normalised x is rounded before the weight multiply, the weighted
    product is rounded again (bf16 * bf16 -> bf16), and the final fp32
    product is rounded once more.  x, gate [..., D]; weight [D]."""
    r = act_round if act_round is not None else (lambda t: t)
    x = np.asarray(x, np.float32)
    var = (x * x).mean(-1, keepdims=True)
    xn = x * (1.0 / np.sqrt(var + np.float32(eps)))
    xw = r(np.asarray(weight, np.float32) * r(xn))
    return r(xw * _silu(np.asarray(gate, np.float32)))


# ---------------------------------------------------------------------------
# the full layer core (after the input projections, before out_proj)
# ---------------------------------------------------------------------------


def gdn_core_decode(mixed_qkv, a, b, z, conv_pool, s_pool, ids, conv_w, a_log,
                    dt_bias, norm_w, HK, DK, HV, DV, eps=1e-6,
                    act_round=round_bf16):
    """The decode (T == 1) branch of Qwen3_5GatedDeltaNet._gdn_padded,
    qwen3_5.py:974-980 (g/beta), :1008-1026 (conv step + split + in-place
    recurrent), :1083-1085 (gated norm).  mixed_qkv [n, conv_dim] is the
    in_proj_qkv output; a, b [n, HV]; z [n, HV*DV].  Returns the normed core
    [n, HV*DV] that out_proj consumes."""
    n = mixed_qkv.shape[0]
    g, beta = fused_g_beta(b, a, a_log, dt_bias, None, act_round)
    y = conv_decode_step(mixed_qkv, conv_pool, ids, conv_w, act_round)
    kd = HK * DK
    q = y[:, :kd].reshape(n, HK, DK)
    k = y[:, kd:2 * kd].reshape(n, HK, DK)
    v = y[:, 2 * kd:].reshape(n, HV, DV)
    o = recurrent_inplace(q, k, v, g, beta, s_pool, ids)
    if act_round is not None:
        o = act_round(o)
    core = rms_norm_gated(o, np.asarray(z, np.float32).reshape(n, HV, DV),
                          norm_w, eps, act_round)
    return core.reshape(n, HV * DV)


def gdn_core_prefill(mixed_qkv, a, b, z, conv_pool, s_pool, ids, cu_seqlens,
                     conv_w, a_log, dt_bias, norm_w, HK, DK, HV, DV, eps=1e-6,
                     act_round=round_bf16, chunk_size=64):
    """The varlen prefill composition, qwen3_5.py:922-963 (g/beta, varlen
    conv with slot state, chunk rule with slot state, gated norm), with the
    conv output split into q | k | v columns (key_dim, key_dim, value_dim) as
    split_qkv does at :997-1001.  Returns the normed core [N, HV*DV]."""
    N = mixed_qkv.shape[0]
    g, beta = fused_g_beta(b, a, a_log, dt_bias, None, act_round)
    y = causal_conv_silu_varlen(mixed_qkv, conv_pool, ids, cu_seqlens, conv_w,
                                act_round)
    kd = HK * DK
    q = y[:, :kd].reshape(N, HK, DK)
    k = y[:, kd:2 * kd].reshape(N, HK, DK)
    v = y[:, 2 * kd:].reshape(N, HV, DV)
    o = chunk_prefill_varlen(q, k, v, g, beta, s_pool, ids, cu_seqlens,
                             chunk_size)
    if act_round is not None:
        o = act_round(o)
    core = rms_norm_gated(o, np.asarray(z, np.float32).reshape(N, HV, DV),
                          norm_w, eps, act_round)
    return core.reshape(N, HV * DV)


# ---------------------------------------------------------------------------
# the whole layer: projections + core + out_proj
# ---------------------------------------------------------------------------


def _linear(x, w, act_round):
    """F.linear without bias; for bf16 models the product is accumulated in
    fp32 and rounded once (layers/linear.py:74-76)."""
    y = np.asarray(x, np.float32) @ np.asarray(w, np.float32).T
    return act_round(y) if act_round is not None else y.astype(np.float32)


def gdn_layer_forward(hidden, W, conv_pool, s_pool, ids, lens, HK, DK, HV, DV,
                      eps=1e-6, act_round=round_bf16):
    """Qwen3_5GatedDeltaNet.forward for one varlen batch (qwen3_5.py:864-920):
    the prefix of length-1 rows goes through the decode branch, the rest
    through the prefill composition.  ``W`` holds the layer's parameters by
    their reference names (in_proj_qkv, in_proj_z, in_proj_b, in_proj_a,
    conv1d [conv_dim, 1, K], A_log, dt_bias, norm, out_proj); pools are
    per-layer views [slots, ...] mutated in place.  Returns [N, hidden]."""
    r = act_round if act_round is not None else (lambda t: np.asarray(t, np.float32))
    Wr = {k: r(np.asarray(v, np.float32)) for k, v in W.items()}
    x = r(np.asarray(hidden, np.float32))
    lens = [int(v) for v in lens]
    ids = np.asarray(ids, np.int64)
    n1 = 0
    while n1 < len(lens) and lens[n1] == 1:
        n1 += 1
    conv_w = Wr["conv1d"].reshape(Wr["conv1d"].shape[0], -1)
    cores = []
    if n1:
        xd = x[:n1]
        cores.append(gdn_core_decode(
            _linear(xd, Wr["in_proj_qkv"], act_round), _linear(xd, Wr["in_proj_a"], act_round),
            _linear(xd, Wr["in_proj_b"], act_round), _linear(xd, Wr["in_proj_z"], act_round),
            conv_pool, s_pool, ids[:n1], conv_w, Wr["A_log"], Wr["dt_bias"], Wr["norm"],
            HK, DK, HV, DV, eps, act_round))
    if n1 < len(lens):
        xp = x[n1:]
        cu = np.concatenate([[0], np.cumsum(lens[n1:])]).astype(np.int64)
        cores.append(gdn_core_prefill(
            _linear(xp, Wr["in_proj_qkv"], act_round), _linear(xp, Wr["in_proj_a"], act_round),
            _linear(xp, Wr["in_proj_b"], act_round), _linear(xp, Wr["in_proj_z"], act_round),
            conv_pool, s_pool, ids[n1:], cu, conv_w, Wr["A_log"], Wr["dt_bias"], Wr["norm"],
            HK, DK, HV, DV, eps, act_round))
    core = np.concatenate(cores, 0)
    return _linear(core, Wr["out_proj"], act_round)
