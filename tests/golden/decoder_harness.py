"""The two-layer decoder harness shared by make_decoder_golden.py (which runs
it on the reference's own decoder layers, on the CPU) and
tests/test_gpu_decoder_dropin.py (which runs it on the reference's decoder
layers with this package's GDN layer installed, on the GPU).  No environment
side effects."""
from __future__ import annotations

import types

import numpy as np
import torch

import inputs as I


def decoder_config():
    c, d = I.C0, I.DEC
    return types.SimpleNamespace(
        hidden_size=c["hidden"], intermediate_size=d["inter"], rms_norm_eps=c["eps"],
        layer_types=["linear_attention"] * d["layers"], linear_num_key_heads=c["HK"],
        linear_num_value_heads=c["HV"], linear_key_head_dim=c["DK"],
        linear_value_head_dim=c["DV"], linear_conv_kernel_dim=c["K"])


def decoder_inputs():
    """(prefill hidden [N, hidden], [16 decode hiddens [4, hidden]]), float32."""
    c = I.C0
    pre = I.layer_hidden(sum(c["lens"]), c["hidden"], seed=77)
    dec = [I.layer_hidden(len(c["lens"]), c["hidden"], seed=400 + s) for s in range(c["n_decode"])]
    return pre, dec


def load_weights(layers, W):
    """Copy the seeded weights into the stack (tp = 1: every loader is a copy)."""
    with torch.no_grad():
        for name, w in W.items():
            i, pname = name.split(".", 1)
            p = layers[int(i)].get_parameter(pname)
            p.data.copy_(torch.from_numpy(w).to(p.dtype).reshape(p.shape))


def run_stack(layers, set_context, reset_context, hidden, ids, lens, device):
    """One forward of the stack (hidden states in, residual None as after the
    embedding); returns (hidden, residual) of the last layer."""
    cu = torch.tensor(I.cu_from_lens(lens), device=device)
    set_context(cu, cu, max(lens), max(lens),
                linear_state_ids=torch.as_tensor(ids, dtype=torch.int64, device=device),
                lens_q=list(lens))
    try:
        with torch.inference_mode():
            h = torch.from_numpy(np.ascontiguousarray(hidden)).to(device).to(torch.bfloat16)
            r = None
            for layer in layers:
                h, r = layer(None, h, r)
            return h, r
    finally:
        reset_context()
