"""Recurrent-state pools and slot lifecycle — the engine contract the GDN
kernels honour.

Mirrors engine/model_runner.py:265-322 (pool layout, per-layer view binding,
dummy slot, zero-on-fresh-prefill).  Slot ids themselves come from the
engine's own free list (engine/linear_state_pool.py), which this package
does not replace:

* ``s_pool``    fp32 [num_slots + 1, L, HV, DK, DV]
* ``conv_pool`` model dtype [num_slots + 1, L, conv_dim, K - 1]
* layer i gets the views ``s_pool[:, i]`` / ``conv_pool[:, i]`` as
  ``module.s_cache`` / ``module.conv_cache``; the kernels index them by slot
  id with the view's slot stride (L * HV * DK * DV elements), no gather.
* slot ``num_slots`` is the dummy slot that CUDA-graph pad rows point at.

Each slot's state is laid out row-major [HV, DK, DV] with the value dim
innermost, so one head's 128 x 128 fp32 state is a single contiguous 64 KiB
run (16-byte aligned), which is what the decode kernel streams.
"""
from __future__ import annotations

import torch


def gdn_modules(model: torch.nn.Module):
    """The GDN layers of a model, discovered as the engine does
    (hasattr(m, "s_cache"), model_runner.py:100, 276)."""
    return [m for m in model.modules() if hasattr(m, "s_cache")]


class StatePools:
    """Allocate the pools for ``modules`` and bind their per-layer views."""

    def __init__(self, modules, num_slots: int, device, conv_dtype=torch.bfloat16):
        modules = list(modules)
        assert modules, "no GDN modules"
        m0 = modules[0]
        L = len(modules)
        H, K, V = m0.num_v_heads, m0.head_k_dim, m0.head_v_dim
        self.num_slots = num_slots
        self.dummy_slot = num_slots
        self.s_pool = torch.zeros(num_slots + 1, L, H, K, V, dtype=torch.float32, device=device)
        self.conv_pool = torch.zeros(num_slots + 1, L, m0.conv_dim, m0.conv_kernel - 1,
                                     dtype=conv_dtype, device=device)
        for i, m in enumerate(modules):
            m.s_cache = self.s_pool[:, i]
            m.conv_cache = self.conv_pool[:, i]

    @staticmethod
    def bytes_per_slot(L, H, K, V, conv_dim, conv_kernel, conv_bytes=2) -> int:
        """model_runner.py:280: L * (H*K*V*4 + conv_dim*(k-1)*2)."""
        return L * (H * K * V * 4 + conv_dim * (conv_kernel - 1) * conv_bytes)

    def reset(self, slot_ids: torch.Tensor):
        """Zero slots (fresh-prefill semantics, model_runner.py:305-308): a
        zero state is the initial state and a zero conv prefix is the causal
        conv's zero left-padding."""
        self.s_pool.index_fill_(0, slot_ids, 0.0)
        self.conv_pool.index_fill_(0, slot_ids, 0.0)
