"""B200-native GatedDeltaNet layer path for nano-vllm-extend.

The directory name is not a Python identifier; load it with
``__graft_entry__.load_package()`` (repo root), which imports it as the
module ``nano_vllm_extend_b200``.

* ``ops``        tensor-level operators over the C ABI (libgdn_b200.so)
* ``layer``      drop-in Qwen3_5GatedDeltaNet + ``install()`` into the engine
* ``state_pool`` recurrent-state pools in the engine's layout (slot ids come from the
                 engine's own free list)
* ``parallel``   V-head sharding, TP linear layers, pipeline stage handoff
* ``context``    per-step Context mirror
"""
from . import _lib, context, parallel, state_pool  # noqa: F401

__all__ = ["ops", "layer", "context", "parallel", "state_pool"]


def __getattr__(name):
    # ops / layer import torch CUDA helpers lazily
    if name in ("ops", "layer"):
        import importlib
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
