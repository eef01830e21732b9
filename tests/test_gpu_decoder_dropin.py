"""The drop-in, end to end inside the reference's own model code: this
package's layer installed into the reference's nanovllm.models.qwen3_5 (the
class its Qwen3_5DecoderLayer constructs), a two-layer stack of the
reference's decoder layers (its RMSNorms, MLPs and residual chain) built at
config-0 shapes in bf16, the state pools made and bound by the reference's own
ModelRunner._allocate_linear_state_pool, then a 4-sequence prefill and 16
decode steps — compared with the same stack run un-swapped on the
reference's torch path (tests/golden/decoder_c0_bf16.npz, written by
tests/golden/make_decoder_golden.py).

Needs the reference package importable: the offline install in
baseline/_ref (next to this repository's root) or a checkout named by
$GDN_REFERENCE_ROOT; skipped otherwise.  The reference's torch.compile'd
norm helpers run eagerly here (dynamo disabled for the test), and its
flashinfer norms are switched off, as in the golden run.

Tolerances (layer-level bf16: the projections and MLPs are different bf16
GEMMs on the two sides, CPU torch against cuBLAS; their one-ulp differences
enter the recurrent state and compound over the 16 decode steps through two
GDN layers and two MLPs): per step, the relative (Frobenius) error of the
hidden outputs and of the residual stream <= 2e-2 and their largest
element-wise error <= 5 % of the largest value (a wiring fault gives errors of
order one); final recurrent states relative <= 2e-2; conv states (raw
projection outputs): layer 0's, projected from the same inputs, within one
bf16 ulp, layer 1's relative <= 2e-2.
"""
import os
import sys
import types

import numpy as np
import pytest
import torch

import inputs as I
from decoder_harness import decoder_config, decoder_inputs, load_weights, run_stack

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DEV = "cuda:0"


def _reference_root():
    for cand in (os.environ.get("GDN_REFERENCE_ROOT"), os.path.join(ROOT, "baseline", "_ref")):
        if cand and os.path.isdir(os.path.join(cand, "nanovllm")):
            return cand
    return None


@pytest.fixture(scope="module")
def ref_modules(pkg):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    root = _reference_root()
    if root is None:
        pytest.skip("the reference package is not installed (baseline/_ref)")
    os.environ.setdefault("NANOVLLM_FI_NORM", "0")
    os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")
    sys.path.insert(0, root)
    try:
        import nanovllm.models.qwen3_5 as Q
        import nanovllm.utils.context as Cx
        import nanovllm.utils.parallel as P
        from nanovllm.engine.model_runner import ModelRunner
    finally:
        sys.path.remove(root)
    torch.cuda.set_device(0)
    return Q, Cx, P, ModelRunner


def _bf16_ulp(x):
    ax = np.maximum(np.abs(x), 1e-30)
    return 2.0 ** (np.floor(np.log2(ax)) - 7)


def test_installed_layer_in_reference_decoder_stack(pkg, ref_modules, golden_dir):
    Q, Cx, P, ModelRunner = ref_modules
    import torch._dynamo
    d = dict(np.load(os.path.join(golden_dir, "decoder_c0_bf16.npz")))
    c, dec_cfg = I.C0, I.DEC
    W = I.decoder_weights(c["hidden"], dec_cfg["inter"], c["HK"], c["DK"], c["HV"], c["DV"],
                          c["K"], layers=dec_cfg["layers"])
    pre, dec = decoder_inputs()
    assert str(d["digest"]) == I.digest(pre, *dec, *W.values())

    previous = pkg.layer.install(Q, P, Cx)
    dynamo_was = torch._dynamo.config.disable
    torch._dynamo.config.disable = True
    prev_dtype = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(DEV):
            layers = [Q.Qwen3_5DecoderLayer(decoder_config(), i)
                      for i in range(dec_cfg["layers"])]
        for layer in layers:
            assert isinstance(layer.linear_attn, pkg.layer.Qwen3_5GatedDeltaNet)
        load_weights(layers, W)
        # the reference's own pool allocation and binding, on a stand-in runner
        runner = types.SimpleNamespace(
            model=torch.nn.ModuleList(layers), world_size=1,
            config=types.SimpleNamespace(max_num_seqs=dec_cfg["slots"]),
            _min_over_group=lambda v: v)
        ModelRunner._allocate_linear_state_pool(runner)
        assert runner.linear_dummy_slot == dec_cfg["slots"]
        ids = np.array(dec_cfg["ids"], np.int64)
        lens = list(c["lens"])
        h, r = run_stack(layers, Cx.set_context, Cx.reset_context, pre, ids, lens, DEV)
        got = [(h, r)]
        for x in dec:
            got.append(run_stack(layers, Cx.set_context, Cx.reset_context, x, ids,
                                 [1] * len(lens), DEV))
        torch.cuda.synchronize()
        pkg.ops.check_status()
        s_rows = runner.linear_s_pool[torch.as_tensor(ids, device=DEV)].cpu().numpy()
        conv_rows = runner.linear_conv_pool[torch.as_tensor(ids, device=DEV)].float().cpu().numpy()
    finally:
        torch.set_default_dtype(prev_dtype)
        torch._dynamo.config.disable = dynamo_was
        pkg.layer.uninstall(previous, Q)

    refs = [(d["h_prefill"], d["r_prefill"])] + [(d["h_decode"][s], d["r_decode"][s])
                                                  for s in range(len(dec))]
    for step, ((h, r), (h_ref, r_ref)) in enumerate(zip(got, refs)):
        h, r = h.float().cpu().numpy(), r.float().cpu().numpy()
        for name, x, x_ref in (("hidden", h, h_ref), ("residual", r, r_ref)):
            rel = np.linalg.norm(x - x_ref) / np.linalg.norm(x_ref)
            worst = np.abs(x - x_ref).max() / np.abs(x_ref).max()
            print(f"step {step} {name}: relative error {rel:.2e}, max-abs / max {worst:.2e}")
            assert rel <= 2e-2, f"step {step}: {name} relative error {rel}"
            assert worst <= 5e-2, f"step {step}: {name} max-abs error / max value {worst}"
    rel = np.linalg.norm(s_rows - d["s_rows"]) / np.linalg.norm(d["s_rows"])
    assert rel <= 2e-2, f"state rel {rel}"
    # layer 0's conv rows are projections of the same inputs on both sides (the
    # decode steps' hidden states): one bf16 ulp; layer 1's come from layer 0's
    # outputs, which carry the stack's bf16 drift: relative error
    c0, c0_ref = conv_rows[:, 0], d["conv_rows"][:, 0]
    ec = np.abs(c0 - c0_ref) - _bf16_ulp(c0_ref)
    assert ec.max() <= 1e-6, f"layer-0 conv state beyond one bf16 ulp by {ec.max()}"
    c1, c1_ref = conv_rows[:, 1], d["conv_rows"][:, 1]
    rel1 = np.linalg.norm(c1 - c1_ref) / np.linalg.norm(c1_ref)
    assert rel1 <= 2e-2, f"layer-1 conv state relative error {rel1}"
