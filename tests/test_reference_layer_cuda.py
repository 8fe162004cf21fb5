"""The drop-in, proved through the reference's own layer file.

The reference's LizardAttention (src/lizard_attention.py:45-97) is loaded
unmodified from an installed copy of its src/ modules (LIZARD_REFERENCE_SRC,
else baseline/_ref at the root of this repository) and run two ways:

  * stock: backend="triton", with lizard_cuda bound as the module `kernels`
    that the layer imports inside forward (src/lizard_attention.py:90-93), so
    the reference's own branch calls kernels.gla / kernels.swa of this backend
    with the exact tensors it builds (fp32, repeat_interleaved, non-contiguous,
    rotated by transformers' apply_rotary_pos_emb);
  * patched: the three-line change that adds a "cuda" backend to the layer
    (the constructor's assert and the forward's branch), applied to a copy of
    the file, with backend="cuda".

Each is compared with the same layer on backend="torch" (the reference's
dense fp32 path) on the same device: output and every parameter gradient,
with the layer tolerances of the reference's own test
(tests/test_kernels.py:137-156) and max|err| / max|ref| <= 1e-2.
"""
import importlib.util
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

import cases
from conftest import ROOT, load_golden
from parity import assert_grad, assert_output

DEV = "cuda"


def _reference_file():
    env = os.environ.get("LIZARD_REFERENCE_SRC")
    cand = Path(env) if env else ROOT / "baseline" / "_ref"
    path = cand / "lizard_attention.py"
    if not path.exists():
        pytest.skip(f"the reference's lizard_attention.py is not installed at {cand}")
    return path


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


# the change that adds the cuda backend, as (old, new) text replacements
PATCH = (
    ("import math\n", "import importlib\nimport math\n"),
    ('assert backend in ("torch", "triton"), backend',
     'assert backend in ("torch", "triton", "cuda"), backend'),
    ('        if self.backend == "triton":\n            import kernels\n',
     '        if self.backend in ("triton", "cuda"):\n'
     '            kernels = importlib.import_module(\n'
     '                "kernels" if self.backend == "triton" else "lizard_cuda")\n'),
)


def _patched(path, tmp_path):
    text = path.read_text()
    for old, new in PATCH:
        assert text.count(old) == 1, f"patch context not found once: {old!r}"
        text = text.replace(old, new)
    out = tmp_path / "lizard_attention_cuda_patch.py"
    out.write_text(text)
    return out


def _layers(mod, case, backend):
    c = cases.LAYER_CASES[case]
    cfg = SimpleNamespace(hidden_size=c["hidden"], num_attention_heads=c["heads"],
                          num_key_value_heads=c["kv_heads"])
    opts = dict(window=c["window"], num_meta=c["num_meta"], feature_dim=c["feature_dim"])
    ref = mod.LizardAttention(cfg, 0, **opts)
    cases.init_layer_params(ref, c["init"])
    ours = mod.LizardAttention(cfg, 0, backend=backend, **opts)
    ours.load_state_dict(ref.state_dict())
    return c, ref.to(DEV), ours.to(DEV)


def _compare(case, c, ref, ours, what):
    fx = load_golden(case)  # the rotary tables the reference fixtures were made with
    x, grad = cases.layer_inputs(c)
    x, grad = x.to(DEV), grad.to(DEV)
    rope = (fx["cos"].to(DEV), fx["sin"].to(DEV))
    y_ref = ref(x, rope)[0]
    y_ref.backward(grad)
    y = ours(x, rope)[0]
    y.backward(grad)
    torch.cuda.synchronize()
    assert_output(y, y_ref.detach(), f"{what} y", layer=True)
    for (n, p), q in zip(ours.named_parameters(), ref.parameters()):
        assert p.grad is not None, f"{what}: no gradient for {n}"
        assert_grad(p.grad, q.grad, f"{what} d{n}")


@pytest.mark.gpu
@pytest.mark.parametrize("case", list(cases.LAYER_CASES))
def test_stock_reference_layer_runs_lizard_cuda_as_its_kernels(case, built_lib, monkeypatch):
    import lizard_cuda
    mod = _load(_reference_file(), "reference_lizard_attention")
    monkeypatch.setitem(sys.modules, "kernels", lizard_cuda)
    c, ref, ours = _layers(mod, case, "triton")
    calls = lizard_cuda.launch_count()
    _compare(case, c, ref, ours, f"stock layer {case}")
    assert lizard_cuda.launch_count() > calls, "the layer did not reach lizard_cuda"


@pytest.mark.gpu
@pytest.mark.parametrize("case", list(cases.LAYER_CASES))
def test_patched_reference_layer_with_cuda_backend(case, built_lib, tmp_path):
    import lizard_cuda
    mod = _load(_patched(_reference_file(), tmp_path), "reference_lizard_attention_cuda")
    c, ref, ours = _layers(mod, case, "cuda")
    calls = lizard_cuda.launch_count()
    _compare(case, c, ref, ours, f"patched layer {case}")
    assert lizard_cuda.launch_count() > calls, "the layer did not reach lizard_cuda"


def test_patch_applies_to_the_reference_layer(tmp_path):
    """CPU check: the patch text matches the reference file exactly once per
    hunk, and the patched layer constructs with backend="cuda" (and still
    rejects unknown backends)."""
    mod = _load(_patched(_reference_file(), tmp_path), "reference_lizard_attention_patch_cpu")
    c = cases.LAYER_CASES["layer_tiny"]
    cfg = SimpleNamespace(hidden_size=c["hidden"], num_attention_heads=c["heads"],
                          num_key_value_heads=c["kv_heads"])
    assert mod.LizardAttention(cfg, 0, backend="cuda").backend == "cuda"
    with pytest.raises(AssertionError):
        mod.LizardAttention(cfg, 0, backend="other")
