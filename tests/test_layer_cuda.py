"""A whole Lizard layer with the cuda backend against the reference's torch
layer (golden fixtures; tests/test_kernels.py:137-156 of the reference)."""
from types import SimpleNamespace

import pytest
import torch

import cases
from conftest import load_golden
from parity import assert_grad, assert_output

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("name", list(cases.LAYER_CASES))
def test_layer_matches_reference_fixture(name, built_lib):
    from lizard_cuda.layer import LizardAttention
    fx = load_golden(name)
    c = fx["case"]
    cfg = SimpleNamespace(hidden_size=c["hidden"], num_attention_heads=c["heads"],
                          num_key_value_heads=c["kv_heads"])
    layer = LizardAttention(cfg, 0, window=c["window"], num_meta=c["num_meta"],
                            feature_dim=c["feature_dim"])
    cases.init_layer_params(layer, c["init"])
    for n, p in layer.named_parameters():
        assert torch.equal(cases.checksum(p), fx["param_sums"][n]), n
    layer = layer.to(DEV)
    x, grad = cases.layer_inputs(c)
    assert torch.equal(cases.checksum(x), fx["x_sum"])
    rope = (fx["cos"].to(DEV), fx["sin"].to(DEV))
    y = layer(x.to(DEV), rope)[0]
    y.backward(grad.to(DEV))
    assert_output(y, fx["y"], f"{name} y", layer=True)
    for n, p in layer.named_parameters():
        assert_grad(p.grad, fx["grads"][n], f"{name} d{n}")
