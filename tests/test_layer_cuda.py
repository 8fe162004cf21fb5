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


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_layer_at_the_reference_training_window(dtype, built_lib):
    """A whole layer at window 128, the reference's training setting
    (configs/lizard-1b*.yaml: window 128, 4 sinks, feature dim 128), head dim 64
    and grouped keys / values 4 / 2, on 300 tokens, against the dense float64
    oracle layer with the same parameters: output and every parameter gradient.
    bf16 activations take the fused RoPE call's decline into the wide
    tensor-core SWA kernels; fp32 ones the split operands."""
    import lizard_oracle as orc
    from lizard_cuda.layer import LizardAttention
    hidden, heads, kv_heads, L, W = 256, 4, 2, 300, 128
    cfg = SimpleNamespace(hidden_size=hidden, num_attention_heads=heads,
                          num_key_value_heads=kv_heads)
    layer = LizardAttention(cfg, 0, window=W, num_meta=4, feature_dim=128)
    cases.init_layer_params(layer, "cfg1", seed=5)
    layer = layer.to(dtype)  # the oracle holds the same (rounded) parameter values
    dense = orc.LizardAttention(hidden, heads, kv_heads, window=W, num_meta=4, feature_dim=128)
    dense.load_state_dict({n: t.float() for n, t in layer.state_dict().items()})
    g = torch.Generator().manual_seed(6)
    x = torch.randn(2, L, hidden, generator=g)
    grad = torch.randn(2, L, hidden, generator=g)
    cos, sin = orc.rotary_tables(L, hidden // heads, 500000.0)
    cos, sin = cos.expand(2, L, -1), sin.expand(2, L, -1)
    layer = layer.to(DEV)
    y = layer(x.to(DEV).to(dtype), (cos.to(DEV).to(dtype), sin.to(DEV).to(dtype)))[0]
    y.backward(grad.to(DEV).to(dtype))
    dense = dense.double()
    ref = dense(x.to(dtype).double(), (cos.to(dtype).double(), sin.to(dtype).double()))[0]
    ref.backward(grad.to(dtype).double())
    assert_output(y.float(), ref.float(), f"layer window 128 {dtype} y", layer=True)
    mine = dict(layer.named_parameters())
    for n, p in dense.named_parameters():
        assert_grad(mine[n].grad.float(), p.grad.float(), f"layer window 128 {dtype} d{n}")
