"""The fused output blend against the reference caller's torch expression
(src/lizard_attention.py:92-97), and the layer's inference path (no fp32
upcast) against its autograd path."""
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib(built_lib):
    import lizard_cuda
    lizard_cuda.load()


def torch_blend(yg, ys, alpha, dtype):
    c = torch.float32
    y = yg.to(c) + alpha.to(c) * ys.to(c)
    return y.to(dtype).transpose(1, 2).flatten(2)


@pytest.mark.parametrize("D", [64, 20])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_blend_forward_backward_match_torch(D, dtype):
    from lizard_cuda import blend
    g = torch.Generator(device=DEV).manual_seed(D)
    B, H, L = 2, 3, 77
    yg = torch.randn(B, H, L, D, generator=g, device=DEV).bfloat16().requires_grad_()
    ys = torch.randn(B, H, L, D, generator=g, device=DEV).bfloat16().requires_grad_()
    alpha = torch.tensor(0.73, device=DEV, requires_grad=True)
    out = blend(yg, ys, alpha, dtype)
    ref_in = [t.detach().clone().requires_grad_() for t in (yg, ys, alpha)]
    ref = torch_blend(*ref_in, dtype)
    assert out.dtype == dtype and out.shape == (B, L, H * D)
    assert torch.equal(out, ref)
    dout = torch.randn(out.shape, generator=g, device=DEV).to(dtype)
    out.backward(dout)
    ref.backward(dout)
    assert torch.equal(yg.grad, ref_in[0].grad)
    assert torch.equal(ys.grad, ref_in[1].grad)
    torch.testing.assert_close(alpha.grad, ref_in[2].grad, rtol=1e-5, atol=1e-5)


def test_layer_inference_equals_autograd_forward():
    """Without autograd the layer skips the fp32 upcast of q, k, v; every
    kernel converts to fp32 itself, so the output is bit-identical."""
    from lizard_cuda.layer import LizardAttention
    cfg = SimpleNamespace(hidden_size=256, num_attention_heads=4, num_key_value_heads=2)
    torch.manual_seed(0)
    layer = LizardAttention(cfg, 0, window=32, num_meta=4, feature_dim=32)
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0, 0.3)
    layer = layer.to(DEV).bfloat16()
    g = torch.Generator(device=DEV).manual_seed(1)
    B, L = 2, 150
    x = torch.randn(B, L, 256, generator=g, device=DEV).bfloat16()
    inv = 1.0 / (1e4 ** (torch.arange(0, 64, 2, device=DEV).float() / 64))
    ang = torch.arange(L, device=DEV).float()[:, None] * inv
    emb = torch.cat([ang, ang], -1)[None].expand(B, L, 64)
    rope = (emb.cos().bfloat16(), emb.sin().bfloat16())
    with torch.no_grad():
        y0 = layer(x, rope)[0]
    y1 = layer(x.clone().requires_grad_(), rope)[0]
    assert torch.equal(y0, y1.detach())
