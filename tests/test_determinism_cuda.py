"""Every training path gives bit-identical outputs and gradients when the same
call runs twice. The kernels sum in a fixed order (no floating-point atomics),
so any difference between two runs means a race inside a kernel; shapes are
large enough to fill the GPU with several waves of CTAs, where such races show.
"""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib(built_lib):
    import lizard_cuda
    lizard_cuda.load()


def _twice(fn, inputs, dy):
    outs = []
    for _ in range(2):
        leaves = [t.detach().clone().requires_grad_() for t in inputs]
        y = fn(*leaves)
        y.backward(dy)
        torch.cuda.synchronize()
        outs.append((y.detach().clone(), [t.grad.clone() for t in leaves]))
    (y0, g0), (y1, g1) = outs
    assert torch.equal(y0, y1), "outputs differ between two identical calls"
    for i, (a, b) in enumerate(zip(g0, g1)):
        assert torch.equal(a, b), f"gradient {i} differs between two identical calls"


def _gen(seed):
    return torch.Generator(device=DEV).manual_seed(seed)


def _features(shape, g):
    return (F.softplus(torch.randn(shape, generator=g, device=DEV)) / math.sqrt(shape[-1])).bfloat16()


@pytest.mark.parametrize("B,H,Hkv,L,Fd,D", [
    (4, 32, 32, 2048, 64, 64),     # config-3 shape: the chunk-parallel schedule
    (2, 32, 8, 2048, 256, 64),     # the model's grouped keys / values, feature dim 256
])
def test_gla_training_is_deterministic(B, H, Hkv, L, Fd, D):
    import lizard_cuda
    g = _gen(B * L + Fd)
    fq, fk = _features((B, H, L, Fd), g), _features((B, Hkv, L, Fd), g)
    v = torch.randn(B, Hkv, L, D, generator=g, device=DEV).bfloat16()
    lg = F.logsigmoid(3 + 1.5 * torch.randn(B, L, generator=g, device=DEV))
    dy = torch.randn(B, H, L, D, generator=g, device=DEV).bfloat16()
    _twice(lizard_cuda.gla, [fq, fk, v, lg], dy)


@pytest.mark.parametrize("B,H,Hkv,dtype", [
    (16, 32, 32, torch.bfloat16),  # the persistent forward, dq and dk / dv
    (2, 32, 8, torch.float32),     # residual split terms, grouped keys / values
])
def test_swa_training_is_deterministic(B, H, Hkv, dtype):
    import lizard_cuda
    g = _gen(B + H + Hkv)
    q = torch.randn(B, H, 2048, 64, generator=g, device=DEV).to(dtype)
    k, v = (torch.randn(B, Hkv, 2048, 64, generator=g, device=DEV).to(dtype) for _ in range(2))
    meta = torch.randn(4, generator=g, device=DEV)
    dy = torch.randn(B, H, 2048, 64, generator=g, device=DEV).bfloat16()
    _twice(lambda a, b, c, m: lizard_cuda.swa(a, b, c, m, 64), [q, k, v, meta], dy)


def test_swa_rope_training_is_deterministic():
    import lizard_cuda
    g = _gen(5)
    inv = 1.0 / (5e5 ** (torch.arange(0, 64, 2, device=DEV).float() / 64))
    ang = torch.arange(4096, device=DEV).float()[:, None] * inv
    emb = torch.cat([ang, ang], -1)[None]
    cos, sin = emb.cos().bfloat16(), emb.sin().bfloat16()
    q = torch.randn(4, 32, 4096, 64, generator=g, device=DEV).bfloat16()
    k, v = (torch.randn(4, 8, 4096, 64, generator=g, device=DEV).bfloat16() for _ in range(2))
    meta = torch.randn(4, generator=g, device=DEV)
    dy = torch.randn(4, 32, 4096, 64, generator=g, device=DEV).bfloat16()
    _twice(lambda a, b, c, m: lizard_cuda.swa_rope(a, b, c, cos, sin, m, 64), [q, k, v, meta], dy)


def test_hedgehog_training_is_deterministic():
    import lizard_cuda
    g = _gen(7)
    x = torch.randn(4, 32, 4096, 64, generator=g, device=DEV)
    w = torch.randn(128, 64, generator=g, device=DEV) * 0.1
    dy = torch.randn(4, 32, 4096, 256, generator=g, device=DEV).bfloat16()
    _twice(lizard_cuda.hedgehog, [x, w], dy)
