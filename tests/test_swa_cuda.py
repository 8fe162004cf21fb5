"""SWA kernels on the GPU against the reference fixtures and the CPU oracle."""
import pytest
import torch
import torch.nn.functional as F

import cases
import lizard_oracle as orc
from conftest import load_golden
from parity import assert_grad, assert_output

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib(built_lib):
    import lizard_cuda
    lizard_cuda.load()


def cuda_swa(q, k, v, meta, window, dy=None):
    import lizard_cuda
    leaves = [t.detach().to(DEV).clone().requires_grad_() for t in (q, k, v, meta)]
    y = lizard_cuda.swa(*leaves, window)
    if dy is not None:
        y.backward(dy.to(DEV).to(y.dtype))
    return y, [t.grad for t in leaves]


def oracle_swa(q, k, v, meta, window, dy=None):
    leaves = [t.detach().float().cpu().clone().requires_grad_() for t in (q, k, v, meta)]
    y = orc.awa(*leaves, window)
    if dy is not None:
        y.backward(dy.float().cpu())
    return y.detach(), [t.grad for t in leaves]


@pytest.mark.parametrize("name", list(cases.SWA_CASES))
def test_swa_matches_reference_fixture(name):
    fx = load_golden(name)
    inp, window = fx["inputs"], fx["window"]
    y, (dq, dk, dv, dmeta) = cuda_swa(inp["q"], inp["k"], inp["v"], inp["meta"], window,
                                      inp["dy"])
    assert y.dtype == torch.bfloat16
    assert_output(y, fx["y"], f"{name} y")
    for g, key in zip((dq, dk, dv), ("dq", "dk", "dv")):
        assert_grad(g, fx[key + "_b"], f"{name} {key}")
    if inp["meta"].numel():
        assert_grad(dmeta, fx["dmeta_b"], f"{name} dmeta")


def config3_inputs(seed=0):
    """B=1, L=2048, H=32, D=64, window 64, 4 sinks ~ N(0,1); q, k rotated with
    RoPE base 5e5 before the call, as the layer does."""
    g = torch.Generator(device=DEV).manual_seed(seed)
    B, H, L, D = 1, 32, 2048, 64
    q, k, v = (torch.randn(B, H, L, D, generator=g, device=DEV) for _ in range(3))
    cos, sin = (t.to(DEV) for t in orc.rotary_tables(L, D, 500000.0))
    q, k = orc.rope(q, cos, sin), orc.rope(k, cos, sin)
    meta = torch.randn(4, generator=g, device=DEV)
    dy = torch.randn(B, H, L, D, generator=g, device=DEV)
    return q.bfloat16(), k.bfloat16(), v.bfloat16(), meta, dy


def test_swa_config3_forward_backward():
    q, k, v, meta, dy = config3_inputs()
    y, grads = cuda_swa(q, k, v, meta, 64, dy)
    ref, rgrads = oracle_swa(q, k, v, meta, 64, dy.bfloat16())
    assert_output(y, ref, "cfg3 y")
    for got, r, n in zip(grads, rgrads, ("dq", "dk", "dv", "dmeta")):
        assert_grad(got, r, f"cfg3 {n}")


def test_swa_head_dim_128_and_wide_window():
    g = torch.Generator(device=DEV).manual_seed(1)
    q, k, v = (torch.randn(2, 2, 300, 128, generator=g, device=DEV).bfloat16() for _ in range(3))
    meta = torch.randn(3, generator=g, device=DEV)
    dy = torch.randn(2, 2, 300, 128, generator=g, device=DEV)
    y, grads = cuda_swa(q, k, v, meta, 200, dy)
    ref, rgrads = oracle_swa(q, k, v, meta, 200, dy.bfloat16())
    assert_output(y, ref, "D=128 y")
    for got, r, n in zip(grads, rgrads, ("dq", "dk", "dv", "dmeta")):
        assert_grad(got, r, f"D=128 {n}")


def test_swa_without_sinks_and_window_is_causal_softmax():
    import lizard_cuda
    g = torch.Generator(device=DEV).manual_seed(2)
    q, k, v = (torch.randn(1, 3, 200, 64, generator=g, device=DEV).bfloat16() for _ in range(3))
    with torch.no_grad():
        y = lizard_cuda.swa(q, k, v, torch.zeros(0, device=DEV), 10**6)
    ref = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=True)
    assert_output(y, ref, "causal softmax")


def test_swa_many_sinks_equal_one_logsumexp_sink():
    import lizard_cuda
    inp = cases.swa_case(100)
    q, k, v, meta = (inp[n].to(DEV) for n in ("q", "k", "v", "meta"))
    one = torch.logsumexp(meta, 0, keepdim=True)
    with torch.no_grad():
        a = lizard_cuda.swa(q, k, v, meta, 16)
        b = lizard_cuda.swa(q, k, v, one, 16)
    assert orc.max_rel(a.cpu(), b.cpu()) < 8e-3


def test_swa_gradient_only_inside_the_window():
    import lizard_cuda
    inp = cases.swa_case(40)
    q, k, v = (inp[n].to(DEV).requires_grad_() for n in ("q", "k", "v"))
    lizard_cuda.swa(q, k, v, inp["meta"].to(DEV), 16)[:, :, 39].float().sum().backward()
    assert (k.grad[:, :, :24] == 0).all()
    assert (k.grad[:, :, 24:].float().abs().sum(-1) > 0).all()


def test_swa_fp32_inputs_use_residual_logits():
    """fp32 q, k with large logits (|s| ~ 40): the bf16 residuals keep the
    sink gradient within 1e-2 of the fp32 oracle."""
    g = torch.Generator(device=DEV).manual_seed(4)
    q, k = (3 * torch.randn(1, 4, 90, 32, generator=g, device=DEV) for _ in range(2))
    v = torch.randn(1, 4, 90, 32, generator=g, device=DEV)
    meta = torch.randn(4, generator=g, device=DEV)
    dy = torch.randn(1, 4, 90, 32, generator=g, device=DEV)
    y, grads = cuda_swa(q, k, v, meta, 16, dy)
    assert all(t.dtype == torch.float32 for t in grads)
    ref, rgrads = oracle_swa(q, k, v, meta, 16, dy.bfloat16())
    assert_output(y, ref, "fp32 y")
    for got, r, n in zip(grads, rgrads, ("dq", "dk", "dv", "dmeta")):
        assert_grad(got, r, f"fp32 {n}")


def test_swa_without_grad_gives_the_same_output():
    import lizard_cuda
    inp = cases.swa_case(150)
    q, k, v, meta = (inp[n].to(DEV) for n in ("q", "k", "v", "meta"))
    y = lizard_cuda.swa(q, k, v.clone().requires_grad_(), meta, 32)
    with torch.no_grad():
        assert torch.equal(lizard_cuda.swa(q, k, v, meta, 32), y)
