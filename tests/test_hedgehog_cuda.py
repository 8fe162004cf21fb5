"""Fused Hedgehog feature map against the oracle's restatement of the
reference (float64 autograd): features and the gradients w.r.t. x and W."""
import pytest
import torch

import lizard_oracle as orc
from parity import assert_grad, assert_output

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib(built_lib):
    import lizard_cuda
    lizard_cuda.load()


@pytest.fixture(params=["rows", "tiles"])
def forward_kernel(request):
    """Small inputs take the warp-per-row forward by default; "tiles" sends
    them to the tiled kernels instead, so both are checked on the same cases."""
    from lizard_cuda import _lib
    lib = _lib.load()
    old = lib.lz_hedgehog_set_rows_max(-1 if request.param == "rows" else 0)
    yield request.param
    lib.lz_hedgehog_set_rows_max(old)


@pytest.mark.parametrize("shape,Fd,xdt,std", [
    ((2, 4, 40, 32), 8, torch.float32, 0.3 * 8),     # layer_tiny: head dim 32, feature dim 8
    ((1, 4, 256, 64), 128, torch.float32, 0.02),     # config 1 layer: the init scale
    ((2, 3, 300, 64), 128, torch.bfloat16, 0.16),    # bf16 heads, trained-size weights
    ((1, 2, 77, 20), 24, torch.float32, 0.5),        # odd sizes, padded tiles
    ((1, 1, 1000, 128), 100, torch.float32, 0.1),
])
def test_hedgehog_matches_reference(shape, Fd, xdt, std, forward_kernel):
    import lizard_cuda
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(shape, generator=g, device=DEV).to(xdt)
    w = std * torch.randn(Fd, shape[-1], generator=g, device=DEV)
    df = torch.randn(*shape[:-1], 2 * Fd, generator=g, device=DEV)
    xl, wl = x.clone().requires_grad_(), w.clone().requires_grad_()
    f = lizard_cuda.hedgehog(xl, wl)
    assert f.dtype == torch.bfloat16 and f.shape == (*shape[:-1], 2 * Fd)
    f.backward(df.bfloat16())
    xr = x.double().cpu().requires_grad_()
    wr = w.double().cpu().requires_grad_()
    ref = orc.hedgehog(xr, wr)
    ref.backward(df.bfloat16().double().cpu())
    assert_output(f, ref.float(), f"hedgehog {shape} f")
    assert_grad(xl.grad, xr.grad.float(), f"hedgehog {shape} dx")
    assert_grad(wl.grad, wr.grad.float(), f"hedgehog {shape} dW")
    assert xl.grad.dtype == xdt and wl.grad.dtype == torch.float32


@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float32])
def test_hedgehog_decode_step_rows(xdt):
    """One token per sequence (decode): x is the [B, 1, H * Dh] projection read
    as [B, H, 1, Dh] heads, R = B * H rows on the warp-per-row kernel; against
    the oracle and the tiled kernels."""
    import lizard_cuda
    from lizard_cuda import _lib
    lib = _lib.load()
    g = torch.Generator(device=DEV).manual_seed(21)
    B, H, Dh, Fd = 32, 32, 64, 128
    proj = torch.randn(B, 1, H * Dh, generator=g, device=DEV).to(xdt)
    x = proj.view(B, 1, H, Dh).transpose(1, 2)
    w = 0.2 * torch.randn(Fd, Dh, generator=g, device=DEV)
    outs = []
    for rows in (-1, 0):
        old = lib.lz_hedgehog_set_rows_max(rows)
        try:
            with torch.no_grad():
                outs.append(lizard_cuda.hedgehog(x, w))
        finally:
            lib.lz_hedgehog_set_rows_max(old)
    ref = orc.hedgehog(x.double().cpu(), w.double().cpu())
    assert_output(outs[0], ref.float(), f"hedgehog decode rows {xdt}")
    diff = (outs[0].float() - outs[1].float()).abs().max().item()
    assert diff <= 2 ** -7 * outs[1].float().abs().max().item(), diff


def test_hedgehog_rows_sum_to_one_and_weights_are_deterministic():
    import lizard_cuda
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(3, 4, 500, 64, generator=g, device=DEV)
    w = (0.05 * torch.randn(128, 64, generator=g, device=DEV)).requires_grad_()
    f = lizard_cuda.hedgehog(x, w)
    s = f.float().view(-1, 2, 128).sum(-1)
    assert torch.allclose(s, torch.ones_like(s), atol=2e-2)
    df = torch.randn_like(f)
    f.backward(df)
    g1 = w.grad.clone()
    w.grad = None
    lizard_cuda.hedgehog(x, w).backward(df)
    assert torch.equal(w.grad, g1)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_hedgehog_reads_projection_views_in_place(dtype):
    """A [B, L, H * Dh] projection viewed as [B, H, L, Dh] goes to the strided
    entry points: features, dx and dW equal those of the contiguous copy."""
    import lizard_cuda
    g = torch.Generator(device="cuda").manual_seed(4)
    B, L, H, Dh, Fd = 2, 77, 3, 64, 128
    proj = torch.randn(B, L, H * Dh, generator=g, device="cuda").to(dtype)
    w = 0.2 * torch.randn(Fd, Dh, generator=g, device="cuda")
    df = torch.randn(B, H, L, 2 * Fd, generator=g, device="cuda").bfloat16()
    outs = []
    for contig in (False, True):
        p = proj.clone().requires_grad_()
        wl = w.clone().requires_grad_()
        x = p.view(B, L, H, Dh).transpose(1, 2)
        if contig:
            x = x.contiguous()
        f = lizard_cuda.hedgehog(x, wl)
        f.backward(df)
        outs.append((f, p.grad, wl.grad))
    (f1, dx1, dw1), (f2, dx2, dw2) = outs
    assert torch.equal(f1, f2)
    assert torch.equal(dx1, dx2)
    assert torch.equal(dw1, dw2)


@pytest.mark.parametrize("strided,L", [(False, 333), (True, 333), (True, 50)])
def test_hedgehog_tensor_core_forward(strided, L):
    """bf16 x with Dh = 64, Fd = 128 (the model's feature map) runs on the
    tensor cores: against the oracle, and within bf16 rounding of the warp-MMA
    kernel (only the order of the softmax sums differs)."""
    import lizard_cuda
    from lizard_cuda import _lib
    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(9)
    B, H, Dh, Fd = 2, 3, 64, 128  # L = 50: one partial tile per head, every store clipped
    proj = torch.randn(B, L, H * Dh, generator=g, device="cuda").bfloat16()
    x = proj.view(B, L, H, Dh).transpose(1, 2)
    if not strided:
        x = x.contiguous()
    w = 0.3 * torch.randn(Fd, Dh, generator=g, device="cuda")
    outs = []
    old_rows = lib.lz_hedgehog_set_rows_max(0)  # the tiled kernels even at this size
    try:
        for on in (1, 0):
            old = lib.lz_hedgehog_set_tc(on)
            try:
                with torch.no_grad():
                    outs.append(lizard_cuda.hedgehog(x, w))
            finally:
                lib.lz_hedgehog_set_tc(old)
    finally:
        lib.lz_hedgehog_set_rows_max(old_rows)
    ref = orc.hedgehog(x.double().cpu(), w.double().cpu())
    assert_output(outs[0], ref.float(), "hedgehog tensor-core forward")
    diff = (outs[0].float() - outs[1].float()).abs().max().item()
    assert diff <= 2 ** -8 * outs[1].float().abs().max().item(), diff
