"""The tensor-core SWA kernels (tcgen05 + TMEM + TMA; head dim 64, windows
<= 64 and 65 ... 128) against the CPU oracle of the reference's attention
(src/lizard_attention.py:34-44 on repeat_interleaved keys / values), through
the public swa / swa_rope entry points, forward and backward; and against the
64-row warp-MMA kernels it replaces at those shapes."""
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


def _rep(x, grp):
    return x.repeat_interleave(grp, dim=1)


def _set_tc(on):
    from lizard_cuda import _lib
    return _lib.load().lz_swa_set_tc(on)


def _inputs(B, H, Hkv, L, W, n_meta, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randn(B, H, L, 64, generator=g, device=DEV).to(dtype)
    k, v = (torch.randn(B, Hkv, L, 64, generator=g, device=DEV).to(dtype) for _ in range(2))
    meta = torch.randn(n_meta, generator=g, device=DEV)
    dy = torch.randn(B, H, L, 64, generator=g, device=DEV).bfloat16()
    return q, k, v, meta, dy


def _oracle(q, k, v, meta, W, dy):
    grp = q.shape[1] // k.shape[1]
    lv = [t.detach().float().cpu().clone().requires_grad_() for t in (q, k, v, meta)]
    m = lv[3] if lv[3].numel() else torch.full((1,), -1e4)
    y = orc.awa(lv[0], _rep(lv[1], grp), _rep(lv[2], grp), m, W)
    y.backward(dy.float().cpu())
    return y.detach(), [t.grad for t in lv]


@pytest.mark.parametrize("B,H,Hkv,L,W,n_meta,dtype", [
    (1, 2, 2, 1, 8, 4, torch.bfloat16),       # one token
    (2, 4, 2, 127, 64, 4, torch.bfloat16),    # one partial 128-row block
    (1, 4, 1, 300, 64, 3, torch.float32),     # fp32: residual logits; grp 4
    (2, 2, 2, 257, 1, 4, torch.bfloat16),     # window 1: each row sees itself
    (1, 8, 2, 200, 17, 0, torch.bfloat16),    # no sinks, odd window
    (1, 2, 2, 2048, 64, 4, torch.bfloat16),   # config-3 length
])
def test_swa_tc_matches_oracle(B, H, Hkv, L, W, n_meta, dtype):
    import lizard_cuda
    q, k, v, meta, dy = _inputs(B, H, Hkv, L, W, n_meta, dtype, seed=L + W)
    lv = [t.detach().clone().requires_grad_() for t in (q, k, v, meta)]
    y = lizard_cuda.swa(*lv, W)
    y.backward(dy)
    ref, rg = _oracle(q, k, v, meta, W, dy)
    tag = f"swa tc B{B} H{H}/{Hkv} L{L} W{W} S{n_meta} {dtype}"
    assert_output(y, ref, tag + " y")
    names = ("dq", "dk", "dv", "dmeta") if n_meta else ("dq", "dk", "dv")
    for t, r, n in zip(lv, rg, names):
        assert_grad(t.grad, r, f"{tag} {n}")


@pytest.mark.parametrize("B,H,Hkv,L,W,n_meta,heads", [
    (2, 32, 32, 5000, 64, 4, ((0, 0), (1, 31), (0, 17))),     # ragged last tile
    (10, 32, 8, 4100, 17, 0, ((0, 0), (4, 13), (9, 31))),     # grp 4, odd window
])
def test_swa_tc_persistent_forward_matches_oracle(B, H, Hkv, L, W, n_meta, heads):
    """bf16 operands with at least 16 x SM-count tiles of 128 query rows take
    the persistent forward (two CTAs per SM, each walking 8 or more tiles);
    sampled heads against the oracle, forward and backward (the backward
    reads the lse and fp32 output it saved)."""
    import lizard_cuda
    nsm = torch.cuda.get_device_properties(0).multi_processor_count
    assert B * Hkv * -(-L // 128) >= 16 * nsm, "shape too small for the persistent forward"
    q, k, v, meta, dy = _inputs(B, H, Hkv, L, W, n_meta, torch.bfloat16, seed=L + W)
    with torch.no_grad():
        y_inf = lizard_cuda.swa(q, k, v, meta, W)
    lv = [t.detach().clone().requires_grad_() for t in (q, k, v, meta)]
    y = lizard_cuda.swa(*lv, W)
    y.backward(dy)
    torch.cuda.synchronize()
    assert torch.equal(y_inf, y.detach())
    grp = H // Hkv
    for b, h in heads:
        hk = h // grp
        qs, ks, vs = q[b:b + 1, h:h + 1], k[b:b + 1, hk:hk + 1], v[b:b + 1, hk:hk + 1]
        ref, rg = _oracle(qs, ks, vs, meta, W, dy[b:b + 1, h:h + 1])
        tag = f"persistent swa B{B} H{H}/{Hkv} L{L} W{W} [{b},{h}]"
        assert_output(y[b:b + 1, h:h + 1], ref, tag + " y")
        assert_grad(lv[0].grad[b:b + 1, h:h + 1], rg[0], tag + " dq")
        if grp == 1:  # dk / dv sum over the group's heads
            assert_grad(lv[1].grad[b:b + 1, hk:hk + 1], rg[1], tag + " dk")
            assert_grad(lv[2].grad[b:b + 1, hk:hk + 1], rg[2], tag + " dv")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_swa_tc_close_to_warp_mma_kernel(dtype):
    """Same products, one softmax pass instead of the online rescaling: the
    outputs agree to bf16 rounding, the saved log-sum-exp to fp32 rounding."""
    import lizard_cuda
    q, k, v, meta, dy = _inputs(2, 4, 2, 333, 64, 4, dtype, seed=5)
    outs = []
    for on in (1, 0):
        old = _set_tc(on)
        try:
            lv = [t.detach().clone().requires_grad_() for t in (q, k, v, meta)]
            y = lizard_cuda.swa(*lv, 64)
            y.backward(dy)
            outs.append((y.detach().float(), [t.grad.float() for t in lv]))
        finally:
            _set_tc(old)
    (y1, g1), (y2, g2) = outs
    diff = (y1 - y2).abs().max().item()
    assert diff <= 2 ** -7 * y2.abs().max().item(), diff
    for a, b in zip(g1, g2):
        assert (a - b).abs().max().item() <= 2e-2 * b.abs().max().item()


def test_swa_rope_tc_reads_projections_in_place():
    """The Lizard layer's call: projections [B, L, heads * 64] (bf16) read as
    heads, RoPE inside, GQA 8 / 2, window 64, 4 sinks; forward and backward
    against the oracle on the rotated inputs."""
    import lizard_cuda
    g = torch.Generator(device=DEV).manual_seed(11)
    B, L, H, Hkv, D, W = 2, 384, 8, 2, 64, 64
    qp = torch.randn(B, L, H * D, generator=g, device=DEV).bfloat16()
    kp = torch.randn(B, L, Hkv * D, generator=g, device=DEV).bfloat16()
    vp = torch.randn(B, L, Hkv * D, generator=g, device=DEV).bfloat16()
    meta = torch.randn(4, generator=g, device=DEV)
    dy = torch.randn(B, H, L, D, generator=g, device=DEV).bfloat16()
    cos, sin = (t.to(DEV).expand(B, L, D) for t in orc.rotary_tables(L, D, 5e5))
    lv = [t.detach().clone().requires_grad_() for t in (qp, kp, vp, meta)]
    q = lv[0].view(B, L, H, D).transpose(1, 2)
    k = lv[1].view(B, L, Hkv, D).transpose(1, 2)
    v = lv[2].view(B, L, Hkv, D).transpose(1, 2)
    y = lizard_cuda.swa_rope(q, k, v, cos, sin, lv[3], W)
    y.backward(dy)
    with torch.no_grad():
        y_inf = lizard_cuda.swa_rope(q, k, v, cos, sin, lv[3], W)
    assert torch.equal(y, y_inf)  # the same kernel with and without the saved buffers
    c, s = cos.double().cpu(), sin.double().cpu()
    rl = [t.detach().double().cpu().clone().requires_grad_() for t in (qp, kp, vp, meta)]
    qr = orc.rope(rl[0].view(B, L, H, D).transpose(1, 2), c, s)
    kr = orc.rope(rl[1].view(B, L, Hkv, D).transpose(1, 2), c, s)
    vr = rl[2].view(B, L, Hkv, D).transpose(1, 2)
    ref = orc.awa(qr, _rep(kr, H // Hkv), _rep(vr, H // Hkv), rl[3], W)
    ref.backward(dy.double().cpu())
    assert_output(y, ref.float(), "swa_rope tc y")
    for t, r, n in zip(lv, rl, ("dq", "dk", "dv", "dmeta")):
        assert_grad(t.grad, r.grad.float(), f"swa_rope tc {n}")


# windows 65 ... 128 (the reference's training configs use 128): the wider
# tensor-core kernels (128 query rows against 256 keys in two halves; dq in four
# 64-key quarters; dk / dv over four 64-row query items per head)
@pytest.mark.parametrize("B,H,Hkv,L,W,n_meta,dtype", [
    (1, 2, 2, 1, 128, 4, torch.bfloat16),     # one token
    (2, 4, 2, 127, 128, 4, torch.bfloat16),   # one partial 128-row block
    (1, 4, 1, 300, 128, 3, torch.float32),    # fp32: residual logits; grp 4
    (2, 2, 2, 257, 65, 4, torch.bfloat16),    # the smallest wide window
    (1, 8, 2, 300, 100, 0, torch.bfloat16),   # no sinks, even window, grp 4
    (1, 2, 2, 1000, 127, 2, torch.float32),   # odd window, ragged tail
    (1, 2, 2, 2048, 128, 4, torch.bfloat16),  # config-3 length
])
def test_swa_tc_wide_window_matches_oracle(B, H, Hkv, L, W, n_meta, dtype):
    test_swa_tc_matches_oracle(B, H, Hkv, L, W, n_meta, dtype)


def _cuda_kernel_names(fn):
    from torch.profiler import ProfilerActivity, profile
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return {e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA}


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_swa_tc_wide_window_runs_tensor_core_kernels(dtype):
    """Window 128: a training step runs the wide tensor-core forward, dq and
    dk / dv kernels, and agrees with the 64-row warp-MMA kernels (switch off)
    to bf16 rounding."""
    import lizard_cuda
    q, k, v, meta, dy = _inputs(2, 4, 2, 333, 128, 4, dtype, seed=6)
    outs = []
    for on in (1, 0):
        old = _set_tc(on)
        try:
            lv = [t.detach().clone().requires_grad_() for t in (q, k, v, meta)]

            def step():
                y = lizard_cuda.swa(*lv, 128)
                y.backward(dy)
                outs.append((y.detach().float(), [t.grad.float() for t in lv]))
            names = _cuda_kernel_names(step)
            wide = {n for n in names if "tc128" in n}
            if on:
                assert len(wide) == 3, sorted(names)
            else:
                assert not wide, sorted(names)
        finally:
            _set_tc(old)
    (y1, g1), (y2, g2) = outs
    diff = (y1 - y2).abs().max().item()
    assert diff <= 2 ** -7 * y2.abs().max().item(), diff
    for a, b in zip(g1, g2):
        assert (a - b).abs().max().item() <= 2e-2 * b.abs().max().item()


def test_swa_tc_wide_window_is_deterministic():
    """Two identical window-128 training steps give bit-identical outputs and
    gradients (every sum in a fixed order) at several waves of CTAs."""
    import lizard_cuda
    q, k, v, meta, dy = _inputs(4, 32, 8, 2048, 128, 4, torch.bfloat16, seed=9)
    res = []
    for _ in range(2):
        lv = [t.detach().clone().requires_grad_() for t in (q, k, v, meta)]
        y = lizard_cuda.swa(*lv, 128)
        y.backward(dy)
        res.append([y.detach()] + [t.grad for t in lv])
    for a, b, n in zip(res[0], res[1], ("y", "dq", "dk", "dv", "dmeta")):
        assert torch.equal(a, b), f"{n} differs between two identical steps"


def test_swa_rope_wide_window_matches_oracle():
    """The layer's fused call at window 128 (the reference's training setting):
    bf16 projections read as heads, RoPE inside, GQA 8 / 2, 4 sinks; forward
    and backward against the oracle on the rotated inputs."""
    import lizard_cuda
    g = torch.Generator(device=DEV).manual_seed(12)
    B, L, H, Hkv, D, W = 2, 400, 8, 2, 64, 128
    qp = torch.randn(B, L, H * D, generator=g, device=DEV).bfloat16()
    kp = torch.randn(B, L, Hkv * D, generator=g, device=DEV).bfloat16()
    vp = torch.randn(B, L, Hkv * D, generator=g, device=DEV).bfloat16()
    meta = torch.randn(4, generator=g, device=DEV)
    dy = torch.randn(B, H, L, D, generator=g, device=DEV).bfloat16()
    cos, sin = (t.to(DEV).expand(B, L, D) for t in orc.rotary_tables(L, D, 5e5))
    lv = [t.detach().clone().requires_grad_() for t in (qp, kp, vp, meta)]
    q = lv[0].view(B, L, H, D).transpose(1, 2)
    k = lv[1].view(B, L, Hkv, D).transpose(1, 2)
    v = lv[2].view(B, L, Hkv, D).transpose(1, 2)
    y = lizard_cuda.swa_rope(q, k, v, cos, sin, lv[3], W)
    y.backward(dy)
    with torch.no_grad():
        y_inf = lizard_cuda.swa_rope(q, k, v, cos, sin, lv[3], W)
    assert torch.equal(y, y_inf)
    c, s = cos.double().cpu(), sin.double().cpu()
    rl = [t.detach().double().cpu().clone().requires_grad_() for t in (qp, kp, vp, meta)]
    qr = orc.rope(rl[0].view(B, L, H, D).transpose(1, 2), c, s)
    kr = orc.rope(rl[1].view(B, L, Hkv, D).transpose(1, 2), c, s)
    vr = rl[2].view(B, L, Hkv, D).transpose(1, 2)
    ref = orc.awa(qr, _rep(kr, H // Hkv), _rep(vr, H // Hkv), rl[3], W)
    ref.backward(dy.double().cpu())
    assert_output(y, ref.float(), "swa_rope window 128 y")
    for t, r, n in zip(lv, rl, ("dq", "dk", "dv", "dmeta")):
        assert_grad(t.grad, r.grad.float(), f"swa_rope window 128 {n}")
