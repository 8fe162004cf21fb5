"""Grouped-query (GQA) gla / swa and the fused RoPE operand pass on the GPU.

The reference's caller repeat_interleaves k and v to the query heads and
rotates q and k with torch ops (src/lizard_attention.py:73-88) before calling
kernels.gla / kernels.swa. The oracle here is exactly that: the CPU
restatement of the reference's attention on repeat_interleaved, rotated
inputs, with autograd carrying the gradients back through repeat_interleave
(the group sums) and the rotation.
"""
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


def _leaves(ts, dev):
    return [t.detach().to(dev).clone().requires_grad_() for t in ts]


def _rep(x, grp):
    return x.repeat_interleave(grp, dim=1)


# ------------------------------------------------------------------ SWA GQA
def oracle_swa_gqa(q, k, v, meta, window, dy):
    grp = q.shape[1] // k.shape[1]
    lv = [t.detach().float().cpu().clone().requires_grad_() for t in (q, k, v, meta)]
    y = orc.awa(lv[0], _rep(lv[1], grp), _rep(lv[2], grp), lv[3], window)
    y.backward(dy.float().cpu())
    return y.detach(), [t.grad for t in lv]


@pytest.mark.parametrize("H,Hkv,dtype", [(4, 2, torch.bfloat16), (8, 2, torch.float32),
                                         (6, 1, torch.bfloat16)])
def test_swa_gqa_matches_oracle(H, Hkv, dtype):
    import lizard_cuda
    g = torch.Generator(device=DEV).manual_seed(H * 10 + Hkv)
    B, L, D, W = 2, 300, 64, 70
    q = torch.randn(B, H, L, D, generator=g, device=DEV).to(dtype)
    k, v = (torch.randn(B, Hkv, L, D, generator=g, device=DEV).to(dtype) for _ in range(2))
    meta = torch.randn(3, generator=g, device=DEV)
    dy = torch.randn(B, H, L, D, generator=g, device=DEV).bfloat16()
    lv = _leaves((q, k, v, meta), DEV)
    y = lizard_cuda.swa(*lv, W)
    y.backward(dy)
    assert lv[1].grad.shape == (B, Hkv, L, D) and lv[2].grad.shape == (B, Hkv, L, D)
    ref, rg = oracle_swa_gqa(q, k, v, meta, W, dy)
    assert_output(y, ref, f"swa gqa {H}/{Hkv} y")
    for t, r, n in zip(lv, rg, ("dq", "dk", "dv", "dmeta")):
        assert_grad(t.grad, r, f"swa gqa {H}/{Hkv} {n}")


def test_swa_gqa_forward_equals_repeated_call():
    """Per query head the grouped forward and dq do the same arithmetic as a
    call on repeat_interleaved k, v: bit-identical y and dq."""
    import lizard_cuda
    g = torch.Generator(device=DEV).manual_seed(5)
    B, H, Hkv, L, D, W = 1, 8, 2, 257, 64, 64
    q = torch.randn(B, H, L, D, generator=g, device=DEV).bfloat16()
    k, v = (torch.randn(B, Hkv, L, D, generator=g, device=DEV).bfloat16() for _ in range(2))
    meta = torch.randn(4, generator=g, device=DEV)
    dy = torch.randn(B, H, L, D, generator=g, device=DEV).bfloat16()
    a = _leaves((q, k, v, meta), DEV)
    b = _leaves((q, _rep(k, H // Hkv), _rep(v, H // Hkv), meta), DEV)
    ya, yb = lizard_cuda.swa(*a, W), lizard_cuda.swa(*b, W)
    assert torch.equal(ya, yb)
    ya.backward(dy)
    yb.backward(dy)
    assert torch.equal(a[0].grad, b[0].grad)
    for i, n in ((1, "dk"), (2, "dv")):
        summed = b[i].grad.float().view(B, Hkv, H // Hkv, L, D).sum(2)
        assert_grad(a[i].grad, summed, f"grouped {n} vs summed repeated {n}")


# ------------------------------------------------------------------ GLA GQA
def oracle_gla_gqa(fq, fk, v, lg, dy):
    grp = fq.shape[1] // fk.shape[1]
    lv = [t.detach().double().cpu().clone().requires_grad_() for t in (fq, fk, v, lg)]
    y = orc.gla(lv[0], _rep(lv[1], grp), _rep(lv[2], grp), lv[3])
    y.backward(dy.double().cpu())
    return y.detach(), [t.grad for t in lv]


def _gla_inputs(B, H, Hkv, L, F, D, per_head, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    fq = (torch.nn.functional.softplus(torch.randn(B, H, L, F, generator=g, device=DEV))
          / F ** 0.5).bfloat16()
    fk = (torch.nn.functional.softplus(torch.randn(B, Hkv, L, F, generator=g, device=DEV))
          / F ** 0.5).bfloat16()
    v = torch.randn(B, Hkv, L, D, generator=g, device=DEV).bfloat16()
    shape = (B, H, L) if per_head else (B, L)
    lg = torch.nn.functional.logsigmoid(3 + 1.5 * torch.randn(*shape, generator=g, device=DEV))
    dy = torch.randn(B, H, L, D, generator=g, device=DEV).bfloat16()
    return fq, fk, v, lg, dy


@pytest.mark.parametrize("schedule", ["walk", "split"])
@pytest.mark.parametrize("shape", [(2, 4, 2, 300, 64, 64, 1), (1, 6, 2, 200, 32, 48, 0),
                                   (2, 4, 1, 384, 128, 128, 0)])
def test_gla_gqa_matches_oracle(schedule, shape):
    """Both schedules; F = D = 128 with aligned inputs runs the tensor-core
    forward and backward with the grouped key/value tiles."""
    import lizard_cuda
    from lizard_cuda import _lib
    B, H, Hkv, L, F, D, per_head = shape
    fq, fk, v, lg, dy = _gla_inputs(B, H, Hkv, L, F, D, per_head, seed=L + H)
    prev = _lib.set_schedule(schedule)
    try:
        lv = _leaves((fq, fk, v, lg), DEV)
        y = lizard_cuda.gla(*lv)
        y.backward(dy)
    finally:
        _lib.set_schedule(prev)
    assert lv[1].grad.shape == (B, Hkv, L, F) and lv[2].grad.shape == (B, Hkv, L, D)
    ref, rg = oracle_gla_gqa(fq, fk, v, lg, dy)
    what = f"gla gqa {shape} {schedule}"
    assert_output(y, ref.float(), f"{what} y")
    for t, r, n in zip(lv, rg, ("dfq", "dfk", "dv", "dlog_gamma")):
        assert_grad(t.grad, r.float(), f"{what} {n}")


@pytest.mark.parametrize("F,D", [(64, 64), (128, 128)])
def test_gla_gqa_forward_equals_repeated_call(F, D):
    import lizard_cuda
    B, H, Hkv, L = 2, 4, 2, 320
    fq, fk, v, lg, _ = _gla_inputs(B, H, Hkv, L, F, D, 1, seed=F)
    ya = lizard_cuda.gla(fq, fk, v, lg)
    yb = lizard_cuda.gla(fq, _rep(fk, 2), _rep(v, 2), lg)
    assert torch.equal(ya, yb)


def test_gla_gqa_bf16_grads_sum_in_fp32():
    """bf16 inputs give bf16 gradients; the grouped dfk / dv are summed in
    fp32 before the one rounding, so they sit within bf16 rounding of the
    fp32 sum of the per-head gradients of a repeated call."""
    import lizard_cuda
    B, H, Hkv, L, F, D = 1, 8, 2, 256, 64, 64
    fq, fk, v, lg, dy = _gla_inputs(B, H, Hkv, L, F, D, 0, seed=3)
    a = _leaves((fq, fk, v, lg), DEV)
    lizard_cuda.gla(*a).backward(dy)
    b = _leaves((fq, _rep(fk, 4).float(), _rep(v, 4).float(), lg), DEV)
    lizard_cuda.gla(*b).backward(dy)
    assert a[1].grad.dtype == torch.bfloat16
    for i, n in ((1, "dfk"), (2, "dv")):
        summed = b[i].grad.view(B, Hkv, 4, L, -1).sum(2)
        err = (a[i].grad.float() - summed).abs().max().item()
        assert err <= 2 ** -8 * summed.abs().max().item(), (n, err)


# ------------------------------------------------------------------ RoPE
def _torch_rope(x, cos, sin):
    """The rotation as the reference's caller evaluates it, in fp32."""
    return orc.rope(x.float(), cos.float(), sin.float())


@pytest.mark.parametrize("xdt,csdt", [(torch.float32, torch.float32),
                                      (torch.bfloat16, torch.bfloat16),
                                      (torch.float32, torch.bfloat16)])
def test_rope_split_is_bit_exact(xdt, csdt):
    """hi = bf16(r), lo = bf16(r - hi) for r = x cos + rotate_half(x) sin with
    each product and the sum rounded once, as the separate torch ops do; x is
    read in place from a projection layout [B, L, H * D]."""
    from lizard_cuda.rope import _tables, rope_split
    g = torch.Generator(device=DEV).manual_seed(2)
    B, H, L, D = 2, 3, 130, 64
    proj = torch.randn(B, L, H * D, generator=g, device=DEV).to(xdt)
    x = proj.view(B, L, H, D).transpose(1, 2)
    cos, sin = (t.to(DEV).to(csdt).expand(B, L, D) for t in orc.rotary_tables(L, D, 5e5))
    c, s, csb, csl = _tables(cos, sin, B, L, D)
    hi, lo = rope_split(x, c, s, csb, csl)
    r = _torch_rope(x, cos, sin)
    rh = r.bfloat16()
    assert torch.equal(hi, rh)
    assert torch.equal(lo, (r - rh.float()).bfloat16())


def test_rope_grad_is_bit_exact():
    from lizard_cuda.rope import _tables, rope_grad
    g = torch.Generator(device=DEV).manual_seed(4)
    B, H, L, D = 2, 3, 100, 64
    x = torch.randn(B, H, L, D, generator=g, device=DEV, requires_grad=True)
    cos, sin = (t.to(DEV) for t in orc.rotary_tables(L, D, 1e4))
    dr = torch.randn(B, H, L, D, generator=g, device=DEV)
    _torch_rope(x, cos, sin).backward(dr)
    c, s, csb, csl = _tables(cos, sin, B, L, D)
    assert torch.equal(rope_grad(dr, c, s, csb, csl, torch.float32), x.grad)


@pytest.mark.parametrize("H,Hkv,xdt", [(4, 2, torch.float32), (4, 4, torch.bfloat16)])
def test_swa_rope_matches_oracle(H, Hkv, xdt):
    """swa_rope(q, k, v, cos, sin) against the reference caller's path:
    rotate (fp32), repeat_interleave k and v, sliding-window attention."""
    import lizard_cuda
    g = torch.Generator(device=DEV).manual_seed(H + Hkv)
    B, L, D, W = 2, 200, 64, 48
    qp = torch.randn(B, L, H * D, generator=g, device=DEV).to(xdt)
    kp = torch.randn(B, L, Hkv * D, generator=g, device=DEV).to(xdt)
    v = torch.randn(B, Hkv, L, D, generator=g, device=DEV).to(xdt)
    meta = torch.randn(4, generator=g, device=DEV)
    dy = torch.randn(B, H, L, D, generator=g, device=DEV).bfloat16()
    cos, sin = (t.to(DEV).expand(B, L, D) for t in orc.rotary_tables(L, D, 5e5))
    qp_, kp_, v_, meta_ = _leaves((qp, kp, v, meta), DEV)
    q = qp_.view(B, L, H, D).transpose(1, 2)
    k = kp_.view(B, L, Hkv, D).transpose(1, 2)
    y = lizard_cuda.swa_rope(q, k, v_, cos, sin, meta_, W)
    y.backward(dy)
    lv = [t.detach().float().cpu().clone().requires_grad_() for t in (qp, kp, v, meta)]
    qr = orc.rope(lv[0].view(B, L, H, D).transpose(1, 2), cos.cpu(), sin.cpu())
    kr = orc.rope(lv[1].view(B, L, Hkv, D).transpose(1, 2), cos.cpu(), sin.cpu())
    grp = H // Hkv
    ref = orc.awa(qr, _rep(kr, grp), _rep(lv[2], grp), lv[3], W)
    ref.backward(dy.float().cpu())
    what = f"swa_rope {H}/{Hkv} {xdt}"
    assert_output(y, ref.detach(), f"{what} y")
    for t, r, n in zip((qp_, kp_, v_, meta_), lv, ("dq", "dk", "dv", "dmeta")):
        assert t.grad.dtype == t.dtype
        assert_grad(t.grad.float(), r.grad, f"{what} {n}")


@pytest.mark.parametrize("schedule", ["walk", "split"])
@pytest.mark.parametrize("shape", [(2, 8, 2, 300, 64, 64), (1, 4, 1, 200, 256, 64)])
def test_gla_gqa_inference_shared_gate(schedule, shape):
    """Without autograd and with a gate shared by the heads, the chunk-parallel
    schedule keeps one state per key/value head (the query heads of a group
    have identical states): the output matches the oracle under both schedules."""
    import lizard_cuda
    from lizard_cuda import _lib
    B, H, Hkv, L, F, D = shape
    fq, fk, v, lg, _ = _gla_inputs(B, H, Hkv, L, F, D, 0, seed=L + F)
    prev = _lib.set_schedule(schedule)
    try:
        with torch.no_grad():
            y = lizard_cuda.gla(fq, fk, v, lg)
    finally:
        _lib.set_schedule(prev)
    ref = orc.gla(fq.double().cpu(), _rep(fk, H // Hkv).double().cpu(),
                  _rep(v, H // Hkv).double().cpu(), lg.double().cpu())
    assert_output(y, ref.float(), f"gla gqa inference {shape} {schedule}")


@pytest.fixture(params=[1, 0], ids=["tc", "warp_mma"])
def swa_tc(request):
    """SWA forwards on the tensor cores (the default) or on the 64-row kernels."""
    from lizard_cuda import _lib
    lib = _lib.load()
    old = lib.lz_swa_set_tc(request.param)
    yield request.param
    lib.lz_swa_set_tc(old)


@pytest.mark.parametrize("D,xdt,csdt,H,Hkv,W,L", [
    (64, torch.bfloat16, torch.bfloat16, 4, 2, 64, 200),
    (64, torch.float32, torch.float32, 4, 4, 16, 130),
    (128, torch.bfloat16, torch.float32, 2, 1, 100, 257),
    (32, torch.float32, torch.bfloat16, 4, 2, 200, 64),
    (64, torch.bfloat16, torch.bfloat16, 4, 2, 128, 300),
])
def test_swa_rope_fused_equals_two_pass(D, xdt, csdt, H, Hkv, W, L, swa_tc):
    """The one-kernel forward (TMA tiles of the unrotated projections, rotation
    and split inside the CTA) equals rotating first and calling the SWA forward:
    the same output, saved buffer and rotated operands, bit for bit. With the
    tensor-core forward on, fp32 projections at its shape are declined (the two
    passes reach the same kernel). Window 128 covers the wide tensor-core
    forward's fused rotation."""
    from lizard_cuda import _lib
    from lizard_cuda.rope import _fused_forward, _tables, _two_pass_forward
    lib = _lib.load()
    g = torch.Generator(device=DEV).manual_seed(D + L)
    B = 2
    qp = torch.randn(B, L, H * D, generator=g, device=DEV).to(xdt)
    kp = torch.randn(B, L, Hkv * D, generator=g, device=DEV).to(xdt)
    vp = torch.randn(B, L, Hkv * D, generator=g, device=DEV).to(xdt)
    q = qp.view(B, L, H, D).transpose(1, 2)
    k = kp.view(B, L, Hkv, D).transpose(1, 2)
    v = vp.view(B, L, Hkv, D).transpose(1, 2)
    meta = torch.randn(4, generator=g, device=DEV)
    cos, sin = (t.to(DEV).to(csdt).expand(B, L, D) for t in orc.rotary_tables(L, D, 5e5))
    c, s, csb, csl = _tables(cos, sin, B, L, D)
    outs = []
    for fused in (True, False):
        y = torch.empty(B, H, L, D, device=DEV, dtype=torch.bfloat16)
        # zeroed: the alignment padding inside the buffer is written by neither path
        saved = torch.zeros(lib.lz_swa_saved_bytes(B, H, L, D), device=DEV, dtype=torch.uint8)
        if fused:
            rot = tuple(torch.empty(B, n, L, D, device=DEV, dtype=torch.bfloat16)
                        for n in (H, H, Hkv, Hkv))
            ok = _fused_forward(q, k, v, c, s, csb, csl, meta, W, y, saved, rot)
            if swa_tc and D == 64 and W <= 128 and xdt == torch.float32:
                assert not ok
                return
            assert ok
        else:
            rot = _two_pass_forward(q, k, v, c, s, csb, csl, meta, W, y, saved)
        outs.append((y, saved, rot))
    (y1, s1, r1), (y2, s2, r2) = outs
    assert torch.equal(y1, y2)
    assert torch.equal(s1, s2)
    for a, b_ in zip(r1, r2):
        assert torch.equal(a, b_)


@pytest.mark.parametrize("D,xdt", [(20, torch.bfloat16), (128, torch.float32)])
def test_swa_rope_fused_declines_shapes_outside_its_tiles(D, xdt):
    """Head dims outside {32, 64, 128}, or tiles that do not fit in shared memory
    (fp32 at D = 128), are declined without a launch; swa_rope then rotates first."""
    import lizard_cuda
    from lizard_cuda.rope import _fused_forward, _tables
    B, H, L = 1, 2, 100
    g = torch.Generator(device=DEV).manual_seed(D)
    q, k, v = (torch.randn(B, H, L, D, generator=g, device=DEV).to(xdt) for _ in range(3))
    meta = torch.randn(2, generator=g, device=DEV)
    cos, sin = (t.to(DEV) for t in orc.rotary_tables(L, D, 1e4))
    c, s, csb, csl = _tables(cos, sin, B, L, D)
    y = torch.empty(B, H, L, D, device=DEV, dtype=torch.bfloat16)
    assert not _fused_forward(q, k, v, c, s, csb, csl, meta, 16, y, None, None)
    out = lizard_cuda.swa_rope(q, k, v, cos, sin, meta, 16)
    qr, kr = orc.rope(q.double().cpu(), cos.double().cpu(), sin.double().cpu()), \
        orc.rope(k.double().cpu(), cos.double().cpu(), sin.double().cpu())
    ref = orc.awa(qr, kr, v.double().cpu(), meta.double().cpu(), 16)
    assert_output(out, ref.float(), f"swa_rope two-pass D={D}")


@pytest.mark.parametrize("shape", [(1, 4, 1, 300, 256, 64, 0), (2, 4, 2, 257, 256, 64, 1),
                                   (1, 4, 4, 200, 128, 64, 0), (1, 2, 2, 130, 128, 128, 1),
                                   (2, 8, 2, 513, 128, 64, 0), (1, 2, 1, 100, 256, 64, 0),
                                   (1, 8, 1, 260, 256, 64, 0)])
def test_gla_split_tensor_core_outputs(shape):
    """Chunk outputs of the chunk-parallel schedule on the tensor cores
    (inference) against the oracle and against the warp-MMA output kernel:
    one 128-token chunk per CTA, or, with a gate shared by the heads and
    grouped keys / values (one state per key/value head), one CTA per
    (key/value head, chunk) walking the group's query heads."""
    import lizard_cuda
    from lizard_cuda import _lib
    lib = _lib.load()
    B, H, Hkv, L, F, D, per_head = shape
    fq, fk, v, lg, _ = _gla_inputs(B, H, Hkv, L, F, D, per_head, seed=L + F + D)
    prev = _lib.set_schedule("split")
    ys = []
    try:
        for tc_on in (1, 0):
            old = lib.lz_gla_set_split_out_tc(tc_on)
            try:
                with torch.no_grad():
                    ys.append(lizard_cuda.gla(fq, fk, v, lg))
            finally:
                lib.lz_gla_set_split_out_tc(old)
    finally:
        _lib.set_schedule(prev)
    ref = orc.gla(fq.double().cpu(), _rep(fk, H // Hkv).double().cpu(),
                  _rep(v, H // Hkv).double().cpu(), lg.double().cpu())
    assert_output(ys[0], ref.float(), f"gla tc outputs {shape}")
    assert_output(ys[0], ys[1].float(), f"gla tc vs warp-MMA outputs {shape}")
