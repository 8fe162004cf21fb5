"""GLA kernels on the GPU against the reference fixtures and the CPU oracle.

Every test runs under both schedules of the kernels: the sequential walk
over each head's chunks and the chunk-parallel schedule."""
import functools
import math

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


@pytest.fixture(autouse=True, params=["walk", "split"])
def schedule(request, _lib):
    from lizard_cuda import _lib as binding
    prev = binding.set_schedule(request.param)
    yield request.param
    binding.set_schedule(prev)


def cuda_gla(fq, fk, v, lg, dy=None, chunk=64):
    import lizard_cuda
    leaves = [t.detach().to(DEV).clone().requires_grad_() for t in (fq, fk, v, lg)]
    y = lizard_cuda.gla(*leaves, chunk)
    if dy is not None:
        y.backward(dy.to(DEV).to(y.dtype))
    return y, [t.grad for t in leaves]


def oracle_gla(fq, fk, v, lg, dy=None):
    leaves = [t.detach().float().cpu().clone().requires_grad_() for t in (fq, fk, v, lg)]
    y = orc.gla(*leaves)
    if dy is not None:
        y.backward(dy.float().cpu())
    return y.detach(), [t.grad for t in leaves]


GRAD_NAMES = ("dfq", "dfk", "dv", "dlog_gamma")


@pytest.mark.parametrize("name", list(cases.GLA_CASES))
def test_gla_matches_reference_fixture(name):
    fx = load_golden(name)
    inp = fx["inputs"]
    y, grads = cuda_gla(inp["fq"], inp["fk"], inp["v"], inp["log_gamma"], inp["dy"])
    assert y.dtype == torch.bfloat16
    assert_output(y, fx["y"], f"{name} y")
    for g, key in zip(grads, GRAD_NAMES):
        assert g.dtype == fx["inputs"][{"dfq": "fq", "dfk": "fk", "dv": "v",
                                        "dlog_gamma": "log_gamma"}[key]].dtype
        assert_grad(g, fx[key + "_b"], f"{name} {key}")


def baseline_inputs(B, H, L, Fd, D, per_head, seed=0, device=DEV):
    """fq, fk = softplus(N(0,1))/sqrt(D), v ~ N(0,1),
    log_gamma = logsigmoid(N(3, 1.5)), dO ~ N(0,1); seeded on the device."""
    g = torch.Generator(device=device).manual_seed(seed)
    fq = (F.softplus(torch.randn(B, H, L, Fd, generator=g, device=device)) / math.sqrt(D)).bfloat16()
    fk = (F.softplus(torch.randn(B, H, L, Fd, generator=g, device=device)) / math.sqrt(D)).bfloat16()
    v = torch.randn(B, H, L, D, generator=g, device=device).bfloat16()
    shape = (B, H, L) if per_head else (B, L)
    lg = F.logsigmoid(3 + 1.5 * torch.randn(shape, generator=g, device=device))
    dy = torch.randn(B, H, L, D, generator=g, device=device)
    return fq, fk, v, lg, dy


CFG2_HEADS = ((0, 0), (3, 17), (5, 31), (7, 8))


@functools.lru_cache(maxsize=None)
def _cfg2_reference():
    fq, fk, v, lg, _ = baseline_inputs(8, 32, 2048, 128, 128, per_head=True)
    refs = {}
    for b, h in CFG2_HEADS:
        sl = (slice(b, b + 1), slice(h, h + 1))
        refs[b, h] = oracle_gla(fq[sl], fk[sl], v[sl], lg[sl])[0]
    return refs


def test_gla_config2_forward_sampled_heads():
    """B=8, L=2048, H=32, F=D=128, per-head gate; 4 (b, h) slices checked."""
    import lizard_cuda
    fq, fk, v, lg, _ = baseline_inputs(8, 32, 2048, 128, 128, per_head=True)
    with torch.no_grad():
        y = lizard_cuda.gla(fq, fk, v, lg)
    torch.cuda.synchronize()
    for (b, h), ref in _cfg2_reference().items():
        sl = (slice(b, b + 1), slice(h, h + 1))
        assert_output(y[sl], ref, f"cfg2 y[{b},{h}]")


@functools.lru_cache(maxsize=None)
def _cfg3_reference():
    fq, fk, v, lg, dy = baseline_inputs(1, 32, 2048, 64, 64, per_head=False)
    ys, dfq, dfk, dv, dlg = [], [], [], [], torch.zeros(1, 2048, dtype=torch.float32)
    for h0 in range(0, 32, 8):
        sl = (slice(None), slice(h0, h0 + 8))
        r, (a, b_, c, d) = oracle_gla(fq[sl], fk[sl], v[sl], lg, dy[sl].bfloat16())
        ys.append(r), dfq.append(a), dfk.append(b_), dv.append(c)
        dlg += d
    return torch.cat(ys, 1), (torch.cat(dfq, 1), torch.cat(dfk, 1), torch.cat(dv, 1), dlg)


def test_gla_config3_forward_backward_all_heads():
    """B=1, L=2048, H=32, F=D=64, per-token gate shared by the heads."""
    fq, fk, v, lg, dy = baseline_inputs(1, 32, 2048, 64, 64, per_head=False)
    y, grads = cuda_gla(fq, fk, v, lg, dy)
    torch.cuda.synchronize()
    ref_y, ref_grads = _cfg3_reference()
    assert_output(y, ref_y, "cfg3 y")
    for got, ref, n in zip(grads, ref_grads, GRAD_NAMES):
        assert_grad(got, ref, f"cfg3 {n}")


def test_gla_schedules_agree():
    """Both schedules on one input: outputs and all gradients within bf16 rounding."""
    from lizard_cuda import _lib as binding
    fq, fk, v, lg, dy = baseline_inputs(2, 3, 777, 64, 48, per_head=False, seed=11)
    prev = binding.set_schedule("walk")
    try:
        yw, gw = cuda_gla(fq, fk, v, lg, dy)
        binding.set_schedule("split")
        ys, gs = cuda_gla(fq, fk, v, lg, dy)
    finally:
        binding.set_schedule(prev)
    assert_output(ys, yw.float(), "split vs walk y")
    for a, b, n in zip(gs, gw, GRAD_NAMES):
        assert_grad(a, b.float(), f"split vs walk {n}")


def test_gla_many_chunks_against_recurrent_float64():
    """256 chunks of one head (L=16384), F=D=64, per-token gate: the scan over
    chunks against the float64 recurrence."""
    import lizard_cuda
    fq, fk, v, lg, _ = baseline_inputs(1, 1, 16384, 64, 64, per_head=False, seed=9)
    with torch.no_grad():
        y = lizard_cuda.gla(fq, fk, v, lg)
    ref = orc.gla_recurrent(fq.double().cpu(), fk.double().cpu(), v.double().cpu(),
                            lg.double().cpu())
    assert_output(y, ref, "L=16384 y")


def test_gla_long_sequence_against_recurrent_float64():
    """64 chunks, F=D=128, per-head gate: the O(L F D) float64 recurrence."""
    import lizard_cuda
    fq, fk, v, lg, _ = baseline_inputs(1, 2, 4096, 128, 128, per_head=True, seed=3)
    with torch.no_grad():
        y = lizard_cuda.gla(fq, fk, v, lg)
    ref = orc.gla_recurrent(fq.double().cpu(), fk.double().cpu(), v.double().cpu(),
                            lg.double().cpu())
    assert_output(y, ref, "L=4096 y")


CFG4_HEADS = ((0, 0), (1, 13))


@functools.lru_cache(maxsize=None)
def _cfg4_long_reference(L):
    """float64 forward and gradients of two sampled heads, chunk by chunk."""
    fq, fk, v, lg, dy = baseline_inputs(2, 16, L, 128, 128, per_head=True, seed=41)
    refs = {}
    for b, h in CFG4_HEADS:
        sl = (slice(b, b + 1), slice(h, h + 1))
        leaves = [t[sl].double().cpu().clone().requires_grad_() for t in (fq, fk, v, lg)]
        y = orc.gla_chunked(*leaves)
        y.backward(dy[sl].bfloat16().double().cpu())
        refs[b, h] = (y.detach(), [t.grad for t in leaves])
    return refs


@pytest.mark.parametrize("L", [8192, 16384])
def test_gla_config4_top_length_forward_backward(L):
    """Config 4's longest sequences (F = D = 128, per-head gate), forward and
    backward over 64 / 128 chunks of 128 tokens: with the walk schedule the
    tensor-core forward, state walk and chunk-gradient kernels (2 x 16
    sequences, 4096 chunk CTAs at L = 16384); two sampled heads against the
    float64 chunked form of the oracle, y and all four gradients."""
    fq, fk, v, lg, dy = baseline_inputs(2, 16, L, 128, 128, per_head=True, seed=41)
    y, grads = cuda_gla(fq, fk, v, lg, dy)
    torch.cuda.synchronize()
    for (b, h), (ref, rgrads) in _cfg4_long_reference(L).items():
        sl = (slice(b, b + 1), slice(h, h + 1))
        assert_output(y[sl], ref, f"L={L} y[{b},{h}]")
        for got, r, n in zip(grads, rgrads, GRAD_NAMES):
            assert_grad(got[sl], r, f"L={L} [{b},{h}] {n}")


@pytest.mark.parametrize("tc_on", [True, False])
@pytest.mark.parametrize("per_head,H,Hkv", [(False, 8, 8), (True, 4, 4), (False, 8, 2)])
def test_gla_f64_d64_training_tensor_core_and_warp_mma(tc_on, per_head, H, Hkv):
    """F = D = 64 (config 3's shape) with an odd tail of 76 tokens: with the
    switch on the chunk outputs and the per-chunk gradients run on the tensor
    cores over 128-token chunks (zero-padded 128-wide operands, the 64-token
    states at stride two), with it off on the warp-MMA kernels; both against
    the oracle, grouped keys / values included."""
    import lizard_cuda
    from lizard_cuda import _lib as binding
    lib = binding.load()
    fq, fk, v, lg, dy = baseline_inputs(2, H, 1100, 64, 64, per_head=per_head, seed=29)
    grp = H // Hkv
    fk_g, v_g = fk[:, ::grp].contiguous(), v[:, ::grp].contiguous()  # one key/value head a group
    old = lib.lz_gla_set_split_out_tc(int(tc_on))
    try:
        leaves = [t.detach().clone().requires_grad_() for t in (fq, fk_g, v_g, lg)]
        y = lizard_cuda.gla(*leaves)
        y.backward(dy.to(y.dtype))
        torch.cuda.synchronize()
    finally:
        lib.lz_gla_set_split_out_tc(old)
    rep = lambda t: t.repeat_interleave(grp, 1)  # noqa: E731
    ref, (rq, rk, rv, rl) = oracle_gla(fq, rep(fk_g), rep(v_g), lg, dy.bfloat16())
    # the gradients of grouped keys / values are the sums over each group
    rk = rk.view(2, Hkv, grp, 1100, 64).sum(2)
    rv = rv.view(2, Hkv, grp, 1100, 64).sum(2)
    assert_output(y, ref, f"F=D=64 tc={tc_on} y")
    for got, r, n in zip([t.grad for t in leaves], (rq, rk, rv, rl), GRAD_NAMES):
        assert_grad(got, r, f"F=D=64 tc={tc_on} {n}")


def test_gla_model_feature_dim_256():
    """F = 2 * feature_dim = 256 (the 1B model), D = 64, fwd + bwd."""
    fq, fk, v, lg, dy = baseline_inputs(1, 4, 300, 256, 64, per_head=False, seed=5)
    y, grads = cuda_gla(fq, fk, v, lg, dy)
    ref, rgrads = oracle_gla(fq, fk, v, lg, dy.bfloat16())
    assert_output(y, ref, "F=256 y")
    for got, r, n in zip(grads, rgrads, GRAD_NAMES):
        assert_grad(got, r, f"F=256 {n}")


def test_gla_without_grad_gives_the_same_output():
    """tests/test_kernels.py:102-107: bit-identical with and without autograd."""
    import lizard_cuda
    inp = cases.gla_case(70)
    fq, fk, v, lg = (inp[n].to(DEV) for n in ("fq", "fk", "v", "log_gamma"))
    y = lizard_cuda.gla(fq, fk, v.clone().requires_grad_(), lg)
    with torch.no_grad():
        assert torch.equal(lizard_cuda.gla(fq, fk, v, lg), y)


def test_gla_chunk_argument_does_not_change_the_result():
    import lizard_cuda
    inp = cases.gla_case(150)
    args = [inp[n].to(DEV) for n in ("fq", "fk", "v", "log_gamma")]
    with torch.no_grad():
        assert torch.equal(lizard_cuda.gla(*args, 16), lizard_cuda.gla(*args))


def test_gla_single_token_returns_v():
    """One token: the row sum uses the same rounded weight, so y = v exactly."""
    import lizard_cuda
    inp = cases.gla_case(1)
    fq, fk, v, lg = (inp[n].to(DEV) for n in ("fq", "fk", "v", "log_gamma"))
    with torch.no_grad():
        assert torch.equal(lizard_cuda.gla(fq, fk, v, lg), v)


def test_gla_very_strong_gate_keeps_only_the_current_token():
    import lizard_cuda
    inp = cases.gla_case(130)
    fq, fk, v = (inp[n].to(DEV) for n in ("fq", "fk", "v"))
    lg = torch.full(inp["log_gamma"].shape, -90.0, device=DEV)
    with torch.no_grad():
        y = lizard_cuda.gla(fq, fk, v, lg)
    assert orc.max_rel(y.cpu(), v.cpu()) < 4e-3


def test_gla_fp32_strided_inputs_give_fp32_grads():
    """The layer feeds fp32, non-contiguous tensors (src/lizard_attention.py:80-86)."""
    inp = cases.gla_case(90)
    fq, fk, v = (inp[n].float().transpose(1, 2).contiguous().transpose(1, 2)
                 for n in ("fq", "fk", "v"))
    assert not fq.is_contiguous()
    y, grads = cuda_gla(fq, fk, v, inp["log_gamma"], inp["dy"])
    assert all(g.dtype == torch.float32 for g in grads)
    ref, rgrads = oracle_gla(fq, fk, v, inp["log_gamma"], inp["dy"].bfloat16())
    assert_output(y, ref, "fp32 y")
    for got, r, n in zip(grads, rgrads, GRAD_NAMES):
        assert_grad(got, r, f"fp32 {n}")


def test_gla_poisoned_outputs_are_fully_written():
    """Direct C-ABI call into NaN-filled y and saved buffers: every element of
    y and of the saved rows is overwritten (no unwritten padding leaks)."""
    from lizard_cuda import _lib
    lib = _lib.load()
    inp = cases.gla_case(77, gates=(3,))
    fq, fk, v, lg = (inp[n].to(DEV).contiguous() for n in ("fq", "fk", "v", "log_gamma"))
    B, H, L, Fd = fq.shape
    D = v.shape[-1]
    y = torch.full((B, H, L, D), float("nan"), device=DEV, dtype=torch.bfloat16)
    nbytes = lib.lz_gla_saved_bytes(B, H, L, Fd, D, 64)
    saved = torch.full((nbytes // 4,), float("nan"), device=DEV, dtype=torch.float32)
    wbytes = lib.lz_gla_fwd_workspace_bytes(B, H, L, Fd, D, 64)
    ws = torch.full((wbytes // 4 + 1,), float("nan"), device=DEV, dtype=torch.float32)
    rc = lib.lz_gla_fwd(_lib.ptr(fq), _lib.ptr(fk), _lib.ptr(v), _lib.ptr(lg), 1, _lib.ptr(y),
                        _lib.ptr(saved), nbytes, _lib.ptr(ws), wbytes, B, H, L, Fd, D, 64,
                        _lib.stream_of(fq))
    _lib.check(rc, "gla forward")
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    y32 = saved[: B * H * L * D].view(B, H, L, D)
    assert torch.isfinite(y32).all()
    assert torch.equal(y32.bfloat16(), y)


@pytest.mark.parametrize("per_head,L", [(False, 300), (True, 256), (True, 1)])
def test_gla_f128_d128_forward_backward(per_head, L):
    """F = D = 128 runs the tensor-core forward (128-token chunks) and, in
    training mode, the 64-token state walk feeding the backward."""
    fq, fk, v, lg, dy = baseline_inputs(2, 3, L, 128, 128, per_head=per_head, seed=11)
    y, grads = cuda_gla(fq, fk, v, lg, dy)
    ref, rgrads = oracle_gla(fq, fk, v, lg, dy.bfloat16())
    assert_output(y, ref, f"F=D=128 L={L} y")
    for got, r, n in zip(grads, rgrads, GRAD_NAMES):
        assert_grad(got, r, f"F=D=128 L={L} {n}")


def _oracle_all_heads(fq, fk, v, lg, dy, group=8):
    """Oracle fwd+bwd head group by head group (the dense L x L temporaries of
    all heads at once would be large); the per-token gate gradient is summed."""
    ys, g = [], [[], [], [], None]
    for h0 in range(0, fq.shape[1], group):
        sl = (slice(None), slice(h0, h0 + group))
        lgs = lg[sl] if lg.dim() == 3 else lg
        r, (a, b_, c, d) = oracle_gla(fq[sl], fk[sl], v[sl], lgs, dy[sl].bfloat16())
        ys.append(r)
        g[0].append(a), g[1].append(b_), g[2].append(c)
        if lg.dim() == 3:
            g[3] = d if g[3] is None else torch.cat([g[3], d], 1)
        else:
            g[3] = d if g[3] is None else g[3] + d
    return torch.cat(ys, 1), [torch.cat(x, 1) for x in g[:3]] + [g[3]]


@pytest.mark.parametrize("per_head", [True, False])
def test_gla_f128_training_many_chunks(per_head):
    """F = D = 128, 64 sequences of 1100 tokens (8 chunks of 128 and a tail):
    with the walk schedule this is the tensor-core forward and backward."""
    fq, fk, v, lg, dy = baseline_inputs(2, 32, 1100, 128, 128, per_head=per_head, seed=17)
    y, grads = cuda_gla(fq, fk, v, lg, dy)
    torch.cuda.synchronize()
    ref, rgrads = _oracle_all_heads(fq, fk, v, lg, dy)
    assert_output(y, ref, "F=D=128 L=1100 y")
    for got, r, n in zip(grads, rgrads, GRAD_NAMES):
        assert_grad(got, r, f"F=D=128 L=1100 {n}")


@pytest.mark.parametrize("tc64", [True, False])
@pytest.mark.parametrize("per_head,H,Hkv,L", [(True, 4, 4, 1000), (False, 8, 2, 257),
                                             (True, 2, 2, 63), (False, 2, 1, 64)])
def test_gla_f128_both_tensor_core_forwards(schedule, tc64, per_head, H, Hkv, L):
    """F = D = 128 under the walk schedule on either tensor-core forward (two
    sequences per SM with 64-token chunks, or one with 128-token chunks), each
    followed by the tensor-core backward on the states it saved: output and all
    gradients against the oracle, grouped keys / values and ragged tails
    included, and the output the same with and without a saved buffer."""
    import lizard_cuda
    from lizard_cuda import _lib as binding
    if schedule != "walk":
        pytest.skip("the walk schedule's forward kernels")
    lib = binding.load()
    prev = lib.lz_gla_set_fwd_tc64(int(tc64))
    try:
        fq, fk, v, lg, dy = baseline_inputs(2, H, L, 128, 128, per_head=per_head, seed=41)
        grp = H // Hkv
        fk, v = fk[:, ::grp].contiguous(), v[:, ::grp].contiguous()
        y, grads = cuda_gla(fq, fk, v, lg, dy)
        with torch.no_grad():
            y_ng = lizard_cuda.gla(fq.to(DEV), fk.to(DEV), v.to(DEV), lg.to(DEV))
        torch.cuda.synchronize()
        assert torch.equal(y_ng, y.detach())
        rep = lambda t: t.repeat_interleave(grp, dim=1).float().cpu().requires_grad_()
        fkr, vr = rep(fk), rep(v)
        leaves = [fq.float().cpu().requires_grad_(), fkr, vr, lg.float().cpu().requires_grad_()]
        ref = orc.gla(leaves[0], fkr, vr, leaves[3])
        ref.backward(dy.bfloat16().float().cpu())
        dfk = fkr.grad.view(2, Hkv, grp, L, 128).sum(2)
        dv = vr.grad.view(2, Hkv, grp, L, 128).sum(2)
        kind = "64-token" if tc64 else "128-token"
        assert_output(y, ref.detach(), f"{kind} forward y")
        for got, r, n in zip(grads, [leaves[0].grad, dfk, dv, leaves[3].grad], GRAD_NAMES):
            assert_grad(got, r, f"{kind} forward {n}")
    finally:
        lib.lz_gla_set_fwd_tc64(prev)


def test_gla_f128_fp32_inputs_give_fp32_grads():
    """fp32 fq, fk, v at F = D = 128: fp32 gradients (stored without staging)."""
    fq, fk, v, lg, dy = baseline_inputs(1, 4, 520, 128, 128, per_head=True, seed=23)
    fq, fk, v = fq.float(), fk.float(), v.float()
    y, grads = cuda_gla(fq, fk, v, lg, dy)
    assert all(g.dtype == torch.float32 for g in grads)
    ref, rgrads = oracle_gla(fq, fk, v, lg, dy.bfloat16())
    assert_output(y, ref, "fp32 F=D=128 y")
    for got, r, n in zip(grads, rgrads, GRAD_NAMES):
        assert_grad(got, r, f"fp32 F=D=128 {n}")


def test_gla_f128_without_grad_gives_the_same_output():
    import lizard_cuda
    fq, fk, v, lg, _ = baseline_inputs(2, 2, 333, 128, 128, per_head=True, seed=12)
    y = lizard_cuda.gla(fq, fk, v.clone().requires_grad_(), lg)
    with torch.no_grad():
        assert torch.equal(lizard_cuda.gla(fq, fk, v, lg), y)


def test_gla_f128_backward_is_deterministic():
    """F = D = 128 training over 128 sequences of 16 chunks: two backward
    passes give bit-identical gradients, and sampled heads match the oracle.
    The reverse state walk hands each chunk from its prep warps to the MMA
    through one barrier that all 128 prep threads arrive on; without a sync
    among those threads a warp that ran ahead to the next chunk could complete
    the current chunk's phase early, and a few heads' state gradients per run
    came out wrong."""
    fq, fk, v, lg, dy = baseline_inputs(4, 32, 2048, 128, 128, per_head=True, seed=31)
    y0, g0 = cuda_gla(fq, fk, v, lg, dy)
    y1, g1 = cuda_gla(fq, fk, v, lg, dy)
    torch.cuda.synchronize()
    assert torch.equal(y0, y1)
    for n, a, b in zip(GRAD_NAMES, g0, g1):
        assert torch.equal(a, b), f"{n} differs between two identical backward passes"
    for b_, h in ((0, 0), (3, 29)):
        sl = (slice(b_, b_ + 1), slice(h, h + 1))
        ref, rg = oracle_gla(fq[sl], fk[sl], v[sl], lg[sl], dy[sl].bfloat16())
        assert_output(y0[sl], ref, f"F=D=128 [{b_},{h}] y")
        for got, r, n in zip(g0, rg, GRAD_NAMES):
            assert_grad(got[sl], r, f"F=D=128 [{b_},{h}] {n}")


@pytest.mark.parametrize("Fd,per_head,B,L", [(128, True, 4, 1100), (64, False, 8, 2048)])
def test_gla_chunk_gradient_prefetch_changes_nothing(schedule, Fd, per_head, B, L):
    """The per-chunk gradient kernel's L2 prefetch of the next CTA's operands
    (one SM count ahead in the grid) moves data only: at shapes with several
    waves of CTAs (a ragged last chunk at F = D = 128; F = D = 64 on the
    64-token states) the output and every gradient are bit-identical with the
    prefetch on and off."""
    from lizard_cuda import _lib as binding
    lib = binding.load()
    fq, fk, v, lg, dy = baseline_inputs(B, 32, L, Fd, Fd, per_head=per_head, seed=57)
    prev = lib.lz_gla_set_bwd_prefetch(1)
    try:
        y1, g1 = cuda_gla(fq, fk, v, lg, dy)
        lib.lz_gla_set_bwd_prefetch(0)
        y0, g0 = cuda_gla(fq, fk, v, lg, dy)
        torch.cuda.synchronize()
    finally:
        lib.lz_gla_set_bwd_prefetch(prev)
    assert torch.equal(y0, y1)
    for n, a, b in zip(GRAD_NAMES, g0, g1):
        assert torch.equal(a, b), f"{n} differs with the prefetch on and off"


def test_no_kernel_wait_timed_out():
    """Every bounded wait inside the tensor-core kernels completed."""
    from lizard_cuda import _lib
    torch.cuda.synchronize()
    assert _lib.device_timeout_flag() == 0
