"""The CPU oracle against the reference's own outputs (golden fixtures) and
against the invariants the reference's tests pin (tests/test_lizard.py)."""
import functools
import math

import pytest
import torch
import torch.nn.functional as F

import cases
import lizard_oracle as orc
from conftest import load_golden

EXACT = 1e-10


def _leaves(*ts):
    return [t.detach().float().clone().requires_grad_() for t in ts]


@pytest.mark.parametrize("name", list(cases.GLA_CASES))
def test_oracle_gla_matches_reference_fixture(name):
    fx = load_golden(name)
    inp = cases.gla_case(**fx["kw"])
    for key in ("fq", "fk", "v", "log_gamma", "dy"):
        assert torch.equal(inp[key], fx["inputs"][key]), key
    fq, fk, v, lg = _leaves(inp["fq"], inp["fk"], inp["v"], inp["log_gamma"])
    y = orc.gla(fq, fk, v, lg)
    y.backward(inp["dy"])
    assert orc.max_rel(y, fx["y"]) < 1e-5
    for got, key in ((fq.grad, "dfq"), (fk.grad, "dfk"), (v.grad, "dv"), (lg.grad, "dlog_gamma")):
        assert orc.max_rel(got, fx[key]) < 1e-4, key


@pytest.mark.parametrize("name", list(cases.SWA_CASES))
def test_oracle_swa_matches_reference_fixture(name):
    fx = load_golden(name)
    kw, window = cases.SWA_CASES[name]
    inp = cases.swa_case(**kw)
    for key in ("q", "k", "v", "meta", "dy"):
        assert torch.equal(inp[key], fx["inputs"][key]), key
    q, k, v = _leaves(inp["q"], inp["k"], inp["v"])
    meta = inp["meta"].clone().requires_grad_()
    y = orc.awa(q, k, v, meta, window)
    y.backward(inp["dy"])
    assert orc.max_rel(y, fx["y"]) < 1e-5
    for got, key in ((q.grad, "dq"), (k.grad, "dk"), (v.grad, "dv")):
        assert orc.max_rel(got, fx[key]) < 1e-4, key
    if meta.numel():
        assert orc.max_rel(meta.grad, fx["dmeta"]) < 1e-4


@pytest.mark.parametrize("name", list(cases.LAYER_CASES))
def test_oracle_layer_matches_reference_fixture(name):
    fx = load_golden(name)
    c = fx["case"]
    layer = orc.LizardAttention(c["hidden"], c["heads"], c["kv_heads"], window=c["window"],
                                num_meta=c["num_meta"], feature_dim=c["feature_dim"])
    cases.init_layer_params(layer, c["init"])
    for n, p in layer.named_parameters():
        assert torch.equal(cases.checksum(p), fx["param_sums"][n]), n
    x, grad = cases.layer_inputs(c)
    assert torch.equal(cases.checksum(x), fx["x_sum"])
    cos, sin = orc.rotary_tables(c["length"], c["hidden"] // c["heads"], c["theta"])
    # the Llama embedding forms angles in fp32 (error ~1e-5 rad at position 255)
    assert orc.max_rel(cos, fx["cos"]) < 1e-4 and orc.max_rel(sin, fx["sin"]) < 1e-4
    y = layer(x, (fx["cos"], fx["sin"]))[0]
    y.backward(grad)
    assert orc.max_rel(y, fx["y"]) < 1e-5
    for n, p in layer.named_parameters():
        assert orc.max_rel(p.grad, fx["grads"][n]) < 1e-4, n


def _gla64(length, batch=2, heads=3, features=6, dim=5, per_head=False):
    fq = torch.randn(batch, heads, length, features).softmax(-1).double()
    fk = torch.randn(batch, heads, length, features).softmax(-1).double()
    v = torch.randn(batch, heads, length, dim).double()
    shape = (batch, heads, length) if per_head else (batch, length)
    lg = F.logsigmoid(2 * torch.randn(shape)).double()
    return fq, fk, v, lg


@pytest.mark.parametrize("length,per_head", [(1, False), (64, False), (300, True)])
def test_dense_matches_recurrent(length, per_head):
    torch.manual_seed(0)
    fq, fk, v, lg = _gla64(length, per_head=per_head)
    assert orc.rel(orc.gla(fq, fk, v, lg), orc.gla_recurrent(fq, fk, v, lg)) < EXACT


@pytest.mark.parametrize("length,per_head,chunk,shift", [
    (1, False, 256, 0.0), (77, False, 7, 0.0), (150, True, 64, 0.0), (300, True, 256, 0.0),
    (200, False, 16, -6.0)])
def test_chunked_matches_dense_with_gradients(length, per_head, chunk, shift):
    """gla_chunked (the long-sequence checker of the GPU tests) equals the dense
    form in float64, outputs and all four gradients, for chunk lengths that do
    and do not divide L, both gate layouts and strong decay."""
    torch.manual_seed(1)
    fq, fk, v, lg = _gla64(length, per_head=per_head)
    lg = lg + shift
    dy = torch.randn(*fq.shape[:3], v.shape[-1], dtype=torch.float64)
    outs = []
    for fn in (orc.gla, functools.partial(orc.gla_chunked, chunk=chunk)):
        leaves = [t.clone().requires_grad_() for t in (fq, fk, v, lg)]
        y = fn(*leaves)
        y.backward(dy)
        outs.append([y.detach()] + [t.grad for t in leaves])
    for a, b in zip(*outs):
        # one token: y = v, so the feature gradients are exactly zero in both
        assert (a - b).norm() <= EXACT * max(b.norm().item(), 1.0)


def test_gate_zero_keeps_only_current_token():
    torch.manual_seed(0)
    fq, fk, v, lg = _gla64(30)
    assert orc.rel(orc.gla(fq, fk, v, torch.full_like(lg, -math.inf)), v) < EXACT


def test_constant_values_stay_constant():
    torch.manual_seed(0)
    fq, fk, v, lg = _gla64(30)
    c = torch.full_like(v, 0.37)
    assert orc.rel(orc.gla(fq, fk, c, lg), c) < EXACT


def test_awa_without_sinks_and_window_is_causal_softmax():
    torch.manual_seed(0)
    q, k, v = (torch.randn(2, 3, 40, 8).double() for _ in range(3))
    expected = F.scaled_dot_product_attention(q, k, v, is_causal=True)
    assert orc.rel(orc.awa(q, k, v, torch.zeros(0).double(), 10**6), expected) < EXACT


def test_awa_many_sinks_equal_one_logsumexp_sink():
    torch.manual_seed(0)
    q, k, v = (torch.randn(2, 3, 40, 8).double() for _ in range(3))
    meta = torch.randn(4).double()
    one = torch.logsumexp(meta, 0, keepdim=True)
    assert orc.rel(orc.awa(q, k, v, meta, 16), orc.awa(q, k, v, one, 16)) < EXACT


def test_awa_gradient_only_inside_window():
    torch.manual_seed(0)
    q, k, v = (torch.randn(1, 2, 40, 8).double().requires_grad_() for _ in range(3))
    orc.awa(q, k, v, torch.randn(4).double(), 16)[:, :, 39].sum().backward()
    assert (k.grad[:, :, :24] == 0).all()
    assert (k.grad[:, :, 24:].abs().sum(-1) > 0).all()


def test_gla_and_awa_pass_gradcheck():
    torch.manual_seed(0)
    fq, fk, v, lg = (t.requires_grad_() for t in _gla64(6, batch=1, heads=2, features=3, dim=2))
    assert torch.autograd.gradcheck(orc.gla, (fq, fk, v, lg))
    q, k, v = (torch.randn(1, 2, 6, 3).double().requires_grad_() for _ in range(3))
    meta = torch.randn(4).double().requires_grad_()
    assert torch.autograd.gradcheck(lambda *a: orc.awa(*a, 3), (q, k, v, meta))
