"""Sequence-parallel GLA through the CUDA segment calls, with P virtual ranks
as threads of one process on one GPU (a barrier stands in for the all_gather),
against the unsharded oracle: forward output and all four gradients."""
import threading

import pytest
import torch

from parity import assert_grad, assert_output
from seq_oracle import ThreadExchange
from test_gla_cuda import GRAD_NAMES, baseline_inputs, oracle_gla

pytestmark = pytest.mark.gpu
DEV = "cuda"


def run_virtual_ranks(bounds, fq, fk, v, lg, dy, per_head):
    from lizard_cuda import seqpar
    P = len(bounds) - 1
    B, H, _, F = fq.shape
    D = v.shape[-1]
    shared = ThreadExchange.make_shared(P)
    out, errs = [None] * P, []

    def rank_main(r):
        try:
            a, b = bounds[r], bounds[r + 1]
            sl = lambda t: t[..., a:b, :].contiguous() if t.dim() == 4 else t[..., a:b].contiguous()  # noqa: E731
            comm = ThreadExchange(shared, r, P)
            ops = seqpar.CudaSegmentOps(B, H, b - a, F, D, int(per_head), torch.device(DEV))
            y, saved, seeded = seqpar.forward_phases(ops, comm, sl(fq), sl(fk), sl(v), sl(lg),
                                                     True)
            grads = seqpar.backward_phases(ops, comm, sl(fq), sl(fk), sl(v), saved,
                                           sl(dy).bfloat16(), seeded, torch.bfloat16)
            out[r] = (y, grads)
        except BaseException as e:  # noqa: BLE001
            errs.append(e)
            shared["barrier"].abort()

    threads = [threading.Thread(target=rank_main, args=(r,)) for r in range(P)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    torch.cuda.synchronize()
    assert not errs, errs
    y = torch.cat([o[0] for o in out], 2)
    grads = [torch.cat([o[1][i] for o in out], -2 if i < 3 else -1) for i in range(4)]
    return y, grads


@pytest.mark.parametrize("bounds,F,D,per_head", [
    ((0, 256, 512, 768, 1024), 128, 128, True),
    ((0, 300, 550, 700), 64, 64, False),
    ((0, 64, 130), 32, 48, True),
])
def test_seqpar_virtual_ranks_match_oracle(bounds, F, D, per_head):
    fq, fk, v, lg, dy = baseline_inputs(1, 4, bounds[-1], F, D, per_head=per_head, seed=21)
    y, grads = run_virtual_ranks(bounds, fq, fk, v, lg, dy, per_head)
    ref, rgrads = oracle_gla(fq, fk, v, lg, dy.bfloat16())
    assert_output(y, ref, f"seqpar P={len(bounds) - 1} y")
    for got, r, n in zip(grads, rgrads, GRAD_NAMES):
        assert_grad(got, r, f"seqpar P={len(bounds) - 1} {n}")


def test_seqpar_single_rank_equals_plain_call():
    """P = 1 runs the segment calls with no seed; same result as gla()."""
    import lizard_cuda
    fq, fk, v, lg, dy = baseline_inputs(2, 3, 333, 64, 64, per_head=False, seed=4)
    y, grads = run_virtual_ranks((0, 333), fq, fk, v, lg, dy, False)
    leaves = [t.detach().clone().requires_grad_() for t in (fq, fk, v, lg)]
    y2 = lizard_cuda.gla(*leaves)
    y2.backward(dy.bfloat16())
    assert_output(y, y2.float(), "P=1 y")
    for got, lf, n in zip(grads, leaves, GRAD_NAMES):
        assert_grad(got, lf.grad.float(), f"P=1 {n}")


def _threads(P, body):
    shared = ThreadExchange.make_shared(P)
    out, errs = [None] * P, []

    def main(r):
        try:
            out[r] = body(r, ThreadExchange(shared, r, P))
        except BaseException as e:  # noqa: BLE001
            errs.append(e)
            shared["barrier"].abort()

    threads = [threading.Thread(target=main, args=(r,)) for r in range(P)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    torch.cuda.synchronize()
    assert not errs, errs
    return out


@pytest.mark.parametrize("bounds,window,heads,kv_heads", [
    ((0, 130, 256), 64, 4, 4),
    ((0, 70, 140, 300), 64, 8, 2),
    ((0, 100, 227), 128, 4, 2),
])
def test_swa_seqpar_virtual_ranks_match_oracle(bounds, window, heads, kv_heads):
    """SWA with the sequence split over P virtual ranks (threads on one GPU):
    the halo of window - 1 keys / values from the previous rank and its
    gradient back, on the CUDA kernels, against the unsharded oracle."""
    import lizard_oracle as orc
    from lizard_cuda import seqpar
    g = torch.Generator(device=DEV).manual_seed(5)
    L, D, B = bounds[-1], 64, 2
    q = torch.randn(B, heads, L, D, generator=g, device=DEV).bfloat16()
    k = torch.randn(B, kv_heads, L, D, generator=g, device=DEV).bfloat16()
    v = torch.randn(B, kv_heads, L, D, generator=g, device=DEV).bfloat16()
    meta = torch.randn(4, generator=g, device=DEV)
    dy = torch.randn(B, heads, L, D, generator=g, device=DEV).bfloat16()

    def body(r, comm):
        a, b = bounds[r], bounds[r + 1]
        leaves = [t[:, :, a:b].contiguous().requires_grad_() for t in (q, k, v)]
        lm = meta.clone().requires_grad_()
        y = seqpar.swa_seqpar(*leaves, lm, window, comm=comm)
        y.backward(dy[:, :, a:b])
        return y.detach(), [t.grad for t in leaves], lm.grad

    out = _threads(len(bounds) - 1, body)
    y = torch.cat([o[0] for o in out], 2)
    grads = [torch.cat([o[1][i] for o in out], 2) for i in range(3)]
    dmeta = sum(o[2] for o in out)
    rep = heads // kv_heads
    ref_leaves = [t.float().cpu().requires_grad_() for t in (q, k, v, meta)]
    ref = orc.awa(ref_leaves[0], ref_leaves[1].repeat_interleave(rep, 1),
                  ref_leaves[2].repeat_interleave(rep, 1), ref_leaves[3], window)
    ref.backward(dy.float().cpu())
    assert_output(y, ref.detach(), f"swa seqpar P={len(bounds) - 1} y")
    for got, rl, n in zip(grads + [dmeta], ref_leaves, ("dq", "dk", "dv", "dmeta")):
        assert_grad(got, rl.grad, f"swa seqpar P={len(bounds) - 1} {n}")


def test_layer_sequence_parallel_matches_unsharded_layer():
    """A whole Lizard layer (GQA 4 / 2 heads, window 16, feature dim 32) over
    three uneven slices of the sequence, virtual ranks as threads: the
    concatenated output and the parameter gradients summed over the ranks
    equal the same layer run on the whole sequence."""
    import copy
    from types import SimpleNamespace

    import lizard_oracle as orc
    from lizard_cuda.layer import LizardAttention
    import cases
    bounds = (0, 40, 96, 160)
    cfg = SimpleNamespace(hidden_size=256, num_attention_heads=4, num_key_value_heads=2)
    layer = LizardAttention(cfg, 0, window=16, num_meta=4, feature_dim=32)
    cases.init_layer_params(layer, "cfg1")
    layer = layer.to(DEV)
    L = bounds[-1]
    torch.manual_seed(2)
    x = torch.randn(2, L, 256, device=DEV)
    grad = torch.randn(2, L, 256, device=DEV)
    cos, sin = (t.expand(2, -1, -1).contiguous().to(DEV)
                for t in orc.rotary_tables(L, 64, 500000.0))
    y_full = layer(x, (cos, sin))[0]
    y_full.backward(grad)
    full_grads = {n: p.grad.detach().clone() for n, p in layer.named_parameters()}

    def body(r, comm):
        a, b = bounds[r], bounds[r + 1]
        mine = copy.deepcopy(layer)
        mine.zero_grad(set_to_none=True)
        y = mine(x[:, a:b], (cos[:, a:b], sin[:, a:b]), seq_comm=comm)[0]
        y.backward(grad[:, a:b])
        return y.detach(), {n: p.grad for n, p in mine.named_parameters()}

    out = _threads(len(bounds) - 1, body)
    y = torch.cat([o[0] for o in out], 1)
    assert_output(y, y_full.detach(), "layer seqpar y", layer=True)
    for n, want in full_grads.items():
        got = sum(o[1][n] for o in out)
        assert_grad(got, want, f"layer seqpar d{n}")
