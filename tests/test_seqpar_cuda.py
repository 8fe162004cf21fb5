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
