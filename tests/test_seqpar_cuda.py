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


class _HostExchange:
    """all_gather of CUDA tensors through a gloo group on host copies (the test's
    stand-in for NCCL when every rank is a process on the same GPU)."""

    def __init__(self, dist):
        self.dist, self.rank, self.size = dist, dist.get_rank(), dist.get_world_size()

    def all_gather(self, t):
        flat = t.detach().contiguous().reshape(-1).cpu()
        out = torch.empty(self.size * flat.numel(), dtype=flat.dtype)
        self.dist.all_gather_into_tensor(out, flat)
        return out.view(self.size, *t.shape).to(t.device)


def _spawn(target, world, *args):
    """Run target(rank, world, port, *args, errq) in `world` processes that all
    use GPU 0 and talk over gloo; fail with the ranks' errors."""
    import socket

    import torch.multiprocessing as mp
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    procs = [ctx.Process(target=target, args=(r, world, port, *args, errq)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    for p in procs:
        if p.is_alive():
            p.kill()
            errs.append("a rank did not finish in 300 s")
    assert not errs and all(p.exitcode == 0 for p in procs), errs


def _rank_setup(rank, world, port):
    import os
    import sys
    from datetime import timedelta

    from conftest import ROOT
    for p in (ROOT, ROOT / "lizard-reproduction_b200", ROOT / "oracle", ROOT / "tests",
              ROOT / "tests" / "golden"):
        sys.path.insert(0, str(p))
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    return dist


def _swa_rank(rank, world, port, bounds, window, heads, kv_heads, errq):
    try:
        dist = _rank_setup(rank, world, port)
        import lizard_oracle as orc
        from lizard_cuda import seqpar
        from parity import assert_grad, assert_output
        g = torch.Generator(device=DEV).manual_seed(5)
        L, D, B = bounds[-1], 64, 2
        q = torch.randn(B, heads, L, D, generator=g, device=DEV).bfloat16()
        k = torch.randn(B, kv_heads, L, D, generator=g, device=DEV).bfloat16()
        v = torch.randn(B, kv_heads, L, D, generator=g, device=DEV).bfloat16()
        meta = torch.randn(4, generator=g, device=DEV)
        dy = torch.randn(B, heads, L, D, generator=g, device=DEV).bfloat16()
        a, b = bounds[rank], bounds[rank + 1]
        leaves = [t[:, :, a:b].contiguous().requires_grad_() for t in (q, k, v)]
        lm = meta.clone().requires_grad_()
        y = seqpar.swa_seqpar(*leaves, lm, window, comm=_HostExchange(dist))
        y.backward(dy[:, :, a:b])
        dmeta = lm.grad.cpu()
        dist.all_reduce(dmeta)  # meta is shared: its gradient is the sum over ranks
        rep = heads // kv_heads
        ref_leaves = [t.float().cpu().requires_grad_() for t in (q, k, v, meta)]
        ref = orc.awa(ref_leaves[0], ref_leaves[1].repeat_interleave(rep, 1),
                      ref_leaves[2].repeat_interleave(rep, 1), ref_leaves[3], window)
        ref.backward(dy.float().cpu())
        assert_output(y, ref.detach()[:, :, a:b], f"rank {rank} y")
        for got, rl, n in zip([t.grad for t in leaves], ref_leaves, ("dq", "dk", "dv")):
            assert_grad(got, rl.grad[:, :, a:b], f"rank {rank} {n}")
        assert_grad(dmeta, ref_leaves[3].grad, f"rank {rank} dmeta")
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent, then fail this process
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("bounds,window,heads,kv_heads", [
    ((0, 130, 256), 64, 4, 4),
    ((0, 70, 140, 300), 64, 8, 2),
    ((0, 130, 257), 128, 4, 2),   # slices just above window - 1 = 127
])
def test_swa_seqpar_ranks_on_one_gpu_match_oracle(bounds, window, heads, kv_heads):
    """SWA with the sequence split over P ranks (processes sharing GPU 0,
    exchanging over gloo): the halo of window - 1 keys / values from the
    previous rank and its gradient back, on the CUDA kernels; every rank's
    slice of y, dq, dk, dv and the summed dmeta against the unsharded oracle."""
    _spawn(_swa_rank, len(bounds) - 1, bounds, window, heads, kv_heads)


def _layer_rank(rank, world, port, bounds, errq):
    try:
        dist = _rank_setup(rank, world, port)
        from types import SimpleNamespace

        import cases
        import lizard_oracle as orc
        from lizard_cuda.layer import LizardAttention
        from parity import assert_grad, assert_output
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
        # the unsharded layer, run by every rank
        y_full = layer(x, (cos, sin))[0]
        y_full.backward(grad)
        full = {n: p.grad.detach().clone() for n, p in layer.named_parameters()}
        layer.zero_grad(set_to_none=True)
        a, b = bounds[rank], bounds[rank + 1]
        y = layer(x[:, a:b], (cos[:, a:b], sin[:, a:b]), seq_comm=_HostExchange(dist))[0]
        y.backward(grad[:, a:b])
        assert_output(y, y_full.detach()[:, a:b], f"rank {rank} layer y", layer=True)
        for n, p in layer.named_parameters():
            got = p.grad.detach().cpu()
            dist.all_reduce(got)  # the ranks' shares of a replicated parameter's gradient
            assert_grad(got, full[n], f"rank {rank} layer d{n}")
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent, then fail this process
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


def test_layer_sequence_parallel_matches_unsharded_layer():
    """A whole Lizard layer (GQA 4 / 2 heads, window 16, feature dim 32) over
    three uneven slices of the sequence, one process per rank on GPU 0: each
    rank's slice of the output and the parameter gradients summed over the
    ranks equal the same layer run on the whole sequence."""
    _spawn(_layer_rank, 3, (0, 40, 96, 160))
