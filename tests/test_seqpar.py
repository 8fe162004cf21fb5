"""Sequence-parallel GLA orchestration over gloo ranks on the CPU.

Each rank runs lizard_cuda.seqpar's real forward/backward orchestration with
the float64 segment oracle (tests/seq_oracle.py) in place of the CUDA phases;
every rank's slice of y and of all four gradients must match the unsharded
oracle. World sizes 2 and 3, equal and unequal slices, per-token and per-head
gates.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(B, H, L, F, D, per_head, seed=0):
    g = torch.Generator().manual_seed(seed)
    bf = lambda t: t.bfloat16().float()  # noqa: E731  (values the kernels see)
    fq = bf(torch.nn.functional.softplus(torch.randn(B, H, L, F, generator=g)) / F ** 0.5)
    fk = bf(torch.nn.functional.softplus(torch.randn(B, H, L, F, generator=g)) / F ** 0.5)
    v = bf(torch.randn(B, H, L, D, generator=g))
    lg = torch.nn.functional.logsigmoid(2 + torch.randn((B, H, L) if per_head else (B, L),
                                                        generator=g))
    dy = bf(torch.randn(B, H, L, D, generator=g))
    return fq, fk, v, lg, dy


def _worker(rank, world, port, bounds, per_head, errq, exchange="all_gather"):
    import sys
    for p in (ROOT, ROOT / "lizard-reproduction_b200", ROOT / "oracle", ROOT / "tests"):
        sys.path.insert(0, str(p))
    try:
        import torch.distributed as dist
        import lizard_oracle as orc
        from lizard_cuda import seqpar
        from seq_oracle import OracleSegmentOps
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        B, H, F, D = 2, 3, 8, 6
        L = bounds[-1]
        fq, fk, v, lg, dy = _inputs(B, H, L, F, D, per_head)
        a, b = bounds[rank], bounds[rank + 1]
        sl = lambda t: t[..., a:b, :] if t.dim() == 4 else t[..., a:b]  # noqa: E731
        leaves = [sl(t).clone().requires_grad_() for t in (fq, fk, v, lg)]
        y = seqpar.gla_seqpar(*leaves, ops=OracleSegmentOps(per_head, H), exchange=exchange)
        y.backward(sl(dy))
        # unsharded float64 oracle
        ref_leaves = [t.double().clone().requires_grad_() for t in (fq, fk, v, lg)]
        ref = orc.gla(*ref_leaves)
        ref.backward(dy.double())
        checks = [("y", y, sl(ref.detach()))] + [
            (n, lf.grad, sl(r.grad)) for n, lf, r in zip(("dfq", "dfk", "dv", "dlog_gamma"),
                                                        leaves, ref_leaves)]
        for n, got, want in checks:
            err = (got.double() - want).abs().max().item() / want.abs().max().item()
            if not err < 1e-5:
                raise AssertionError(f"rank {rank}: {n} max rel err {err:.3e}")
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent, then fail this process
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("exchange", ["all_gather", "chain"])
@pytest.mark.parametrize("bounds,per_head", [
    ((0, 96, 192), False),        # 2 ranks, equal 96-token slices (chunk tails on both)
    ((0, 128, 200, 330), True),   # 3 ranks, unequal slices, per-head gates
    ((0, 64, 128, 130), False),   # 3 ranks, a 2-token last slice
])
def test_seqpar_matches_unsharded_oracle(bounds, per_head, exchange):
    """The chunk-state summaries moved by one all_gather per direction, or by
    the rank-to-rank send / recv chain: every rank's slice matches."""
    world = len(bounds) - 1
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, bounds, per_head, errq, exchange))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    for p in procs:
        if p.is_alive():
            p.kill()
            errs.append("a rank did not finish in 180 s")
    assert not errs and all(p.exitcode == 0 for p in procs), errs


def _swa_worker(rank, world, port, bounds, window, heads, kv_heads, errq):
    import sys
    for p in (ROOT, ROOT / "lizard-reproduction_b200", ROOT / "oracle", ROOT / "tests"):
        sys.path.insert(0, str(p))
    try:
        import torch.distributed as dist
        import lizard_oracle as orc
        from lizard_cuda import seqpar
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=60))
        B, D, L = 2, 8, bounds[-1]
        g = torch.Generator().manual_seed(3)
        q = torch.randn(B, heads, L, D, generator=g, dtype=torch.float64)
        k = torch.randn(B, kv_heads, L, D, generator=g, dtype=torch.float64)
        v = torch.randn(B, kv_heads, L, D, generator=g, dtype=torch.float64)
        meta = torch.randn(3, generator=g, dtype=torch.float64)
        dy = torch.randn(B, heads, L, D, generator=g, dtype=torch.float64)
        rep = heads // kv_heads

        def attn(q_, k_, v_, m_, w_):  # the float64 oracle with grouped keys / values
            return orc.awa(q_, k_.repeat_interleave(rep, 1), v_.repeat_interleave(rep, 1), m_, w_)

        a, b = bounds[rank], bounds[rank + 1]
        leaves = [t[:, :, a:b].clone().requires_grad_() for t in (q, k, v)]
        lm = meta.clone().requires_grad_()
        y = seqpar.swa_seqpar(*leaves, lm, window, attn=attn)
        y.backward(dy[:, :, a:b])
        dist.all_reduce(lm.grad)  # meta is shared: its gradient is the sum over ranks
        ref_leaves = [t.clone().requires_grad_() for t in (q, k, v, meta)]
        ref = attn(*ref_leaves, window)
        ref.backward(dy)
        checks = [("y", y, ref.detach()[:, :, a:b])] + [
            (n, lf.grad, r.grad[:, :, a:b]) for n, lf, r in zip(("dq", "dk", "dv"), leaves,
                                                              ref_leaves)] + [
            ("dmeta", lm.grad, ref_leaves[3].grad)]
        for n, got, want in checks:
            err = (got - want).abs().max().item() / want.abs().max().item()
            if not err < 1e-10:
                raise AssertionError(f"rank {rank}: {n} max rel err {err:.3e}")
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:  # report to the parent, then fail this process
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("bounds,window,heads,kv_heads", [
    ((0, 40, 80), 16, 2, 2),          # 2 ranks, halo of 15 rows
    ((0, 30, 51, 90), 21, 4, 2),      # 3 ranks, unequal slices, a slice as long as the halo,
                                      # grouped keys / values
    ((0, 25, 50), 1, 2, 1),           # window 1: no halo
])
def test_swa_seqpar_halo_matches_unsharded_oracle(bounds, window, heads, kv_heads):
    """Sliding-window attention with each rank holding a slice of the sequence:
    the last window - 1 keys / values of the previous rank arrive as a halo
    (and their gradients go back); every rank's slice of y and of dq, dk, dv,
    and the summed dmeta equal the unsharded float64 oracle."""
    world = len(bounds) - 1
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_swa_worker,
                         args=(r, world, port, bounds, window, heads, kv_heads, errq))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    for p in procs:
        if p.is_alive():
            p.kill()
            errs.append("a rank did not finish in 180 s")
    assert not errs and all(p.exitcode == 0 for p in procs), errs
