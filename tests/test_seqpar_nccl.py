"""Sequence-parallel GLA over NCCL: one process per GPU (2 to 4 GPUs; skipped
with fewer), each owning a slice of one sequence, against the unsharded
oracle. NCCL's NVLS is switched off for this test, as for every multi-rank
test on a shared node."""
import os
import socket

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, errq, exchange="all_gather"):
    import sys
    for p in (ROOT, ROOT / "lizard-reproduction_b200", ROOT / "oracle", ROOT / "tests",
              ROOT / "tests" / "golden"):
        sys.path.insert(0, str(p))
    try:
        from datetime import timedelta

        import torch.distributed as dist
        from lizard_cuda import seqpar
        from parity import assert_grad, assert_output
        from test_gla_cuda import GRAD_NAMES, baseline_inputs, oracle_gla
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port),
                          NCCL_NVLS_ENABLE="0")
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        dist.init_process_group("nccl", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        L = 256 * world
        fq, fk, v, lg, dy = baseline_inputs(1, 4, L, 128, 128, per_head=True, seed=8,
                                            device=dev)
        a, b = rank * 256, (rank + 1) * 256
        leaves = [(t[..., a:b, :] if t.dim() == 4 else t[..., a:b]).detach().clone()
                  .requires_grad_() for t in (fq, fk, v, lg)]
        y = seqpar.gla_seqpar(*leaves, exchange=exchange)
        y.backward(dy[..., a:b, :].bfloat16())
        torch.cuda.synchronize()
        ref, rgrads = oracle_gla(fq, fk, v, lg, dy.bfloat16())
        assert_output(y, ref[..., a:b, :], f"rank {rank} {exchange} y")
        for got, r, n in zip([t.grad for t in leaves], rgrads, GRAD_NAMES):
            assert_grad(got, r[..., a:b, :] if r.dim() == 4 else r[..., a:b],
                        f"rank {rank} {exchange} {n}")
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as e:
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("exchange", ["all_gather", "chain"])
def test_seqpar_over_nccl_matches_oracle(exchange):
    """GLA sequence-parallel over NCCL (2 to 4 GPUs), the chunk-state summaries
    moved by one all_gather per direction or by the send / recv chain: every
    rank's slice of y and of the gradients against the oracle."""
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 or more GPUs")
    world = min(n, 4)
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    errq = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, errq, exchange))
             for r in range(world)]
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
