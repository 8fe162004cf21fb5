"""lz_swa_bwd_noalloc, the SWA backward for callers that cannot allocate
(a host that hands a plugin only its inputs and outputs, with no way to
request a workspace). It must give the same gradients as lz_swa_bwd with a
caller-owned workspace, on consecutive calls that share its fixed scratch.

This file is collected last on purpose: a failure here leaves every other
test already run."""
import pytest
import torch

import cases
from parity import assert_grad

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _forward(lib, _lib, q, k, v, meta, window):
    B, H, L, D = q.shape
    y = torch.empty_like(q)
    saved = torch.empty(lib.lz_swa_saved_bytes(B, H, L, D), device=DEV, dtype=torch.uint8)
    rc = lib.lz_swa_fwd(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), None, None, _lib.ptr(meta),
                        meta.numel(), window, _lib.ptr(y), _lib.ptr(saved), saved.numel(), B, H,
                        L, D, _lib.stream_of(q))
    _lib.check(rc, "swa forward")
    return saved


def _grads(q):
    return [torch.full(q.shape, float("nan"), device=DEV) for _ in range(3)]


def test_swa_backward_without_allocation_matches_workspace_version(built_lib):
    from lizard_cuda import _lib
    lib = _lib.load()
    inp = cases.swa_case(150, dim=64)
    q, k, v = (inp[n].to(DEV).contiguous() for n in ("q", "k", "v"))
    meta = inp["meta"].to(DEV).contiguous()
    dy = inp["dy"].to(DEV).bfloat16().contiguous()
    B, H, L, D = q.shape
    window, nm = 32, meta.numel()
    saved = _forward(lib, _lib, q, k, v, meta, window)

    # the existing entry point with a caller-owned workspace
    ws = torch.empty(lib.lz_swa_bwd_workspace_bytes(B, H, L, D, nm), device=DEV,
                     dtype=torch.uint8)
    dq, dk, dv = _grads(q)
    dmeta = torch.zeros(nm, device=DEV)
    rc = lib.lz_swa_bwd(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), None, None, _lib.ptr(meta), nm,
                        window, _lib.ptr(saved), saved.numel(), _lib.ptr(dy), _lib.ptr(dq),
                        _lib.ptr(dk), _lib.ptr(dv), _lib.LZ_DTYPE_F32, _lib.ptr(dmeta),
                        _lib.ptr(ws), ws.numel(), B, H, L, D, _lib.stream_of(q))
    _lib.check(rc, "swa backward")
    ref = (dq, dk, dv, dmeta)

    # two calls in a row of the no-allocation entry point
    for call in range(2):
        nq, nk, nv = _grads(q)
        nmeta = torch.full((nm,), float("nan"), device=DEV)
        rc = lib.lz_swa_bwd_noalloc(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), None, None,
                                    _lib.ptr(meta), nm, window, _lib.ptr(saved), saved.numel(),
                                    _lib.ptr(dy), _lib.ptr(nq), _lib.ptr(nk), _lib.ptr(nv),
                                    _lib.LZ_DTYPE_F32, _lib.ptr(nmeta), B, H, L, D,
                                    _lib.stream_of(q))
        _lib.check(rc, "swa backward without allocation")
        torch.cuda.synchronize()
        for got, want, name in zip((nq, nk, nv, nmeta), ref, ("dq", "dk", "dv", "dmeta")):
            assert torch.isfinite(got).all(), f"call {call} {name} not fully written"
            assert_grad(got, want, f"call {call} {name}")


def test_swa_backward_without_allocation_rejects_oversized_problems(built_lib):
    from lizard_cuda import _lib
    lib = _lib.load()
    # B*H*L = 2^21 rows need 8 MiB of delta: above the fixed scratch
    rc = lib.lz_swa_bwd_noalloc(None, None, None, None, None, None, 0, 64, None, 0, None, None,
                                None, None, 0, None, 64, 32, 1024, 64, None)
    assert rc == 2
    assert b"4 MiB" in lib.lz_last_error_string()
