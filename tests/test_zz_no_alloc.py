"""lz_swa_bwd_noalloc, the SWA backward for callers that cannot allocate
(a host that hands a plugin only its inputs and outputs, with no way to
request a workspace). It must give the same gradients as lz_swa_bwd with a
caller-owned workspace, on consecutive calls that share its fixed scratch.

Both entry points run the same deterministic kernels on the same inputs, so
the gradients must be bit-identical. Between the two checked calls a call of
another shape and sink count leaves different data in the shared scratch, so
a kernel that read a delta or a sink partial before writing it would show.

This file is collected last on purpose: a failure here leaves every other
test already run."""
import pytest
import torch

import cases

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(length, dim, sinks, seed):
    inp = cases.swa_case(length, dim=dim, sinks=sinks, seed=seed)
    q, k, v = (inp[n].to(DEV).contiguous() for n in ("q", "k", "v"))
    meta = inp["meta"].to(DEV).contiguous()
    dy = inp["dy"].to(DEV).bfloat16().contiguous()
    return q, k, v, meta, dy


def _forward(lib, _lib, q, k, v, meta, window):
    B, H, L, D = q.shape
    y = torch.empty_like(q)
    saved = torch.empty(lib.lz_swa_saved_bytes(B, H, L, D), device=DEV, dtype=torch.uint8)
    rc = lib.lz_swa_fwd(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), None, None, _lib.ptr(meta),
                        meta.numel(), window, _lib.ptr(y), _lib.ptr(saved), saved.numel(), B, H,
                        L, D, _lib.stream_of(q))
    _lib.check(rc, "swa forward")
    return saved


def _nan_grads(q, nm):
    return [torch.full(q.shape, float("nan"), device=DEV) for _ in range(3)] + \
        [torch.full((nm,), float("nan"), device=DEV)]


def _noalloc(lib, _lib, q, k, v, meta, window, saved, dy):
    B, H, L, D = q.shape
    nm = meta.numel()
    out = _nan_grads(q, nm)
    rc = lib.lz_swa_bwd_noalloc(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), None, None,
                                _lib.ptr(meta), nm, window, _lib.ptr(saved), saved.numel(),
                                _lib.ptr(dy), *(_lib.ptr(t) for t in out[:3]),
                                _lib.LZ_DTYPE_F32, _lib.ptr(out[3]), B, H, L, D,
                                _lib.stream_of(q))
    _lib.check(rc, "swa backward without allocation")
    return out


@pytest.mark.parametrize("length,dim,window", [
    (150, 64, 32),    # head dim 64, window <= 64: the tensor-core kernels
    (150, 32, 128),   # other head dims and windows: the 64-row kernels
])
def test_swa_backward_without_allocation_matches_workspace_version(built_lib, length, dim,
                                                                  window):
    from lizard_cuda import _lib
    lib = _lib.load()
    q, k, v, meta, dy = _inputs(length, dim, 4, seed=0)
    B, H, L, D = q.shape
    nm = meta.numel()
    saved = _forward(lib, _lib, q, k, v, meta, window)

    # the existing entry point with a caller-owned workspace
    ws = torch.empty(lib.lz_swa_bwd_workspace_bytes(B, H, L, D, nm), device=DEV,
                     dtype=torch.uint8)
    ref = _nan_grads(q, nm)
    rc = lib.lz_swa_bwd(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), None, None, _lib.ptr(meta), nm,
                        window, _lib.ptr(saved), saved.numel(), _lib.ptr(dy),
                        *(_lib.ptr(t) for t in ref[:3]), _lib.LZ_DTYPE_F32, _lib.ptr(ref[3]),
                        _lib.ptr(ws), ws.numel(), B, H, L, D, _lib.stream_of(q))
    _lib.check(rc, "swa backward")

    # another shape and sink count in between fills the shared scratch with other data
    q2, k2, v2, meta2, dy2 = _inputs(77, 64, 2, seed=5)
    saved2 = _forward(lib, _lib, q2, k2, v2, meta2, 16)

    for call in range(2):
        got = _noalloc(lib, _lib, q, k, v, meta, window, saved, dy)
        torch.cuda.synchronize()
        for g, want, name in zip(got, ref, ("dq", "dk", "dv", "dmeta")):
            assert torch.isfinite(g).all(), f"call {call} {name} not fully written"
            assert torch.equal(g, want), f"call {call} {name} differs from lz_swa_bwd"
        if call == 0:
            _noalloc(lib, _lib, q2, k2, v2, meta2, 16, saved2, dy2)


def test_swa_backward_without_allocation_rejects_oversized_problems(built_lib):
    from lizard_cuda import _lib
    lib = _lib.load()
    # B*H*L = 2^21 rows need 8 MiB of delta: above the fixed scratch
    rc = lib.lz_swa_bwd_noalloc(None, None, None, None, None, None, 0, 64, None, 0, None, None,
                                None, None, 0, None, 64, 32, 1024, 64, None)
    assert rc == 2
    assert b"4 MiB" in lib.lz_last_error_string()
