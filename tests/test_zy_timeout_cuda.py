"""The bounded-wait protocol, exercised without a GPU fault.

Every wait on a barrier inside this library's kernels gives up after about
2 s, records where in a per-device flag and lets the kernel return instead of
hanging. Here the SWA decode kernel is told (a test switch) to arm its
ring-copy barrier without issuing the copy: nothing ever completes the
barrier, so the wait must run out. The test checks that the call returns, the
flag names the wait's site, the context still works, and that after clearing
the flag the next decode step is correct again.

It holds no tensor memory, issues no copy that could still be in flight, and
touches no bad address. The file is collected after the other GPU tests, which
check that no wait ever timed out."""
import pytest
import torch

import lizard_oracle as orc
from parity import assert_output

pytestmark = pytest.mark.gpu
DEV = "cuda"
SITE_RING_COPY = 0x80000000 | 90  # the ring-copy wait of the SWA decode kernel


def _rep(x, grp):
    return x.repeat_interleave(grp, dim=1) if grp > 1 else x


def test_decode_wait_times_out_reports_its_site_and_recovers(built_lib):
    from lizard_cuda import _lib
    from lizard_cuda.decode import swa_decode, swa_ring
    lib = _lib.load()
    B, H, Hkv, W, D, L0 = 2, 4, 2, 16, 64, 24
    g = torch.Generator(device=DEV).manual_seed(17)
    q = torch.randn(B, H, L0 + 1, D, generator=g, device=DEV)
    k = torch.randn(B, Hkv, L0 + 1, D, generator=g, device=DEV)
    v = torch.randn(B, Hkv, L0 + 1, D, generator=g, device=DEV)
    meta = torch.randn(4, generator=g, device=DEV)
    cos, sin = (t.to(DEV).expand(B, L0 + 1, D) for t in orc.rotary_tables(L0 + 1, D, 5e5))
    k_ring, v_ring = swa_ring(k[:, :, :L0], v[:, :, :L0], cos[:, :L0], sin[:, :L0], W)
    kr0, vr0 = k_ring.clone(), v_ring.clone()
    pos = torch.full((B,), L0, dtype=torch.int32, device=DEV)
    torch.cuda.synchronize()
    assert _lib.device_timeout_flag() == 0

    _lib.check(lib.lz_test_withhold_decode_ring_copy(1), "withhold switch")
    try:
        swa_decode(q[:, :, L0], k[:, :, L0], v[:, :, L0], cos[:, L0], sin[:, L0], meta,
                   k_ring, v_ring, pos)
        torch.cuda.synchronize()  # the call ends: the wait gave up instead of hanging
    finally:
        _lib.check(lib.lz_test_withhold_decode_ring_copy(0), "withhold switch")
    assert _lib.device_timeout_flag() == SITE_RING_COPY
    # the CTAs left before writing: the rings are untouched
    assert torch.equal(k_ring, kr0) and torch.equal(v_ring, vr0)

    _lib.clear_device_timeout_flag()
    assert _lib.device_timeout_flag() == 0
    y = swa_decode(q[:, :, L0], k[:, :, L0], v[:, :, L0], cos[:, L0], sin[:, L0], meta,
                   k_ring, v_ring, pos)
    torch.cuda.synchronize()
    assert _lib.device_timeout_flag() == 0
    c, s = cos.cpu().double(), sin.cpu().double()
    qr, kr = orc.rope(q.double().cpu(), c, s), orc.rope(k.double().cpu(), c, s)
    ref = orc.awa(qr, _rep(kr, H // Hkv), _rep(v.double().cpu(), H // Hkv),
                  meta.double().cpu(), W)[:, :, L0]
    assert_output(y, ref.float(), "decode step after the timeout")
