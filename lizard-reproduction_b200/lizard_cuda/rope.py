"""swa_rope(q, k, v, cos, sin, meta, window): sliding-window attention over
queries and keys that are rotated on the way in.

The reference's caller rotates q and k with torch ops in the layer's compute
dtype (src/lizard_attention.py:87-88, Llama's rotate-half form) and hands the
rotated copies to kernels.swa (src/lizard_attention.py:93). Here one kernel
reads the unrotated q and k (any batch / head / token strides, so the
projection output [B, L, H * Dh] is read in place as [B, H, L, Dh]), rotates
them in fp32 and writes the bf16 value and bf16 residual pair the SWA kernels
take (about 16 mantissa bits of each rotated element, as swa() keeps for fp32
inputs). k and v may carry fewer heads than q (GQA). The forward is one
kernel (lz_swa_rope_fwd: TMA tiles of q, k, v, rotation inside the CTA); for
head dims or strides its TMA tiles cannot take it rotates first (lz_rope_split)
and calls the SWA forward, with the same results. The backward runs the SWA
backward and then the transpose rotation, dx = R^T dr, in one more pass.

    swa_rope(q, k, v, cos, sin, meta, window)
        == swa(rope(q), rope(k), v, meta, window)   within bf16 rounding

cos and sin take no gradient (they are the rotary tables).
"""
import torch

from . import _lib
from .swa import _check_blocks, FWD_BLOCKS, BWD_BLOCKS

_DT = {torch.float32: _lib.LZ_DTYPE_F32, torch.bfloat16: _lib.LZ_DTYPE_BF16}


def _as_input(x):
    """x with a supported dtype and a contiguous last dimension (no copy when it has both)."""
    if x.dtype not in _DT:
        x = x.float()
    if x.stride(-1) != 1:
        x = x.contiguous()
    return x


def _tables(cos, sin, B, L, Dh):
    """cos / sin as ([B or 1, L, Dh] or [L, Dh]) tensors with their batch and token strides."""
    if cos.shape != sin.shape:
        raise ValueError(f"cos and sin differ in shape: {tuple(cos.shape)}, {tuple(sin.shape)}")
    if cos.dtype != sin.dtype or cos.dtype not in _DT:
        cos, sin = cos.float(), sin.float()
    if cos.stride(-1) != 1 or sin.stride() != cos.stride():
        cos, sin = cos.contiguous(), sin.contiguous()
    if cos.dim() == 2 and tuple(cos.shape) == (L, Dh):
        return cos, sin, 0, cos.stride(0)
    if cos.dim() == 3 and tuple(cos.shape[1:]) == (L, Dh) and cos.shape[0] in (1, B):
        return cos, sin, (cos.stride(0) if cos.shape[0] == B and B > 1 else 0), cos.stride(1)
    raise ValueError(f"cos / sin must be [B, L, Dh], [1, L, Dh] or [L, Dh] with L = {L}, "
                     f"Dh = {Dh}, got {tuple(cos.shape)}")


def rope_split(x, cos, sin, csb, csl):
    """(bf16(r), bf16(r - bf16(r))) for r = x * cos + rotate_half(x) * sin, contiguous
    [B, Hx, L, Dh]; x [B, Hx, L, Dh] at any strides with a contiguous last dim."""
    B, Hx, L, Dh = x.shape
    hi = torch.empty(B, Hx, L, Dh, device=x.device, dtype=torch.bfloat16)
    lo = torch.empty_like(hi)
    lib = _lib.load()
    rc = lib.lz_rope_split(_lib.ptr(x), _DT[x.dtype], x.stride(0), x.stride(1), x.stride(2),
                           _lib.ptr(cos), _lib.ptr(sin), _DT[cos.dtype], csb, csl,
                           _lib.ptr(hi), _lib.ptr(lo), B, Hx, L, Dh, _lib.stream_of(x))
    _lib.check(rc, "rope split")
    return hi, lo


def rope_grad(dr, cos, sin, csb, csl, dtype):
    """R^T dr for fp32 contiguous dr [B, Hx, L, Dh], in `dtype` (fp32 or bf16)."""
    B, Hx, L, Dh = dr.shape
    out_dt = dtype if dtype in _DT else torch.float32
    dx = torch.empty(B, Hx, L, Dh, device=dr.device, dtype=out_dt)
    lib = _lib.load()
    rc = lib.lz_rope_bwd(_lib.ptr(dr), _lib.ptr(cos), _lib.ptr(sin), _DT[cos.dtype], csb, csl,
                         _lib.ptr(dx), _DT[out_dt], B, Hx, L, Dh, _lib.stream_of(dr))
    _lib.check(rc, "rope backward")
    return dx.to(dtype)


def _fused_forward(q, k, v, cos, sin, csb, csl, meta32, window, y, saved, rot):
    """One kernel: TMA tiles of the unrotated q, k, v, rotation and split in the
    CTA, the SWA forward. rot = (q_hi, q_lo, k_hi, k_lo) to fill for the
    backward, or None. Returns False (nothing launched) when the head dim or the
    strides are outside the kernel's TMA tiles."""
    B, H, L, D = q.shape
    Hkv = k.shape[1]
    xdt = q.dtype if q.dtype in _DT else torch.float32
    q, k, v = (_as_input(t.to(xdt)) for t in (q, k, v))
    lib = _lib.load()
    n_meta = meta32.numel()
    rp = [_lib.ptr(t) for t in rot] if rot is not None else [None] * 4
    rc = lib.lz_swa_rope_fwd(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _DT[xdt], q.stride(0),
                             q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
                             v.stride(0), v.stride(1), v.stride(2), _lib.ptr(cos), _lib.ptr(sin),
                             _DT[cos.dtype], csb, csl, _lib.ptr(meta32) if n_meta else None,
                             n_meta, window, _lib.ptr(y), _lib.ptr(saved),
                             0 if saved is None else saved.numel(), *rp, B, H, Hkv, L, D,
                             _lib.stream_of(q))
    if rc == _lib.LZ_ERR_UNSUPPORTED:
        return False
    _lib.check(rc, "swa_rope forward")
    return True


def _two_pass_forward(q, k, v, cos, sin, csb, csl, meta32, window, y, saved):
    """lz_rope_split on q and k, then lz_swa_fwd_gqa. Returns (q_hi, q_lo, k_hi, k_lo)."""
    B, H, L, D = q.shape
    Hkv = k.shape[1]
    q_hi, q_lo = rope_split(_as_input(q), cos, sin, csb, csl)
    k_hi, k_lo = rope_split(_as_input(k), cos, sin, csb, csl)
    v16 = v.to(torch.bfloat16).contiguous()
    lib = _lib.load()
    n_meta = meta32.numel()
    rc = lib.lz_swa_fwd_gqa(_lib.ptr(q_hi), _lib.ptr(k_hi), _lib.ptr(v16), _lib.ptr(q_lo),
                            _lib.ptr(k_lo), _lib.ptr(meta32) if n_meta else None, n_meta,
                            window, _lib.ptr(y), _lib.ptr(saved),
                            0 if saved is None else saved.numel(), B, H, Hkv, L, D,
                            _lib.stream_of(q))
    _lib.check(rc, "swa_rope forward")
    return q_hi, q_lo, k_hi, k_lo


class _SWARope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, cos, sin, meta, window):
        _lib.require_cuda(q, k, v, meta, cos, sin)
        if (q.dim() != 4 or k.dim() != 4 or v.shape != k.shape or k.shape[0] != q.shape[0]
                or k.shape[2:] != q.shape[2:] or k.shape[1] < 1 or q.shape[1] % k.shape[1]):
            raise ValueError("q must be [B, H, L, D] and k, v [B, Hkv, L, D] with Hkv "
                             f"dividing H, got {tuple(q.shape)}, {tuple(k.shape)}, "
                             f"{tuple(v.shape)}")
        if meta.dim() != 1:
            raise ValueError(f"meta must be 1-D, got {tuple(meta.shape)}")
        B, H, L, D = q.shape
        Hkv = k.shape[1]
        if D % 2:
            raise ValueError(f"the rotated head dim must be even, got {D}")
        ctx.dtypes = (q.dtype, k.dtype, v.dtype, meta.dtype)
        cos, sin, csb, csl = _tables(cos, sin, B, L, D)
        meta32 = meta.float().contiguous()
        lib = _lib.load()
        y = torch.empty(B, H, L, D, device=q.device, dtype=torch.bfloat16)
        save = any(ctx.needs_input_grad[:3]) or ctx.needs_input_grad[5]
        saved = rot = None
        if save:
            saved = torch.empty(_lib.size_query("lz_swa_saved_bytes", B, H, L, D), device=q.device,
                                dtype=torch.uint8)
            rot = tuple(torch.empty(B, n, L, D, device=q.device, dtype=torch.bfloat16)
                        for n in (H, H, Hkv, Hkv))
        with _lib.on_device(q.device):
            if not _fused_forward(q, k, v, cos, sin, csb, csl, meta32, int(window), y, saved,
                                  rot):
                rot = _two_pass_forward(q, k, v, cos, sin, csb, csl, meta32, int(window), y,
                                        saved)
        if save:
            v16 = v.to(torch.bfloat16).contiguous()
            ctx.save_for_backward(*rot, v16, meta32, saved, cos, sin)
            ctx.tables = (csb, csl)
        ctx.window = int(window)
        return y

    @staticmethod
    def backward(ctx, dy):
        q_hi, q_lo, k_hi, k_lo, v16, meta32, saved, cos, sin = ctx.saved_tensors
        csb, csl = ctx.tables
        B, H, L, D = q_hi.shape
        Hkv = k_hi.shape[1]
        n_meta = meta32.numel()
        lib = _lib.load()
        dy = dy.to(torch.bfloat16).contiguous()
        dqr = torch.empty(B, H, L, D, device=dy.device, dtype=torch.float32)
        dkr = torch.empty(B, Hkv, L, D, device=dy.device, dtype=torch.float32)
        dv = torch.empty_like(dkr)
        dmeta = torch.empty(n_meta, device=dy.device, dtype=torch.float32)
        nws = _lib.size_query("lz_swa_bwd_workspace_bytes", B, H, L, D, n_meta)
        ws = torch.empty(nws, device=dy.device, dtype=torch.uint8)
        with _lib.on_device(dy.device):
            rc = lib.lz_swa_bwd_gqa(_lib.ptr(q_hi), _lib.ptr(k_hi), _lib.ptr(v16),
                                    _lib.ptr(q_lo), _lib.ptr(k_lo),
                                    _lib.ptr(meta32) if n_meta else None, n_meta, ctx.window,
                                    _lib.ptr(saved), saved.numel(), _lib.ptr(dy),
                                    _lib.ptr(dqr), _lib.ptr(dkr), _lib.ptr(dv),
                                    _lib.LZ_DTYPE_F32, _lib.ptr(dmeta) if n_meta else None,
                                    _lib.ptr(ws), ws.numel(), B, H, Hkv, L, D,
                                    _lib.stream_of(dy))
            _lib.check(rc, "swa_rope backward")
            qdt, kdt, vdt, mdt = ctx.dtypes
            dq = rope_grad(dqr, cos, sin, csb, csl, qdt) if ctx.needs_input_grad[0] else None
            dk = rope_grad(dkr, cos, sin, csb, csl, kdt) if ctx.needs_input_grad[1] else None
        return dq, dk, dv.to(vdt), None, None, dmeta.to(mdt), None


def swa_rope(q, k, v, cos, sin, meta, window, fwd_blocks=FWD_BLOCKS, bwd_blocks=BWD_BLOCKS):
    """swa(rope(q), rope(k), v, meta, window) with the rotation fused into one
    pass per operand. q [B, H, L, D], k, v [B, Hkv, L, D] (Hkv dividing H; q and
    k may be strided views such as a projection output transposed to heads);
    cos, sin [B, L, D], [1, L, D] or [L, D]; D even. Returns bf16 [B, H, L, D];
    gradients flow to q, k, v and meta in their dtypes."""
    _check_blocks(fwd_blocks, "fwd_blocks")
    _check_blocks(bwd_blocks, "bwd_blocks")
    if int(window) < 1:
        raise ValueError("window must be >= 1")
    return _SWARope.apply(q, k, v, cos, sin, meta, int(window))
