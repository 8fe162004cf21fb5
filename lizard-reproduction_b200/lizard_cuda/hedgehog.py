"""hedgehog(x, weight): the Hedgehog feature map [softmax(x W^T), softmax(-x W^T)]
of the reference (src/lizard_attention.py:9-11), fused into one kernel.

x [..., Dh] (fp32 or bf16; other float dtypes are computed as fp32), weight
[Fd, Dh] with Dh, Fd <= 128. A 4-D x [B, H, L, Dh] with a contiguous last
dimension is read in place at its strides (a projection output [B, L, H * Dh]
viewed as heads); other layouts are made contiguous first. Returns the features [..., 2 Fd] in bf16, the
dtype the GLA kernels consume (the reference returns x's dtype and GLA then
casts to bf16, src/kernels/gla.py:217). Gradients flow to x (in x's dtype) and
to weight (in weight's dtype).
"""
import torch

from . import _lib


class _Hedgehog(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight):
        _lib.require_cuda(x, weight)
        if weight.dim() != 2 or x.shape[-1] != weight.shape[1]:
            raise ValueError(f"weight must be [Fd, Dh] with Dh = x.shape[-1], got "
                             f"{tuple(weight.shape)} for x {tuple(x.shape)}")
        lib = _lib.load()
        Fd, Dh = weight.shape
        ctx.dtypes = (x.dtype, weight.dtype)
        xc = x if x.dtype in (torch.float32, torch.bfloat16) else x.float()
        strided = xc.dim() == 4 and xc.stride(-1) == 1 and not xc.is_contiguous()
        if not strided:
            xc = xc.contiguous()
        w32 = weight.float().contiguous()
        R = xc.numel() // Dh
        f = torch.empty(*x.shape[:-1], 2 * Fd, device=x.device, dtype=torch.bfloat16)
        xdt = _lib.LZ_DTYPE_BF16 if xc.dtype == torch.bfloat16 else _lib.LZ_DTYPE_F32
        with _lib.on_device(x.device):
            if strided:
                B, H, L, _ = xc.shape
                rc = lib.lz_hedgehog_fwd_strided(_lib.ptr(xc), xdt, xc.stride(0), xc.stride(1),
                                                 xc.stride(2), B, H, L, _lib.ptr(w32),
                                                 _lib.ptr(f), Dh, Fd, _lib.stream_of(x))
            else:
                rc = lib.lz_hedgehog_fwd(_lib.ptr(xc), xdt, _lib.ptr(w32), _lib.ptr(f), R, Dh,
                                         Fd, _lib.stream_of(x))
        _lib.check(rc, "hedgehog forward")
        ctx.save_for_backward(xc, w32)
        ctx.xdt = xdt
        ctx.strided = strided
        return f

    @staticmethod
    def backward(ctx, df):
        xc, w32 = ctx.saved_tensors
        lib = _lib.load()
        Fd, Dh = w32.shape
        R = xc.numel() // Dh
        dfc = df.contiguous() if df.dtype in (torch.float32, torch.bfloat16) else df.float().contiguous()
        gdt = _lib.LZ_DTYPE_BF16 if dfc.dtype == torch.bfloat16 else _lib.LZ_DTYPE_F32
        dx = torch.empty(xc.shape, device=xc.device, dtype=torch.float32)
        dw = torch.empty(Fd, Dh, device=xc.device, dtype=torch.float32)
        nws = lib.lz_hedgehog_bwd_workspace_bytes(R, Dh, Fd)
        ws = torch.empty(nws, device=xc.device, dtype=torch.uint8)
        with _lib.on_device(xc.device):
            if ctx.strided:
                B, H, L, _ = xc.shape
                rc = lib.lz_hedgehog_bwd_strided(_lib.ptr(xc), ctx.xdt, xc.stride(0),
                                                 xc.stride(1), xc.stride(2), B, H, L,
                                                 _lib.ptr(w32), _lib.ptr(dfc), gdt, _lib.ptr(dx),
                                                 _lib.ptr(dw), _lib.ptr(ws), nws, Dh, Fd,
                                                 _lib.stream_of(xc))
            else:
                rc = lib.lz_hedgehog_bwd(_lib.ptr(xc), ctx.xdt, _lib.ptr(w32), _lib.ptr(dfc),
                                         gdt, _lib.ptr(dx), _lib.ptr(dw), _lib.ptr(ws), nws, R,
                                         Dh, Fd, _lib.stream_of(xc))
        _lib.check(rc, "hedgehog backward")
        return dx.to(ctx.dtypes[0]), dw.to(ctx.dtypes[1])


def hedgehog(x, weight):
    """[softmax(x W^T), softmax(-x W^T)] as bf16 features (see the module docstring)."""
    return _Hedgehog.apply(x, weight)
