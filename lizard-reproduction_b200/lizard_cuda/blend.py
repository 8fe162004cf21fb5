"""blend(y_gla, y_swa, alpha, dtype): the Lizard layer's output blend, fused.

The reference's caller (src/lizard_attention.py:92-97) computes
    y = gla(...).to(c) + alpha_blend.to(c) * swa(...).to(c)      (c: compute dtype)
    o_proj(y.to(x.dtype).transpose(1, 2).flatten(2))
This does the blend, the cast to `dtype` and the transpose in one kernel and
returns [B, L, H * D] ready for the output projection; the values are
identical to the torch ops (one rounding per product and sum). The backward
returns bf16 gradients for both branches (what their backward kernels take)
and the gradient of alpha.
"""
import torch

from . import _lib

_DT = {torch.float32: _lib.LZ_DTYPE_F32, torch.bfloat16: _lib.LZ_DTYPE_BF16}


class _Blend(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y_gla, y_swa, alpha, dtype):
        _lib.require_cuda(y_gla, y_swa, alpha)
        if y_gla.shape != y_swa.shape or y_gla.dim() != 4:
            raise ValueError(f"branch outputs must be [B, H, L, D] of one shape, got "
                             f"{tuple(y_gla.shape)}, {tuple(y_swa.shape)}")
        if dtype not in _DT:
            raise ValueError(f"output dtype must be float32 or bfloat16, got {dtype}")
        B, H, L, D = y_gla.shape
        yg = y_gla.to(torch.bfloat16).contiguous()
        ys = y_swa.to(torch.bfloat16).contiguous()
        a32 = alpha.float().reshape(1).contiguous()
        out = torch.empty(B, L, H * D, device=yg.device, dtype=dtype)
        lib = _lib.load()
        rc = lib.lz_blend_fwd(_lib.ptr(yg), _lib.ptr(ys), _lib.ptr(a32), _lib.ptr(out), _DT[dtype],
                              B, H, L, D, _lib.stream_of(yg))
        _lib.check(rc, "blend forward")
        ctx.save_for_backward(ys, a32)
        ctx.in_dtypes = (y_gla.dtype, y_swa.dtype, alpha.dtype)
        ctx.alpha_shape = alpha.shape
        return out

    @staticmethod
    def backward(ctx, dout):
        ys, a32 = ctx.saved_tensors
        B, H, L, D = ys.shape
        g = dout if dout.dtype in _DT else dout.float()
        g = g.contiguous()
        lib = _lib.load()
        dyg = torch.empty(B, H, L, D, device=ys.device, dtype=torch.bfloat16)
        dys = torch.empty_like(dyg)
        da = torch.empty(1, device=ys.device, dtype=torch.float32)
        ws = torch.empty(lib.lz_blend_bwd_workspace_bytes(B, H, L, D), device=ys.device,
                         dtype=torch.uint8)
        rc = lib.lz_blend_bwd(_lib.ptr(g), _DT[g.dtype], _lib.ptr(ys), _lib.ptr(a32),
                              _lib.ptr(dyg), _lib.ptr(dys), _lib.ptr(da), _lib.ptr(ws),
                              ws.numel(), B, H, L, D, _lib.stream_of(ys))
        _lib.check(rc, "blend backward")
        gd, sd, ad = ctx.in_dtypes
        return dyg.to(gd), dys.to(sd), da.reshape(ctx.alpha_shape).to(ad), None


def blend(y_gla, y_swa, alpha, dtype):
    """to(dtype)(float(y_gla) + alpha * float(y_swa)) transposed to [B, L, H * D]."""
    return _Blend.apply(y_gla, y_swa, alpha, dtype)
