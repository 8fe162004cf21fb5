"""gla(fq, fk, v, log_gamma, chunk=64): chunked gated linear attention.

Drop-in for the reference's kernels.gla (src/kernels/gla.py:259-263): same
arguments, same output dtype (bf16), gradients returned in each input's dtype
(gla.py:216, 255) and a gradient for log_gamma, which may be [B, L] (one gate
per token, shared by the heads) or [B, H, L] (one gate per head).

fk and v may carry fewer heads than fq (grouped-query attention, H % Hkv == 0):
query head h then reads key/value head h // (H // Hkv), which is what the
reference's caller computes with repeat_interleave before the feature map
(src/lizard_attention.py:73-85), and dfk, dv come back with Hkv heads, summed
over each group.
"""
import torch

from . import _lib

CHUNK = 64


def _shapes(fq, fk, v, log_gamma):
    if (fq.dim() != 4 or fk.dim() != 4 or fk.shape[0] != fq.shape[0]
            or fk.shape[2:] != fq.shape[2:] or fk.shape[1] < 1 or fq.shape[1] % fk.shape[1]):
        raise ValueError(f"fq must be [B, H, L, F] and fk [B, Hkv, L, F] with Hkv dividing H, "
                         f"got {tuple(fq.shape)} and {tuple(fk.shape)}")
    B, H, L, F = fq.shape
    Hkv = fk.shape[1]
    if v.dim() != 4 or tuple(v.shape[:3]) != (B, Hkv, L):
        raise ValueError(f"v must be [B, Hkv, L, D] matching fk, got {tuple(v.shape)}")
    if tuple(log_gamma.shape) == (B, L):
        per_head = 0
    elif tuple(log_gamma.shape) == (B, H, L):
        per_head = 1
    else:
        raise ValueError(f"log_gamma must be [B, L] or [B, H, L], got {tuple(log_gamma.shape)}")
    return B, H, Hkv, L, F, v.shape[-1], per_head


class _GLA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, fq, fk, v, log_gamma, chunk):
        _lib.require_cuda(fq, fk, v, log_gamma)
        B, H, Hkv, L, F, D, per_head = _shapes(fq, fk, v, log_gamma)
        lib = _lib.load()
        ctx.dtypes = (fq.dtype, fk.dtype, v.dtype, log_gamma.dtype)
        fq, fk, v = (t.to(torch.bfloat16).contiguous() for t in (fq, fk, v))
        lg = log_gamma.float().contiguous()
        save = any(ctx.needs_input_grad[:4])
        y = torch.empty(B, H, L, D, device=v.device, dtype=torch.bfloat16)
        saved = None
        if save:
            nbytes = _lib.size_query("lz_gla_saved_bytes", B, H, L, F, D, chunk)
            saved = torch.empty(nbytes, device=v.device, dtype=torch.uint8)
        wbytes = _lib.size_query("lz_gla_fwd_gqa_workspace_bytes", B, H, Hkv, L, F, D, chunk,
                                 per_head, int(save))
        ws = torch.empty(wbytes, device=v.device, dtype=torch.uint8) if wbytes else None
        with _lib.on_device(v.device):
            rc = lib.lz_gla_fwd_gqa(_lib.ptr(fq), _lib.ptr(fk), _lib.ptr(v), _lib.ptr(lg),
                                    per_head, _lib.ptr(y), _lib.ptr(saved),
                                    0 if saved is None else saved.numel(), _lib.ptr(ws), wbytes,
                                    B, H, Hkv, L, F, D, chunk, _lib.stream_of(v))
        _lib.check(rc, "gla forward")
        if save:
            ctx.save_for_backward(fq, fk, v, lg, saved)
        ctx.dims = (B, H, Hkv, L, F, D, per_head, chunk)
        return y

    @staticmethod
    def backward(ctx, dy):
        fq, fk, v, lg, saved = ctx.saved_tensors
        B, H, Hkv, L, F, D, per_head, chunk = ctx.dims
        lib = _lib.load()
        dy = dy.to(torch.bfloat16).contiguous()
        all_bf16 = all(d == torch.bfloat16 for d in ctx.dtypes[:3])
        gdt = _lib.LZ_DTYPE_BF16 if all_bf16 else _lib.LZ_DTYPE_F32
        gtorch = torch.bfloat16 if all_bf16 else torch.float32
        dfq = torch.empty(B, H, L, F, device=fq.device, dtype=gtorch)
        dfk = torch.empty(B, Hkv, L, F, device=fq.device, dtype=gtorch)
        dv = torch.empty(B, Hkv, L, D, device=fq.device, dtype=gtorch)
        dlg = torch.empty_like(lg)
        nws = _lib.size_query("lz_gla_bwd_gqa_workspace_bytes", B, H, Hkv, L, F, D, chunk)
        ws = torch.empty(nws, device=fq.device, dtype=torch.uint8)
        with _lib.on_device(fq.device):
            rc = lib.lz_gla_bwd_gqa(_lib.ptr(fq), _lib.ptr(fk), _lib.ptr(v), _lib.ptr(lg),
                                    per_head, _lib.ptr(saved), saved.numel(), _lib.ptr(dy),
                                    _lib.ptr(dfq), _lib.ptr(dfk), _lib.ptr(dv), gdt,
                                    _lib.ptr(dlg), _lib.ptr(ws), ws.numel(), B, H, Hkv, L, F, D,
                                    chunk, _lib.stream_of(fq))
        _lib.check(rc, "gla backward")
        grads = (dfq, dfk, dv, dlg)
        dfq, dfk, dv, dlg = (g.to(d) for g, d in zip(grads, ctx.dtypes))
        return dfq, dfk, dv, dlg, None


def gla(fq, fk, v, log_gamma, chunk=CHUNK):
    """Gated linear attention y_i = sum_{t<=i} w_it v_t / max(sum_t w_it, FLT_MIN),
    w_it = (fq_i . fk_t) exp(G_i - G_t), G = cumsum(log_gamma).

    fq [B, H, L, F], fk [B, Hkv, L, F] non-negative features (Hkv dividing H);
    v [B, Hkv, L, D]; log_gamma <= 0,
    [B, L] or [B, H, L]; any float dtypes. Returns bf16 [B, H, L, D].
    `chunk` is the reference's chunk-length argument; the kernels always use
    64-token chunks and any chunk >= 1 gives the same result within bf16
    tolerance.
    """
    if int(chunk) < 1:
        raise ValueError("chunk must be >= 1")
    return _GLA.apply(fq, fk, v, log_gamma, int(chunk))
