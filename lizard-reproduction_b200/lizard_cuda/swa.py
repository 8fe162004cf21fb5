"""swa(q, k, v, meta, window, fwd_blocks, bwd_blocks): sliding-window softmax
attention with sink logits.

Drop-in for the reference's kernels.swa (src/kernels/swa.py:182-183): same
arguments and defaults, bf16 output, gradients in each input's dtype
(swa.py:139, 178). `meta` may be empty (no sinks). The block tuples are
accepted for signature compatibility; the kernels use 64 x 64 tiles.

k and v may carry fewer heads than q (grouped-query attention, H % Hkv == 0):
query head h then attends with key/value head h // (H // Hkv), as if the
caller had repeat_interleaved k and v (src/lizard_attention.py:73-76), and
dk, dv come back with Hkv heads, summed over each group.

When q or k is not bf16 (the Lizard layer passes fp32), each is sent as a bf16
value plus its bf16 residual, and the kernels form the logits from both, so a
large logit keeps about 16 mantissa bits instead of 8.
"""
import torch

from . import _lib

FWD_BLOCKS = (64, 64)
BWD_BLOCKS = (64, 64)


class _SWA(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, meta, window, fwd_blocks, bwd_blocks):
        _lib.require_cuda(q, k, v, meta)
        if (q.dim() != 4 or k.dim() != 4 or v.shape != k.shape
                or k.shape[0] != q.shape[0] or k.shape[2:] != q.shape[2:]
                or k.shape[1] < 1 or q.shape[1] % k.shape[1]):
            raise ValueError("q must be [B, H, L, D] and k, v [B, Hkv, L, D] with Hkv "
                             f"dividing H, got {tuple(q.shape)}, {tuple(k.shape)}, "
                             f"{tuple(v.shape)}")
        if meta.dim() != 1:
            raise ValueError(f"meta must be 1-D, got {tuple(meta.shape)}")
        B, H, L, D = q.shape
        Hkv = k.shape[1]
        lib = _lib.load()
        ctx.dtypes = (q.dtype, k.dtype, v.dtype, meta.dtype)
        q_lo = k_lo = None
        if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16:
            q, q_lo = _split(q)
            k, k_lo = _split(k)
        else:
            q, k = q.contiguous(), k.contiguous()
        v = v.to(torch.bfloat16).contiguous()
        meta = meta.float().contiguous()
        n_meta = meta.numel()
        y = torch.empty(B, H, L, D, device=q.device, dtype=torch.bfloat16)
        save = any(ctx.needs_input_grad[:4])
        saved = None
        if save:
            saved = torch.empty(_lib.size_query("lz_swa_saved_bytes", B, H, L, D), device=q.device,
                                dtype=torch.uint8)
        with _lib.on_device(q.device):
            rc = lib.lz_swa_fwd_gqa(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(q_lo),
                                    _lib.ptr(k_lo), _lib.ptr(meta) if n_meta else None,
                                    n_meta, int(window), _lib.ptr(y), _lib.ptr(saved),
                                    0 if saved is None else saved.numel(), B, H, Hkv, L, D,
                                    _lib.stream_of(q))
        _lib.check(rc, "swa forward")
        if save:
            ctx.save_for_backward(q, k, v, meta, saved, q_lo, k_lo)
        ctx.window = int(window)
        return y

    @staticmethod
    def backward(ctx, dy):
        q, k, v, meta, saved, q_lo, k_lo = ctx.saved_tensors
        B, H, L, D = q.shape
        Hkv = k.shape[1]
        n_meta = meta.numel()
        lib = _lib.load()
        dy = dy.to(torch.bfloat16).contiguous()
        all_bf16 = all(d == torch.bfloat16 for d in ctx.dtypes[:3])
        gdt = _lib.LZ_DTYPE_BF16 if all_bf16 else _lib.LZ_DTYPE_F32
        gtorch = torch.bfloat16 if all_bf16 else torch.float32
        dq = torch.empty(B, H, L, D, device=q.device, dtype=gtorch)
        dk = torch.empty(B, Hkv, L, D, device=q.device, dtype=gtorch)
        dv = torch.empty_like(dk)
        dmeta = torch.empty(n_meta, device=q.device, dtype=torch.float32)
        nws = _lib.size_query("lz_swa_bwd_workspace_bytes", B, H, L, D, n_meta)
        ws = torch.empty(nws, device=q.device, dtype=torch.uint8)
        with _lib.on_device(q.device):
            rc = lib.lz_swa_bwd_gqa(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _lib.ptr(q_lo),
                                    _lib.ptr(k_lo), _lib.ptr(meta) if n_meta else None,
                                    n_meta, ctx.window, _lib.ptr(saved), saved.numel(),
                                    _lib.ptr(dy), _lib.ptr(dq), _lib.ptr(dk), _lib.ptr(dv), gdt,
                                    _lib.ptr(dmeta) if n_meta else None, _lib.ptr(ws),
                                    ws.numel(), B, H, Hkv, L, D, _lib.stream_of(q))
        _lib.check(rc, "swa backward")
        grads = (dq, dk, dv, dmeta)
        dq, dk, dv, dmeta = (g.to(d) for g, d in zip(grads, ctx.dtypes))
        return dq, dk, dv, dmeta, None, None, None


def _split(x):
    """x -> (bf16(x), bf16(x - bf16(x))), both contiguous."""
    hi = x.to(torch.bfloat16).contiguous()
    lo = (x.float() - hi.float()).to(torch.bfloat16).contiguous()
    return hi, lo


def _check_blocks(blocks, name):
    if len(blocks) != 2 or any(int(b) < 1 for b in blocks):
        raise ValueError(f"{name} must be two positive block sizes, got {blocks!r}")


def swa(q, k, v, meta, window, fwd_blocks=FWD_BLOCKS, bwd_blocks=BWD_BLOCKS):
    """y_i = sum_{t in [i-window+1, i]} e^{s_it} v_t / (sum_j e^{meta_j} + sum_t e^{s_it}),
    s_it = q_i . k_t / sqrt(D). q [B, H, L, D], k, v [B, Hkv, L, D] with Hkv
    dividing H (q, k already rotated);
    meta [n_meta] sink logits (may be empty). Returns bf16 [B, H, L, D]."""
    _check_blocks(fwd_blocks, "fwd_blocks")
    _check_blocks(bwd_blocks, "bwd_blocks")
    if int(window) < 1:
        raise ValueError("window must be >= 1")
    return _SWA.apply(q, k, v, meta, window, tuple(fwd_blocks), tuple(bwd_blocks))
