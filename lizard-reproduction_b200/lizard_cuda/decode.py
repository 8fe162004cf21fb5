"""Recurrent decode for the Lizard layer: O(1) work per new token.

The reference has no cache; its layer recomputes the whole sequence on every
call (src/lizard_attention.py:78-97). Both branches have a recurrent form
that gives the full-sequence output at the new position:
  * GLA: a running state S [F, D] and normaliser z [F] (fp32), decayed by the
    token's gate and extended by fk^T v, read out as fq S / (fq . z);
  * SWA: a ring of the last `window` rotated keys and values (fp32), attended
    with the sink logits.
gla_state / swa_ring build both from a prompt; gla_decode / swa_decode advance
them by one token on the GPU (lz_gla_decode, lz_swa_decode).

With a gate shared by the heads (log_gamma [B, L], the layer's case) and
grouped keys / values, the H / Hkv query heads of a group read the same state,
so the cache keeps Hkv states per batch row.
"""
from dataclasses import dataclass

import torch

from . import _lib

_DT = {torch.float32: _lib.LZ_DTYPE_F32, torch.bfloat16: _lib.LZ_DTYPE_BF16}


def gla_state(fk, v, log_gamma):
    """(S [B, Hs, F, D], z [B, Hs, F]) fp32 after the prompt, from a zero state.
    fk [B, Hs, L, F], v [B, Hs, L, D], log_gamma [B, L] or [B, Hs, L]."""
    _lib.require_cuda(fk, v, log_gamma)
    B, Hs, L, F = fk.shape
    D = v.shape[-1]
    if tuple(v.shape[:3]) != (B, Hs, L):
        raise ValueError(f"v must be [B, Hs, L, D] matching fk, got {tuple(v.shape)}")
    per_head = {(B, L): 0, (B, Hs, L): 1}.get(tuple(log_gamma.shape))
    if per_head is None:
        raise ValueError(f"log_gamma must be [B, L] or [B, Hs, L], got {tuple(log_gamma.shape)}")
    lib = _lib.load()
    fk16, v16 = fk.to(torch.bfloat16).contiguous(), v.to(torch.bfloat16).contiguous()
    lg = log_gamma.float().contiguous()
    ws = torch.empty(lib.lz_gla_seg_workspace_bytes(B, Hs, L, F, D), device=fk.device,
                     dtype=torch.uint8)
    summary = torch.empty(lib.lz_gla_seg_summary_floats(B, Hs, F, D), device=fk.device,
                          dtype=torch.float32)
    with _lib.on_device(fk.device):
        rc = lib.lz_gla_seg_fwd_begin(_lib.ptr(fk16), _lib.ptr(v16), _lib.ptr(lg), per_head,
                                      _lib.ptr(summary), _lib.ptr(ws), ws.numel(), B, Hs, L, F,
                                      D, _lib.stream_of(fk))
    _lib.check(rc, "gla state")
    nS, nZ = B * Hs * F * D, B * Hs * F
    return summary[:nS].view(B, Hs, F, D).clone(), summary[nS:nS + nZ].view(B, Hs, F).clone()


def gla_decode(fq, fk, v, log_gamma, state, zstate):
    """One token: fq [B, H, F], fk [B, Hkv, F], v [B, Hkv, D], log_gamma [B] or
    [B, H]; state [B, Hs, F, D] and zstate [B, Hs, F] (fp32, Hs = H or Hkv)
    advance in place. Returns y bf16 [B, H, D]."""
    _lib.require_cuda(fq, fk, v, log_gamma, state, zstate)
    B, H, F = fq.shape
    Hkv, D = fk.shape[1], v.shape[-1]
    Hs = state.shape[1]
    if state.dtype != torch.float32 or not state.is_contiguous() or not zstate.is_contiguous():
        raise ValueError("state and zstate must be contiguous fp32 tensors")
    if tuple(state.shape) != (B, Hs, F, D) or tuple(zstate.shape) != (B, Hs, F):
        raise ValueError(f"state must be [B, Hs, F, D] and zstate [B, Hs, F], got "
                         f"{tuple(state.shape)}, {tuple(zstate.shape)}")
    per_head = 1 if log_gamma.dim() == 2 else 0
    lib = _lib.load()
    fq16, fk16, v16 = (t.to(torch.bfloat16).contiguous() for t in (fq, fk, v))
    lg = log_gamma.float().contiguous()
    y = torch.empty(B, H, D, device=fq.device, dtype=torch.bfloat16)
    rc = lib.lz_gla_decode(_lib.ptr(fq16), _lib.ptr(fk16), _lib.ptr(v16), _lib.ptr(lg),
                           per_head, _lib.ptr(state), _lib.ptr(zstate), _lib.ptr(y), B, H, Hkv,
                           Hs, F, D, _lib.stream_of(fq))
    _lib.check(rc, "gla decode")
    return y


def rotate(x, cos, sin):
    """Llama rotate-half RoPE in fp32, as the reference's caller evaluates it
    (src/lizard_attention.py:87-88): x [B, Hx, L, D], cos / sin [B, L, D]."""
    x, cos, sin = x.float(), cos.float()[:, None], sin.float()[:, None]
    half = x.shape[-1] // 2
    return x * cos + torch.cat([-x[..., half:], x[..., :half]], -1) * sin


def swa_ring(k, v, cos, sin, window):
    """Rings after a prompt: rotated keys and values of its last `window`
    tokens (fp32 [B, Hkv, window, D]), token t in slot t % window. k, v
    [B, Hkv, L, D] (k unrotated); cos, sin [B, L, D] or [1, L, D]."""
    B, Hkv, L, D = k.shape
    n = min(L, window)
    t = torch.arange(L - n, L, device=k.device)
    kr = rotate(k[:, :, L - n:], cos[:, L - n:].expand(B, n, D), sin[:, L - n:].expand(B, n, D))
    k_ring = torch.zeros(B, Hkv, window, D, device=k.device, dtype=torch.float32)
    v_ring = torch.zeros_like(k_ring)
    k_ring[:, :, t % window] = kr
    v_ring[:, :, t % window] = v[:, :, L - n:].float()
    return k_ring, v_ring


def swa_decode(q, k, v, cos, sin, meta, k_ring, v_ring, pos):
    """One token: q [B, H, D], k, v [B, Hkv, D] (q, k unrotated; strided views
    with a contiguous last dim are read in place), cos, sin [B, D] or [1, D]
    at the token's position, meta [n_meta], rings fp32 [B, Hkv, W, D] and pos
    int32 [B] (tokens before this one; the caller advances it). The new key
    and value go into slot pos % W. Returns y bf16 [B, H, D]."""
    _lib.require_cuda(q, k, v, cos, sin, k_ring, v_ring, pos)
    B, H, D = q.shape
    Hkv, W = k.shape[1], k_ring.shape[2]
    xdt = q.dtype if q.dtype in _DT else torch.float32
    q, k, v = (t if (t.dtype == xdt and t.stride(-1) == 1) else t.to(xdt).contiguous()
               for t in (q, k, v))
    if cos.dtype != sin.dtype or cos.dtype not in _DT:
        cos, sin = cos.float(), sin.float()
    cos, sin = cos.reshape(-1, D).contiguous(), sin.reshape(-1, D).contiguous()
    cs_sb = D if cos.shape[0] == B and B > 1 else 0
    if tuple(k_ring.shape) != (B, Hkv, W, D) or k_ring.dtype != torch.float32:
        raise ValueError(f"k_ring must be fp32 [B, Hkv, W, D], got {tuple(k_ring.shape)}")
    if pos.dtype != torch.int32 or pos.numel() != B:
        raise ValueError("pos must be int32 [B]")
    meta32 = meta.float().contiguous()
    lib = _lib.load()
    y = torch.empty(B, H, D, device=q.device, dtype=torch.bfloat16)
    rc = lib.lz_swa_decode(_lib.ptr(q), _lib.ptr(k), _lib.ptr(v), _DT[xdt], q.stride(0),
                           q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
                           _lib.ptr(cos), _lib.ptr(sin), _DT[cos.dtype], cs_sb,
                           _lib.ptr(k_ring), _lib.ptr(v_ring), _lib.ptr(pos),
                           _lib.ptr(meta32) if meta32.numel() else None, meta32.numel(),
                           _lib.ptr(y), B, H, Hkv, W, D, _lib.stream_of(q))
    _lib.check(rc, "swa decode")
    return y


@dataclass
class LayerCache:
    """Decode state of one Lizard layer."""
    state: torch.Tensor   # fp32 [B, Hs, F, D]
    zstate: torch.Tensor  # fp32 [B, Hs, F]
    k_ring: torch.Tensor  # fp32 [B, Hkv, W, D], rotated keys
    v_ring: torch.Tensor  # fp32 [B, Hkv, W, D]
    pos: torch.Tensor     # int32 [B], tokens seen


class LizardCache(dict):
    """layer_idx -> LayerCache. Pass as `lizard_cache=` to a model whose
    attention layers are lizard_cuda LizardAttention: the first call with a
    layer's index missing runs the full forward over the prompt and stores the
    layer's state; later calls decode their tokens one at a time. Position ids
    of the new tokens must be given to the model (position_ids=)."""
