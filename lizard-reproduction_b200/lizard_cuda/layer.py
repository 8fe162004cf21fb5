"""LizardAttention with the `cuda` backend.

Mirror of the reference layer (src/lizard_attention.py:47-107): same
constructor arguments, parameter names and forward contract
(forward(hidden_states, position_embeddings) -> (out, None)), with the two
attention branches running on this package's gla / swa kernels exactly where
the reference's `triton` backend calls kernels.gla / kernels.swa
(src/lizard_attention.py:90-93), and the Hedgehog feature map on the fused
kernel (lizard_cuda.hedgehog, bf16 features straight into gla).

Keys and values stay at their Hkv heads: the reference repeat_interleaves k
and v to H heads (src/lizard_attention.py:73-76) before the feature map and
both branches, which gives every query head of a group the same fk and v; the
grouped-query kernels read each key/value head once instead, and the feature
map runs on Hkv heads of k. RoPE is fused into the SWA operand pass
(lizard_cuda.swa_rope) and reads the projections in place, and the output
blend, cast and transpose are one kernel (lizard_cuda.blend). Under
torch.no_grad the projections go to the kernels without the reference's fp32
upcast: every kernel converts its inputs to fp32 itself, so the values are the
same, and the upcast copies are skipped. With autograd on, the upcast stays, so
the gradients of q and k add in fp32 as in the reference. The projections and
the gate are the same torch operations as the reference.

Sequence parallelism: forward(..., seq_comm=comm) runs the layer on this
rank's contiguous slice of every sequence (position_embeddings for the slice's
own positions). The GLA branch hands its chunk state to the later ranks
(seqpar.gla_seqpar) and the SWA branch takes the previous rank's last
window - 1 keys and values as a halo (seqpar.swa_seqpar); everything else in
the layer is per token. Parameter gradients are this rank's share, summed over
the group by the caller as for any replicated parameter.
"""
import torch
import torch.nn as nn
import torch.nn.functional as F

from .blend import blend
from .decode import LayerCache, gla_decode, gla_state, swa_decode, swa_ring
from .gla import gla
from .hedgehog import hedgehog as fused_hedgehog
from .rope import swa_rope
from .seqpar import gla_seqpar, swa_seqpar

BACKENDS = ("cuda",)


class LizardAttention(nn.Module):
    def __init__(self, config, layer_idx, window=128, num_meta=4, feature_dim=128,
                 backend="cuda"):
        super().__init__()
        if backend not in BACKENDS:
            raise ValueError(f"this layer runs the cuda backend only, got {backend!r}; the "
                             "torch and triton backends live in the reference package")
        self.backend = backend
        hidden = config.hidden_size
        self.layer_idx = layer_idx
        self.heads = config.num_attention_heads
        self.kv_heads = config.num_key_value_heads
        self.head_dim = hidden // self.heads
        self.window = window
        kv_dim = self.kv_heads * self.head_dim
        self.q_proj = nn.Linear(hidden, hidden, bias=False)
        self.k_proj = nn.Linear(hidden, kv_dim, bias=False)
        self.v_proj = nn.Linear(hidden, kv_dim, bias=False)
        self.o_proj = nn.Linear(hidden, hidden, bias=False)
        self.phi_q = nn.Linear(self.head_dim, feature_dim, bias=False)
        self.phi_k = nn.Linear(self.head_dim, feature_dim, bias=False)
        self.W_gamma = nn.Linear(hidden, 1, bias=False)
        self.meta_tokens = nn.Parameter(torch.zeros(num_meta))
        self.alpha_blend = nn.Parameter(torch.ones(()))
        nn.init.normal_(self.phi_q.weight, std=0.02)
        nn.init.normal_(self.phi_k.weight, std=0.02)
        nn.init.zeros_(self.W_gamma.weight)
        self._casts = {}

    def param_as(self, p, dtype):
        """Parameter p in `dtype`. With autograd on this is p.to(dtype). Without
        it the cast is kept and reused while p is unchanged (same version
        counter and storage), so inference and decode steps do not re-cast the
        small fp32 parameters every call; a cast first made while a CUDA graph
        is being captured is not kept (its values exist only at replay)."""
        if p.dtype == dtype:
            return p
        if torch.is_grad_enabled() and p.requires_grad:
            return p.to(dtype)
        key = (id(p), dtype)
        hit = self._casts.get(key)
        if hit is not None and hit[0] == p._version and hit[1] == p.data_ptr():
            return hit[2]
        out = p.detach().to(dtype)
        if not torch.cuda.is_current_stream_capturing():
            self._casts[key] = (p._version, p.data_ptr(), out)
        return out

    def split(self, x, heads):
        """The reference's head split with repeat_interleave to H heads
        (src/lizard_attention.py:73-76); kept for callers of the method. The
        forward uses heads_view instead."""
        return self.heads_view(x, heads).repeat_interleave(self.heads // heads, dim=1)

    def heads_view(self, x, heads):
        """[B, L, heads * Dh] -> [B, heads, L, Dh] as a view (no copy)."""
        b, n, _ = x.shape
        return x.view(b, n, heads, self.head_dim).transpose(1, 2)

    def forward(self, hidden_states, position_embeddings, lizard_cache=None, seq_comm=None,
                **kwargs):
        """(out, None) as the reference layer. With `lizard_cache` (a
        decode.LizardCache), a layer whose index is in the cache decodes its
        tokens one at a time against the stored state; otherwise it runs the
        full forward and, given a cache, stores its state there. With
        `seq_comm` (a seqpar.DistExchange, or any object with rank, size and
        all_gather) hidden_states is this rank's slice of the sequence."""
        if seq_comm is not None and lizard_cache is not None:
            raise ValueError("a sequence-parallel forward does not fill a decode cache")
        if lizard_cache is not None and self.layer_idx in lizard_cache:
            return self.decode(hidden_states, position_embeddings,
                               lizard_cache[self.layer_idx]), None
        x = hidden_states
        dtype = torch.promote_types(x.dtype, torch.float32)
        up = torch.is_grad_enabled()
        q = self.heads_view(self.q_proj(x), self.heads)
        k = self.heads_view(self.k_proj(x), self.kv_heads)
        v = self.heads_view(self.v_proj(x), self.kv_heads)
        if up:
            q, k, v = q.to(dtype), k.to(dtype), v.to(dtype)
        z = self.W_gamma(x).to(dtype).squeeze(-1)
        fq = fused_hedgehog(q, self.param_as(self.phi_q.weight, dtype))
        fk = fused_hedgehog(k, self.param_as(self.phi_k.weight, dtype))  # Hkv heads
        cos, sin = position_embeddings
        alpha = self.param_as(self.alpha_blend, dtype)
        meta = self.param_as(self.meta_tokens, dtype)
        lg = F.logsigmoid(z)
        if seq_comm is not None:
            y_gla, y_swa = self._seqpar_branches(q, k, v, fq, fk, lg, cos, sin, meta, seq_comm)
        else:
            y_gla = gla(fq, fk, v, lg)
            y_swa = swa_rope(q, k, v, cos, sin, meta, self.window)
        if lizard_cache is not None:
            with torch.no_grad():
                state, zstate = gla_state(fk, v, lg)  # Hkv states: the gate is per token
                k_ring, v_ring = swa_ring(k, v, cos, sin, self.window)
                pos = torch.full((x.shape[0],), x.shape[1], dtype=torch.int32, device=x.device)
                lizard_cache[self.layer_idx] = LayerCache(state, zstate, k_ring, v_ring, pos)
        return self.o_proj(blend(y_gla, y_swa, alpha, x.dtype)), None

    def _seqpar_branches(self, q, k, v, fq, fk, lg, cos, sin, meta, comm):
        """Both attention branches on this rank's slice of the sequence. The
        sequence-parallel GLA takes keys / values at the query head count, so
        the grouped fk and v are repeated here, as the reference's caller does
        (src/lizard_attention.py:73-76); q and k are rotated in fp32 with the
        slice's own positions, as the reference's apply_rotary_pos_emb
        (src/lizard_attention.py:87-88), and the SWA halo carries rotated keys."""
        rep = self.heads // self.kv_heads
        fk_r = fk.repeat_interleave(rep, dim=1) if rep > 1 else fk
        v_r = v.repeat_interleave(rep, dim=1) if rep > 1 else v
        y_gla = gla_seqpar(fq, fk_r, v_r, lg, comm=comm)
        c, s_ = cos.float()[:, None], sin.float()[:, None]
        half = self.head_dim // 2

        def rot(x):
            x = x.float()
            return x * c + torch.cat([-x[..., half:], x[..., :half]], dim=-1) * s_
        y_swa = swa_seqpar(rot(q), rot(k), v, meta, self.window, comm=comm)
        return y_gla, y_swa

    @torch.no_grad()
    def decode(self, hidden_states, position_embeddings, cache):
        """Output for new tokens hidden_states [B, T, hidden] that follow the
        tokens in `cache` (advanced in place), one token at a time: the same
        values as the full forward at those positions, within bf16 rounding.
        position_embeddings are the new tokens' (cos, sin) [B, T, Dh]."""
        x = hidden_states
        dtype = torch.promote_types(x.dtype, torch.float32)
        q = self.heads_view(self.q_proj(x), self.heads)
        k = self.heads_view(self.k_proj(x), self.kv_heads)
        v = self.heads_view(self.v_proj(x), self.kv_heads)
        lg = F.logsigmoid(self.W_gamma(x).to(dtype).squeeze(-1))
        fq = fused_hedgehog(q, self.param_as(self.phi_q.weight, dtype))
        fk = fused_hedgehog(k, self.param_as(self.phi_k.weight, dtype))
        cos, sin = position_embeddings
        meta = self.param_as(self.meta_tokens, dtype)
        y_gla, y_swa = [], []
        for t in range(x.shape[1]):
            y_gla.append(gla_decode(fq[:, :, t], fk[:, :, t], v[:, :, t], lg[:, t], cache.state,
                                    cache.zstate))
            y_swa.append(swa_decode(q[:, :, t], k[:, :, t], v[:, :, t], cos[:, t], sin[:, t],
                                    meta, cache.k_ring, cache.v_ring, cache.pos))
            cache.pos += 1
        if len(y_gla) == 1:  # one new token: views, no stacking copies
            y_gla, y_swa = y_gla[0].unsqueeze(2), y_swa[0].unsqueeze(2)
        else:
            y_gla, y_swa = torch.stack(y_gla, 2), torch.stack(y_swa, 2)
        y = blend(y_gla, y_swa, self.param_as(self.alpha_blend, dtype), x.dtype)
        return self.o_proj(y)


def from_llama(attention, config, **options):
    """Build a LizardAttention from a Llama attention layer, copying q/k/v/o
    (src/lizard_attention.py:100-107)."""
    weight = attention.q_proj.weight
    layer = LizardAttention(config, attention.layer_idx, **options)
    layer = layer.to(weight.device, weight.dtype)
    for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
        getattr(layer, name).load_state_dict(getattr(attention, name).state_dict())
    return layer
