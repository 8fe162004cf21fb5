"""CPU oracle for Lizard's GLA and SWA branches.

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and the
cpu_baseline / reference legs of bench.py may import this module, and only as
the checker or the timed CPU baseline. The CUDA product path never calls it.

It restates, in plain PyTorch on dense L x L tensors, the reference's own
torch backend (mahdikhashan/lizard-reproduction, src/lizard_attention.py),
which the reference uses as the correctness oracle of its kernels
(tests/test_kernels.py:61-70, 121-122):

  hedgehog        src/lizard_attention.py:9-11
  window_mask     src/lizard_attention.py:14-17
  gate_products   src/lizard_attention.py:20-25
  gla             src/lizard_attention.py:28-31
  sink_softmax    src/lizard_attention.py:34-38
  awa             src/lizard_attention.py:41-44
  LizardAttention src/lizard_attention.py:47-97 (torch backend only)
  gla_recurrent   tests/test_lizard.py:41-52 (O(L F D) float64 form)
  rope            tests/test_lizard.py:66-69 (rotate-half RoPE)

Pinning: tests/golden/*.pt hold inputs, outputs and gradients produced by the
reference's own src/lizard_attention.py (script: tests/golden/make_golden.py);
tests/test_oracle.py checks this module against every fixture.

Differences from the reference signatures, both deliberate:
  * gla takes log gates (the argument of the kernel API, src/kernels/gla.py:259)
    instead of gates, and accepts a per-head [B, H, L] gate directly (the
    reference folds B*H into the batch for that case, tests/test_kernels.py:66-70);
  * awa accepts an empty `meta` (no sinks), which the kernel API allows
    (src/kernels/swa.py:34-35) but the dense reference cannot evaluate.
"""
import math

import torch
import torch.nn as nn


def hedgehog(x, weight):
    """[softmax(x W^T), softmax(-x W^T)] along the feature axis."""
    xw = x @ weight.T
    return torch.cat([torch.softmax(xw, -1), torch.softmax(-xw, -1)], dim=-1)


def window_mask(length, window, device=None):
    """True where key t may be seen by query i: t <= i and i - t < window."""
    i = torch.arange(length, device=device)[:, None]
    t = torch.arange(length, device=device)[None, :]
    return (t <= i) & (i - t < window)


def gate_products(gamma):
    """P[..., i, t] = prod_{s=t+1..i} gamma[..., s] for t <= i, else 0.

    Same construction as the reference: mask the gates above the diagonal to
    one, take the reversed cumulative product along t, shift by one column.
    """
    length = gamma.shape[-1]
    causal = window_mask(length, length, gamma.device)
    g = torch.where(causal, gamma[..., None, :], torch.ones((), dtype=gamma.dtype))
    prods = torch.flip(torch.cumprod(torch.flip(g, [-1]), -1), [-1])
    shifted = torch.cat([prods[..., 1:], torch.ones_like(prods[..., :1])], dim=-1)
    return shifted * causal


def gla(fq, fk, v, log_gamma):
    """Dense gated linear attention with a clamped row sum.

    fq, fk [B, H, L, F]; v [B, H, L, D]; log_gamma [B, L] (shared by heads) or
    [B, H, L]. Returns [B, H, L, D] in the inputs' dtype.
    """
    gamma = torch.exp(log_gamma)
    decay = gate_products(gamma)
    if gamma.dim() == 2:
        decay = decay[:, None]
    w = (fq @ fk.transpose(-1, -2)) * decay
    tiny = torch.finfo(w.dtype).tiny
    return (w @ v) / w.sum(-1, keepdim=True).clamp_min(tiny)


def gla_recurrent(fq, fk, v, log_gamma):
    """Recurrent form S_i = g_i S_{i-1} + fk_i v_i^T, y_i = fq_i S_i / fq_i z_i."""
    b, h, n, f = fq.shape
    gamma = torch.exp(log_gamma)
    if gamma.dim() == 2:
        gamma = gamma[:, None].expand(b, h, n)
    S = torch.zeros(b, h, f, v.shape[-1], dtype=fq.dtype)
    z = torch.zeros(b, h, f, dtype=fq.dtype)
    out = []
    for i in range(n):
        g = gamma[:, :, i, None]
        S = g[..., None] * S + fk[:, :, i, :, None] * v[:, :, i, None, :]
        z = g * z + fk[:, :, i]
        num = torch.einsum("bhf,bhfd->bhd", fq[:, :, i], S)
        out.append(num / (fq[:, :, i] * z).sum(-1, keepdim=True))
    return torch.stack(out, dim=2)


def gla_chunked(fq, fk, v, log_gamma, chunk=256):
    """The same map as gla(), evaluated chunk by chunk with a carried state, so
    memory is O(L chunk) instead of O(L^2) and long sequences (L = 16384) fit,
    gradients included (plain autograd through the chunk loop).

    Within a chunk the weights are dense, (fq_i . fk_t) exp(G_i - G_t) for
    t <= i; the keys before the chunk enter through
    S = sum_t exp(G_prev - G_t) fk_t v_t^T and z = sum_t exp(G_prev - G_t) fk_t,
    G_prev the running log gate at the chunk's start, so every exponent is
    <= 0. This is the chunk decomposition of src/kernels/gla.py:33-101
    (states measured from chunk boundaries) without its bf16 roundings; in
    float64 it agrees with gla() and gla_recurrent() to rounding.
    """
    b, h, n, f = fq.shape
    G = torch.cumsum(log_gamma, -1)
    if G.dim() == 2:
        G = G[:, None].expand(b, h, n)
    S = fq.new_zeros(b, h, f, v.shape[-1])
    z = fq.new_zeros(b, h, f)
    g_prev = fq.new_zeros(b, h)
    tiny = torch.finfo(fq.dtype).tiny
    out = []
    for c0 in range(0, n, chunk):
        c1 = min(n, c0 + chunk)
        q, k, vv, g = fq[:, :, c0:c1], fk[:, :, c0:c1], v[:, :, c0:c1], G[:, :, c0:c1]
        causal = torch.ones(c1 - c0, c1 - c0, dtype=torch.bool, device=fq.device).tril()
        diff = (g[..., :, None] - g[..., None, :]).masked_fill(~causal, float("-inf"))
        A = (q @ k.transpose(-1, -2)) * torch.exp(diff)
        qt = q * torch.exp(g - g_prev[..., None])[..., None]
        num = A @ vv + qt @ S
        den = A.sum(-1) + (qt * z[:, :, None, :]).sum(-1)
        out.append(num / den.clamp_min(tiny)[..., None])
        g_end = g[..., -1]
        kt = k * torch.exp(g_end[..., None] - g)[..., None]
        lam = torch.exp(g_end - g_prev)
        S = lam[..., None, None] * S + kt.transpose(-1, -2) @ vv
        z = lam[..., None] * z + kt.sum(-2)
        g_prev = g_end
    return torch.cat(out, dim=2)


def sink_softmax(scores, meta):
    """Softmax over the last axis with exp(meta_j) added to the denominator.

    The running max is detached, as in the reference; with no sinks it is the
    plain softmax.
    """
    m = scores.amax(-1, keepdim=True)
    if meta.numel():
        m = torch.maximum(m, meta.max())
    m = m.detach()
    e = torch.exp(scores - m)
    den = e.sum(-1, keepdim=True)
    if meta.numel():
        den = den + torch.exp(meta - m).sum(-1, keepdim=True)
    return e / den


def awa(q, k, v, meta, window):
    """Sliding-window softmax attention with sink logits, scale 1/sqrt(D)."""
    mask = window_mask(q.shape[-2], window, q.device)
    scores = q @ k.transpose(-1, -2) / math.sqrt(q.shape[-1])
    return sink_softmax(scores.masked_fill(~mask, float("-inf")), meta) @ v


def rotate_half(x):
    half = x.shape[-1] // 2
    return torch.cat([-x[..., half:], x[..., :half]], dim=-1)


def rope(x, cos, sin):
    """x [B, H, L, Dh]; cos, sin [B, L, Dh] (the Llama rotary embedding)."""
    return x * cos[:, None] + rotate_half(x) * sin[:, None]


def rotary_tables(length, head_dim, theta, dtype=torch.float32, start=0):
    """cos/sin [1, L, Dh] of the default Llama rotary embedding (no scaling)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    pos = torch.arange(start, start + length, dtype=torch.float64)
    freqs = torch.outer(pos, inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos()[None].to(dtype), emb.sin()[None].to(dtype)


class LizardAttention(nn.Module):
    """Dense torch restatement of the Lizard layer (parameter names match).

    forward(hidden_states, position_embeddings) -> (out, None), GQA heads
    repeated, math in at least fp32, output in the input dtype.
    """

    def __init__(self, hidden, heads, kv_heads, window=128, num_meta=4, feature_dim=128):
        super().__init__()
        self.heads, self.kv_heads = heads, kv_heads
        self.head_dim = hidden // heads
        self.window = window
        kv_dim = kv_heads * self.head_dim
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

    def split(self, x, heads):
        b, n, _ = x.shape
        x = x.view(b, n, heads, self.head_dim).transpose(1, 2)
        return x.repeat_interleave(self.heads // heads, dim=1)

    def forward(self, hidden_states, position_embeddings, **kwargs):
        x = hidden_states
        dtype = torch.promote_types(x.dtype, torch.float32)
        q = self.split(self.q_proj(x), self.heads).to(dtype)
        k = self.split(self.k_proj(x), self.kv_heads).to(dtype)
        v = self.split(self.v_proj(x), self.kv_heads).to(dtype)
        z = self.W_gamma(x).to(dtype).squeeze(-1)
        fq = hedgehog(q, self.phi_q.weight.to(dtype))
        fk = hedgehog(k, self.phi_k.weight.to(dtype))
        cos, sin = (t.to(dtype) for t in position_embeddings)
        qr, kr = rope(q, cos, sin), rope(k, cos, sin)
        alpha, meta = self.alpha_blend.to(dtype), self.meta_tokens.to(dtype)
        y = gla(fq, fk, v, torch.nn.functional.logsigmoid(z))
        y = y + alpha * awa(qr, kr, v, meta, self.window)
        return self.o_proj(y.to(x.dtype).transpose(1, 2).flatten(2)), None


def rel(a, b):
    """Relative Frobenius error (tests/test_kernels.py:18-20)."""
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm()).item()


def close(a, b, tol, atol=1e-3):
    """||a-b|| <= tol ||b|| + atol sqrt(n) (tests/test_kernels.py:23-25)."""
    a, b = a.double(), b.double()
    return bool((a - b).norm() <= tol * b.norm() + atol * b.numel() ** 0.5)


def max_rel(a, b):
    """max|a-b| / max|b|, the north-star tolerance metric."""
    a, b = a.double(), b.double()
    den = b.abs().max().item()
    return (a - b).abs().max().item() / (den if den > 0 else 1.0)
