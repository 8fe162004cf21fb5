"""Test infrastructure: the segment phases of sequence-parallel GLA restated
densely in float64 on the CPU, with the same interface as
lizard_cuda.seqpar.CudaSegmentOps. It lets the CPU tests run the real
orchestration (lizard_cuda.seqpar.forward_phases / backward_phases, over gloo)
and check it against the unsharded oracle. Not used by the product path.

Conventions shared with the CUDA segment calls (include/lizard_cuda.h):
summary = state [BH,F,D] | zstate [BH,F] | logdecay [BH]; seed = state | zstate;
the z part of a backward summary or seed is -dL/dz, as the reference's dz
(src/kernels/gla.py:131-132, 188).
"""
import torch


class ThreadExchange:
    """all_gather between threads of one process (virtual ranks on one GPU)."""

    def __init__(self, shared, rank, size):
        self.shared, self.rank, self.size = shared, rank, size

    @staticmethod
    def make_shared(size):
        import threading
        return {"barrier": threading.Barrier(size, timeout=120), "slots": [None] * size}

    def all_gather(self, t):
        sh = self.shared
        sh["slots"][self.rank] = t.contiguous()
        sh["barrier"].wait()
        out = torch.stack(sh["slots"])
        sh["barrier"].wait()
        return out


class OracleSegmentOps:
    def __init__(self, per_head, heads):
        self.per_head, self.H = per_head, heads
        self.st = {}

    def _G(self, lg):
        G = torch.cumsum(lg.double(), -1)
        if not self.per_head:
            G = G[:, None].expand(-1, self.H, -1)
        return G

    @staticmethod
    def _split(x, BH, F, D, with_decay=True):
        nS, nZ = BH * F * D, BH * F
        S = x[..., :nS].reshape(*x.shape[:-1], BH, F, D)
        z = x[..., nS:nS + nZ].reshape(*x.shape[:-1], BH, F)
        lam = x[..., nS + nZ:nS + nZ + BH] if with_decay else None
        return S, z, lam

    def fwd_begin(self, fk, v, lg):
        self.dims = (fk.shape[0], fk.shape[1], fk.shape[3], v.shape[-1])
        fk, v = fk.double(), v.double()
        G = self._G(lg)
        w = torch.exp(G[..., -1:] - G)
        E = torch.einsum("bhl,bhlf,bhld->bhfd", w, fk, v)
        zE = torch.einsum("bhl,bhlf->bhf", w, fk)
        return torch.cat([E.flatten(), zE.flatten(), G[..., -1].flatten()])

    def seed_floats(self):
        B, H, F, D = self.dims
        return B * H * F * (D + 1)

    def combine(self, summaries, rank, reverse):
        B, H, F, D = self.dims
        S, z, lam = self._split(summaries.double(), B * H, F, D)
        h, hz = torch.zeros_like(S[0]), torch.zeros_like(z[0])
        order = range(rank) if not reverse else range(summaries.shape[0] - 1, rank, -1)
        for q in order:
            e = torch.exp(lam[q])
            h = h * e[:, None, None] + S[q]
            hz = hz * e[:, None] + z[q]
        return torch.cat([h.flatten(), hz.flatten()])

    def _segment(self, fq, fk, v, G, S_in, z_in):
        L = fq.shape[2]
        causal = torch.ones(L, L, dtype=torch.bool).tril()
        dec = torch.exp((G[..., :, None] - G[..., None, :]).masked_fill(~causal, float("-inf")))
        A = (fq @ fk.transpose(-1, -2)) * dec
        Qt = fq * torch.exp(G)[..., None]
        num = A @ v + Qt @ S_in
        den = A.sum(-1) + (Qt * z_in[:, :, None, :]).sum(-1)
        y = num / den[..., None]
        w = torch.exp(G[..., -1:] - G)
        lam = torch.exp(G[..., -1])
        S_out = lam[..., None, None] * S_in + torch.einsum("bhl,bhlf,bhld->bhfd", w, fk, v)
        z_out = lam[..., None] * z_in + torch.einsum("bhl,bhlf->bhf", w, fk)
        return y, den, S_out, z_out

    def fwd_end(self, fq, fk, v, lg, seed, save):
        B, H, L, F = fq.shape
        D = v.shape[-1]
        self.dims = (B, H, F, D)
        G = self._G(lg)
        if seed is None:
            S_in = torch.zeros(B, H, F, D, dtype=torch.float64)
            z_in = torch.zeros(B, H, F, dtype=torch.float64)
        else:
            S, z, _ = self._split(seed.double(), B * H, F, D, with_decay=False)
            S_in, z_in = S.reshape(B, H, F, D), z.reshape(B, H, F)
        y, den, _, _ = self._segment(fq.double(), fk.double(), v.double(), G, S_in, z_in)
        self.st = dict(G=G, S_in=S_in, z_in=z_in, y=y, den=den)
        return y.float(), torch.zeros(1)

    def bwd_begin(self, fq, saved, dy):
        st = self.st
        Qh = fq.double() * (torch.exp(st["G"]) / st["den"])[..., None]
        delta = (dy.double() * st["y"]).sum(-1)
        Dst = torch.einsum("bhlf,bhld->bhfd", Qh, dy.double())
        dz = torch.einsum("bhlf,bhl->bhf", Qh, delta)
        return torch.cat([Dst.flatten(), dz.flatten(), st["G"][..., -1].flatten()])

    def bwd_end(self, fq, fk, v, saved, dy, dseed, seeded_forward, grad_dtype):
        st = self.st
        B, H, F, D = self.dims
        leaves = [t.double().detach().requires_grad_() for t in (fq, fk, v)]
        with torch.enable_grad():
            y, _, S_out, z_out = self._segment(*leaves, st["G"], st["S_in"], st["z_in"])
            loss = (dy.double() * y).sum()
            if dseed is not None:
                dS, dz, _ = self._split(dseed.double(), B * H, F, D, with_decay=False)
                loss = loss + (dS.reshape(B, H, F, D) * S_out).sum() - \
                    (dz.reshape(B, H, F) * z_out).sum()
            dfq, dfk, dv = torch.autograd.grad(loss, leaves)
        dG = (leaves[0].detach() * dfq - leaves[1].detach() * dfk).sum(-1)
        if not self.per_head:
            dG = dG.sum(1)
        dlg = torch.flip(torch.cumsum(torch.flip(dG, [-1]), -1), [-1])
        return dfq.to(grad_dtype), dfk.to(grad_dtype), dv.to(grad_dtype), dlg.float()

    def gate_offset(self, dlg, totals, rank):
        later = totals[rank + 1:].sum(0) if rank + 1 < totals.shape[0] else 0 * totals[0]
        dlg += later.reshape(dlg.shape[:-1])[..., None]
