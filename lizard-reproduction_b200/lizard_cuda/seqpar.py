"""Sequence-parallel GLA: one long sequence split over the ranks of a group.

Rank r of P owns tokens [r*Ls, (r+1)*Ls) of every head. The chunked GLA
recurrence (the reference's state pass, src/kernels/gla.py:44-57 forward and
118-132 backward) is linear in the state, so each rank runs its own segment
from a zero state and the ranks only exchange one summary each:

forward   state after the segment from a zero start, its normaliser z, and the
          segment's total log decay; rank r's incoming state is the walk
          h <- h * exp(logdecay_q) + state_q over the ranks q < r.
backward  the gradient w.r.t. the state entering the segment from the
          segment's own outputs (computed after the forward, so it already
          uses the final denominators); rank r's outgoing-state gradient is the
          same walk over the ranks q > r, last rank first. The log-gate
          gradient is a reverse cumsum, so each rank also adds the totals of
          the later ranks.

One all_gather per direction (plus one of P*rows floats for the gate totals)
replaces a rank-to-rank chain of P-1 dependent hops. The arithmetic of every
phase runs in liblizard_cuda (lz_gla_seg_*); torch.distributed only moves the
summaries.
"""
import torch

from . import _lib
from .gla import _shapes


class DistExchange:
    """all_gather over a torch.distributed process group (NCCL on GPUs)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist, self.group = dist, group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)

    def all_gather(self, t):
        """[size, *t.shape]: every rank's t, gathered straight into one buffer
        (no per-rank tensors and no stacking copy)."""
        flat = t.contiguous().reshape(-1)
        out = torch.empty(self.size * flat.numel(), dtype=t.dtype, device=t.device)
        self.dist.all_gather_into_tensor(out, flat, group=self.group)
        return out.view(self.size, *t.shape)


class ChainExchange(DistExchange):
    """Rank-to-rank send / recv instead of all_gather (NCCL point-to-point over
    NVLink on GPUs): the partial summary of the ranks before this one (forward)
    or after it (backward) travels along the chain, and each rank folds its own
    summary in with the same combine step before passing it on. P - 1 dependent
    hops per direction instead of one collective; the arithmetic is the
    all_gather path's step for step, so the states are the same."""

    chain = True

    def _peer(self, r):
        return r if self.group is None else self.dist.get_global_rank(self.group, r)

    def chain_seed(self, ops, summary, reverse):
        """This rank's seed (None at the chain's start): the combined summary of
        the ranks before it (forward) or after it (backward)."""
        P, r = self.size, self.rank
        src, dst = (r + 1, r - 1) if reverse else (r - 1, r + 1)
        part = None
        if 0 <= src < P:
            part = torch.empty_like(summary)
            self.dist.recv(part, self._peer(src), group=self.group)
        if 0 <= dst < P:
            if part is None:
                out = summary
            else:
                # a three-entry buffer whose combine walks the received partial,
                # then this rank (entries 0, 1 forward; 2, 1 backward)
                buf = torch.zeros(3, summary.numel(), dtype=summary.dtype, device=summary.device)
                if reverse:
                    buf[1], buf[2] = summary, part
                    folded = ops.combine(buf, 0, reverse=True)
                else:
                    buf[0], buf[1] = part, summary
                    folded = ops.combine(buf, 2, reverse=False)
                n = folded.numel()  # the state and normaliser; the total log decays add
                out = torch.cat([folded.to(summary.dtype), part[n:] + summary[n:]])
            self.dist.send(out.contiguous(), self._peer(dst), group=self.group)
        return None if part is None else part[:ops.seed_floats()]

    def chain_later_totals(self, own):
        """Sum of the log-gate gradient totals of the ranks after this one."""
        P, r = self.size, self.rank
        later = torch.zeros_like(own)
        if r + 1 < P:
            self.dist.recv(later, self._peer(r + 1), group=self.group)
        if r > 0:
            self.dist.send((later + own).contiguous(), self._peer(r - 1), group=self.group)
        return later


class CudaSegmentOps:
    """The segment phases through the C ABI (lz_gla_seg_* in include/lizard_cuda.h)."""

    def __init__(self, B, H, L, F, D, per_head, device):
        self.lib = _lib.load()
        self.dims = (B, H, L, F, D)
        self.per_head = per_head
        self.device = device
        self.nsum = self.lib.lz_gla_seg_summary_floats(B, H, F, D)
        nbytes = self.lib.lz_gla_seg_workspace_bytes(B, H, L, F, D)
        self.ws = torch.empty(nbytes, device=device, dtype=torch.uint8)

    def _call(self, name, *args):
        with _lib.on_device(self.device):
            rc = getattr(self.lib, name)(*args)
        _lib.check(rc, name)

    def _stream(self):
        return _lib.stream_of(self.ws)

    def seed_floats(self):
        B, H, L, F, D = self.dims
        return B * H * F * (D + 1)

    def fwd_begin(self, fk, v, lg):
        B, H, L, F, D = self.dims
        summary = torch.empty(self.nsum, device=self.device, dtype=torch.float32)
        self._call("lz_gla_seg_fwd_begin", _lib.ptr(fk), _lib.ptr(v), _lib.ptr(lg), self.per_head,
                   _lib.ptr(summary), _lib.ptr(self.ws), self.ws.numel(), B, H, L, F, D,
                   self._stream())
        return summary

    def combine(self, summaries, rank, reverse):
        B, H, L, F, D = self.dims
        P = summaries.shape[0]
        seed = torch.empty(B * H * F * (D + 1), device=self.device, dtype=torch.float32)
        self._call("lz_gla_seg_combine", _lib.ptr(summaries), P, rank, int(reverse),
                   _lib.ptr(seed), B, H, F, D, self._stream())
        return seed

    def fwd_end(self, fq, fk, v, lg, seed, save):
        B, H, L, F, D = self.dims
        y = torch.empty(B, H, L, D, device=self.device, dtype=torch.bfloat16)
        saved = None
        if save:
            saved = torch.empty(self.lib.lz_gla_saved_bytes(B, H, L, F, D, 64),
                                device=self.device, dtype=torch.uint8)
        self._call("lz_gla_seg_fwd_end", _lib.ptr(fq), _lib.ptr(fk), _lib.ptr(v), _lib.ptr(lg),
                   self.per_head, _lib.ptr(seed), _lib.ptr(y), _lib.ptr(saved),
                   0 if saved is None else saved.numel(), _lib.ptr(self.ws), self.ws.numel(),
                   B, H, L, F, D, self._stream())
        return y, saved

    def bwd_begin(self, fq, saved, dy):
        B, H, L, F, D = self.dims
        summary = torch.empty(self.nsum, device=self.device, dtype=torch.float32)
        self._call("lz_gla_seg_bwd_begin", _lib.ptr(fq), _lib.ptr(saved), saved.numel(),
                   _lib.ptr(dy), _lib.ptr(summary), _lib.ptr(self.ws), self.ws.numel(),
                   B, H, L, F, D, self._stream())
        return summary

    def bwd_end(self, fq, fk, v, saved, dy, dseed, seeded_forward, grad_dtype):
        B, H, L, F, D = self.dims
        gdt = _lib.LZ_DTYPE_BF16 if grad_dtype == torch.bfloat16 else _lib.LZ_DTYPE_F32
        dfq = torch.empty(B, H, L, F, device=self.device, dtype=grad_dtype)
        dfk = torch.empty_like(dfq)
        dv = torch.empty(B, H, L, D, device=self.device, dtype=grad_dtype)
        shape = (B, H, L) if self.per_head else (B, L)
        dlg = torch.empty(shape, device=self.device, dtype=torch.float32)
        self._call("lz_gla_seg_bwd_end", _lib.ptr(fq), _lib.ptr(fk), _lib.ptr(v), self.per_head,
                   _lib.ptr(saved), saved.numel(), _lib.ptr(dy), _lib.ptr(dseed),
                   int(seeded_forward), _lib.ptr(dfq), _lib.ptr(dfk), _lib.ptr(dv), gdt,
                   _lib.ptr(dlg), _lib.ptr(self.ws), self.ws.numel(), B, H, L, F, D,
                   self._stream())
        return dfq, dfk, dv, dlg

    def gate_offset(self, dlg, totals, rank):
        rows, L = dlg.numel() // dlg.shape[-1], dlg.shape[-1]
        self._call("lz_gla_seg_gate_offset", _lib.ptr(dlg), _lib.ptr(totals), totals.shape[0],
                   rank, rows, L, self._stream())


def _seed(ops, comm, summary, reverse):
    """The seed of this rank from every rank's summary: one all_gather and a
    combine, or the send / recv chain of a ChainExchange. None for the first
    rank (forward) or the last (backward)."""
    if getattr(comm, "chain", False):
        return comm.chain_seed(ops, summary, reverse)
    summaries = comm.all_gather(summary)
    edge = comm.size - 1 if reverse else 0
    return None if comm.rank == edge else ops.combine(summaries, comm.rank, reverse)


def forward_phases(ops, comm, fq, fk, v, lg, save):
    """One rank's forward: returns (y, saved, seeded)."""
    summary = ops.fwd_begin(fk, v, lg)
    seed = _seed(ops, comm, summary, reverse=False)
    y, saved = ops.fwd_end(fq, fk, v, lg, seed, save)
    return y, saved, seed is not None


def backward_phases(ops, comm, fq, fk, v, saved, dy, seeded, grad_dtype):
    """One rank's backward: returns (dfq, dfk, dv, dlog_gamma) for its segment."""
    summary = ops.bwd_begin(fq, saved, dy)
    dseed = _seed(ops, comm, summary, reverse=True)
    dfq, dfk, dv, dlg = ops.bwd_end(fq, fk, v, saved, dy, dseed, seeded, grad_dtype)
    own = dlg[..., 0].contiguous().reshape(-1)
    if getattr(comm, "chain", False):
        later = comm.chain_later_totals(own)
        ops.gate_offset(dlg, torch.stack([torch.zeros_like(later), later]), 0)
    else:
        ops.gate_offset(dlg, comm.all_gather(own), comm.rank)
    return dfq, dfk, dv, dlg


class _GLASeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, fq, fk, v, log_gamma, comm, ops):
        ctx.dtypes = (fq.dtype, fk.dtype, v.dtype, log_gamma.dtype)
        fq, fk, v = (t.to(torch.bfloat16).contiguous() for t in (fq, fk, v))
        lg = log_gamma.float().contiguous()
        save = any(ctx.needs_input_grad[:4])
        y, saved, seeded = forward_phases(ops, comm, fq, fk, v, lg, save)
        if save:
            ctx.save_for_backward(fq, fk, v, saved)
        ctx.comm, ctx.ops, ctx.seeded = comm, ops, seeded
        return y

    @staticmethod
    def backward(ctx, dy):
        fq, fk, v, saved = ctx.saved_tensors
        dy = dy.to(torch.bfloat16).contiguous()
        all_bf16 = all(d == torch.bfloat16 for d in ctx.dtypes[:3])
        gtorch = torch.bfloat16 if all_bf16 else torch.float32
        grads = backward_phases(ctx.ops, ctx.comm, fq, fk, v, saved, dy, ctx.seeded, gtorch)
        dfq, dfk, dv, dlg = (g.to(d) for g, d in zip(grads, ctx.dtypes))
        return dfq, dfk, dv, dlg, None, None


def gla_seqpar(fq, fk, v, log_gamma, group=None, comm=None, ops=None, exchange="all_gather"):
    """gla() of one sequence split over the ranks of `group` (default: the world).

    fq, fk [B, H, Ls, F], v [B, H, Ls, D] and log_gamma [B, Ls] or [B, H, Ls] are
    this rank's contiguous slice of the sequence (rank order = sequence order;
    the slices may differ in length). Returns this rank's slice of
    y (bf16); gradients flow to all four inputs as in gla(). `comm` (an object
    with rank, size and all_gather) and `ops` (the segment phases) default to
    torch.distributed and the CUDA library. `exchange` picks how the default
    comm moves the chunk-state summaries: "all_gather" (one collective per
    direction, the default) or "chain" (rank-to-rank send / recv, P - 1
    dependent hops).
    """
    B, H, Hkv, L, F, D, per_head = _shapes(fq, fk, v, log_gamma)
    if Hkv != H:
        raise ValueError("gla_seqpar takes fk and v with the query head count; "
                         "repeat_interleave grouped keys / values first")
    if exchange not in ("all_gather", "chain"):
        raise ValueError(f"exchange must be 'all_gather' or 'chain', got {exchange!r}")
    if comm is None:
        comm = ChainExchange(group) if exchange == "chain" else DistExchange(group)
    if ops is None:
        _lib.require_cuda(fq, fk, v, log_gamma)
        ops = CudaSegmentOps(B, H, L, F, D, per_head, fq.device)
    return _GLASeq.apply(fq, fk, v, log_gamma, comm, ops)


class _SWASeq(torch.autograd.Function):
    """Sliding-window attention of one sequence split over the ranks of `comm`.

    A query sees the keys of the W - 1 positions before it (the reference's key
    loop starts W - 1 rows before the query block, src/kernels/swa.py:40-41), so
    rank r needs the last W - 1 rows of k and v of rank r - 1: its halo. Every
    rank all-gathers its tail once (forward) and every halo gradient once
    (backward), so all ranks make the same collective calls. The rank's own
    slice runs as one plain call; its first W - 1 outputs, which lack the halo,
    are replaced by a second call over [halo, first W - 1 rows] whose halo
    positions carry zero queries and zero output gradients (they add nothing to
    any gradient). The key/value gradient of the halo goes back to the rank that
    sent it and is added to its last W - 1 rows.
    """

    @staticmethod
    def forward(ctx, q, k, v, meta, window, comm, attn):
        h = int(window) - 1
        Ls = q.shape[2]
        if h > Ls:
            raise ValueError(f"swa_seqpar needs at least window - 1 = {h} positions per rank, "
                             f"this rank has {Ls}")
        rank = comm.rank
        tails = comm.all_gather(torch.stack([k[:, :, Ls - h:], v[:, :, Ls - h:]])) if h else None
        with torch.enable_grad():
            leaves = [t.detach().requires_grad_(t.requires_grad or t.is_floating_point())
                      for t in (q, k, v, meta)]
            lq, lk, lv, lm = leaves
            y = attn(lq, lk, lv, lm, window)
            halo = None
            if rank > 0 and h:
                halo = tails[rank - 1].detach().requires_grad_()
                zq = torch.zeros_like(lq[:, :, :h])
                ys = attn(torch.cat([zq, lq[:, :, :h]], 2), torch.cat([halo[0], lk[:, :, :h]], 2),
                          torch.cat([halo[1], lv[:, :, :h]], 2), lm, window)[:, :, h:]
                y = torch.cat([ys, y[:, :, h:]], 2)
        ctx.inner = (y, leaves, halo)
        ctx.h, ctx.comm = h, comm
        return y.detach()

    @staticmethod
    def backward(ctx, dy):
        y, leaves, halo = ctx.inner
        h, comm = ctx.h, ctx.comm
        inputs = leaves + ([halo] if halo is not None else [])
        grads = list(torch.autograd.grad(y, inputs, dy, allow_unused=True))
        for i, t in enumerate(inputs):
            if grads[i] is None:
                grads[i] = torch.zeros_like(t)
        if h:
            dhalo = grads.pop() if halo is not None else None
            k = leaves[1]
            send = dhalo if dhalo is not None else torch.zeros(
                (2,) + tuple(k.shape[:2]) + (h, k.shape[-1]), dtype=grads[1].dtype,
                device=k.device)
            back = comm.all_gather(send.to(grads[1].dtype))
            if comm.rank + 1 < comm.size:  # the next rank's halo is this rank's tail
                Ls = k.shape[2]
                grads[1][:, :, Ls - h:] += back[comm.rank + 1][0].to(grads[1].dtype)
                grads[2][:, :, Ls - h:] += back[comm.rank + 1][1].to(grads[2].dtype)
        ctx.inner = None
        return grads[0], grads[1], grads[2], grads[3], None, None, None


def swa_seqpar(q, k, v, meta, window, group=None, comm=None, attn=None):
    """swa() of one sequence split over the ranks of `group` (default: the world).

    q [B, H, Ls, D], k, v [B, Hkv, Ls, D] (rotated, as swa() takes them) are this
    rank's contiguous slice (rank order = sequence order, every slice at least
    window - 1 long); meta [n_meta] is shared. Returns this rank's slice of y.
    Gradients flow to q, k, v and meta; meta's gradient is this rank's share,
    to be summed over the group like any replicated parameter's. `attn` is the
    attention call (default lizard_cuda.swa); `comm` as in gla_seqpar.
    """
    if comm is None:
        comm = DistExchange(group)
    if attn is None:
        from .swa import swa as attn
    return _SWASeq.apply(q, k, v, meta, int(window), comm, attn)
