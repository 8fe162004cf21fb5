#!/usr/bin/env python
"""Throughput of the Lizard GLA forward on B200.

One step = one gla(fq, fk, v, log_gamma) forward over B=8, H=32, L=2048,
F=D=128 bf16 with a per-head gate [B, H, L] (the reference's Table-3 shape
family, src/benchmark.py:28-41). Inputs (386 MB) exceed the 126 MB L2, so no
flush is needed between steps. With N GPUs every rank runs its own config-2
batch (batch x head shards, weak scaling, no collective on the data path);
value = all ranks' tokens / max-over-ranks device time.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Rank 0 prints one JSON line. `--impl reference` times the CPU oracle (the
restatement of the reference's torch backend, oracle/lizard_oracle.py) on the
host cores for the same metric.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "lizard-reproduction_b200"))

B, H, L, FD, D = 8, 32, 2048, 128, 128
METRIC = "gla_fwd_tokens_per_s"
UNIT = "tokens/s"
BYTES_PER_TOKEN_HEAD = 2 * (2 * FD + 2 * D) + 4         # fq, fk, v, y bf16 + G fp32
FLOPS_PER_TOKEN_HEAD = 2 * (2 * FD * D + 64 * FD + 64 * D)  # state, inter, intra s, intra av
CONFIG = {
    "workload": "gla_fwd config 2: B=8 H=32 L=2048 F=D=128 bf16, per-head gate [B,H,L]",
    "B": B, "H": H, "L": L, "F": FD, "D": D, "gate": "per-head",
    "global_batch_per_gpu": B,
    "l2": "inputs 386 MB > 126 MB L2 (no flush)",
}


# --case workloads: (B, H, L, F = D, per-head gate, forward+backward, op)
CASES = {
    "cfg2-fwd": (8, 32, 2048, 128, True, False, "gla"),
    "cfg3-gla-train": (1, 32, 2048, 64, False, True, "gla"),
    "cfg3-swa-train": (1, 32, 2048, 64, False, True, "swa"),
    "cfg4-train": (16, 32, 16384, 128, True, True, "gla"),
    # feature map of one projection: x [B, H, L, 64] fp32, feature dim 128
    "prologue-fwd": (4, 32, 4096, 64, False, False, "hedgehog"),
    "prologue-train": (4, 32, 4096, 64, False, True, "hedgehog"),
    # config 5: whole-model prefill (B, L only; the architecture is LLAMA_1B)
    "cfg5-prefill": (32, 32, 4096, 64, False, False, "model"),
    # config-5 layer kernels at a batch slice (inference): SWA with RoPE inside on
    # the q / k / v projections (32 / 8 heads, head dim 64, window 64, 4 sinks),
    # and GLA with F = 256, D = 64, grouped keys / values and a per-token gate
    "cfg5-swa-rope": (4, 32, 4096, 64, False, False, "swa_rope"),
    "cfg5-gla": (4, 32, 4096, 256, False, False, "gla_gqa"),
    # the layer's feature map on bf16 projections [B, L, H * 64] (tensor-core forward),
    # its output blend, and one decode step of both branches (B sequences, 8 key/value
    # heads with F = 256 states, window 64)
    "cfg5-hedgehog": (4, 32, 4096, 64, False, False, "hedgehog_bf16"),
    "cfg5-blend": (8, 32, 4096, 64, False, False, "blend"),
    "cfg5-decode": (32, 32, 4096, 256, False, False, "decode"),
    # the same-box comparison against the reference's Triton kernels (and FLA)
    "reference-gpu": (0, 0, 0, 0, False, False, "reference_gpu"),
    # the sequence-parallel leg alone (with its parity check at N > 1)
    "seqpar": (1, 32, 16384, 128, True, True, "seqpar"),
}


def parse():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--no-secondary", action="store_true",
                    help="skip the config-3 fwd+bwd side measurements")
    ap.add_argument("--case", choices=sorted(CASES),
                    help="run only this workload for --steps steps after --warmup steps and "
                         "print its device ms per step (for profiling; not the driver contract)")
    ap.add_argument("--B", type=int, help="batch for --case (default: the config's)")
    ap.add_argument("--L", type=int, help="sequence length for --case (default: the config's)")
    ap.add_argument("--schedule", choices=("auto", "walk", "split"), default="auto",
                    help="GLA schedule for --case (default: chosen per shape)")
    ap.add_argument("--window", type=int, default=64,
                    help="SWA window for --case cfg3-swa-train (default 64)")
    return ap.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("LOCAL_RANK", "0")),
            int(os.environ.get("WORLD_SIZE", "1")))


def make_inputs(torch, device, seed):
    import torch.nn.functional as F
    g = torch.Generator(device=device).manual_seed(seed)
    fq = (F.softplus(torch.randn(B, H, L, FD, generator=g, device=device)) / math.sqrt(D)).bfloat16()
    fk = (F.softplus(torch.randn(B, H, L, FD, generator=g, device=device)) / math.sqrt(D)).bfloat16()
    v = torch.randn(B, H, L, D, generator=g, device=device).bfloat16()
    lg = F.logsigmoid(3 + 1.5 * torch.randn(B, H, L, generator=g, device=device))
    return fq, fk, v, lg


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(",") for r in out.strip().splitlines() if r.count(",") >= 8]
        sm, mx, reasons = [], 0.0, set()
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
            except ValueError:
                continue
            for name, val in zip(self.NAMES, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def physical_gpu(local_rank):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def profiled_traffic():
    """dram bytes per launch of the forward kernel from the committed ncu summary."""
    p = ROOT / "profiles" / "gla_fwd_tc_kernel_cfg2.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


# -------------------------------------------------------------- CPU baseline
def cpu_oracle_rate(torch, fq, fk, v, lg, heads, budget_s, min_runs=1):
    """tokens/s of the dense CPU oracle on `heads` heads of batch row 0."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import lizard_oracle as orc
    a, b_, c, d = (t[0:1, :heads].float().cpu() for t in (fq, fk, v, lg))
    runs, t0 = 0, time.perf_counter()
    with torch.no_grad():
        while runs < min_runs or time.perf_counter() - t0 < budget_s:
            orc.gla(a, b_, c, d)
            runs += 1
    dt = time.perf_counter() - t0
    tokens = runs * L * heads / H  # a token is one position of one batch row, all H heads
    return tokens / dt, runs, dt


def run_reference(args, torch):
    rank, _, world = env_rank()
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    fq, fk, v, lg = make_cpu_inputs(torch)
    sys.path.insert(0, str(ROOT / "oracle"))
    import lizard_oracle as orc
    # size one step so the whole run stays within about two minutes
    probe, _, _ = cpu_oracle_rate(torch, fq, fk, v, lg, 1, 0.0)
    per_head_s = (L / H) / probe
    total = max(1, args.steps + args.warmup)
    heads = int(max(1, min(H, 120.0 / total / per_head_s)))
    a, b_, c, d = (t[0:1, :heads].float() for t in (fq, fk, v, lg))
    with torch.no_grad():
        for _ in range(args.warmup):
            orc.gla(a, b_, c, d)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            orc.gla(a, b_, c, d)
        dt = time.perf_counter() - t0
    tokens = args.steps * L * heads / H
    value = tokens / dt
    sample = (f"each step: dense fp32 torch oracle on {heads} of {B * H} heads "
              f"(batch row 0) of the config-2 workload, L={L}")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3 / max(1, args.steps), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": CONFIG,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def make_cpu_inputs(torch):
    """The config-2 distributions for one batch row, generated on the CPU."""
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(0)
    fq = (F.softplus(torch.randn(1, H, L, FD, generator=g)) / math.sqrt(D)).bfloat16()
    fk = (F.softplus(torch.randn(1, H, L, FD, generator=g)) / math.sqrt(D)).bfloat16()
    v = torch.randn(1, H, L, D, generator=g).bfloat16()
    lg = F.logsigmoid(3 + 1.5 * torch.randn(1, H, L, generator=g))
    return fq, fk, v, lg


# ---------------------------------------------------------------- ours
SEQ_L, SEQ_H, SEQ_FD = 16384, 32, 128


def seqpar_measure(torch, lizard_cuda, device, dist, world, rank, steps=10, warmup=3):
    """Config 4's long sequence: B=1, L=16384, H=32, F=D=128, per-head gate. With
    N ranks each owns L/N tokens of every head and the ranks hand the chunk
    state over through lizard_cuda.seqpar (one all_gather per direction);
    with one GPU it is the plain call. Device ms per step, max over ranks,
    for the forward (no grad) and forward+backward; L2 is not flushed (every
    rank's inputs are >= 201 MB / N per tensor)."""
    import torch.nn.functional as F
    from lizard_cuda import seqpar
    Ls = SEQ_L // world
    g = torch.Generator(device=device).manual_seed(4321 + rank)
    shape = (1, SEQ_H, Ls, SEQ_FD)
    fq = (F.softplus(torch.randn(shape, generator=g, device=device)) / math.sqrt(SEQ_FD)).bfloat16()
    fk = (F.softplus(torch.randn(shape, generator=g, device=device)) / math.sqrt(SEQ_FD)).bfloat16()
    v = torch.randn(shape, generator=g, device=device).bfloat16()
    lg = F.logsigmoid(3 + 1.5 * torch.randn(1, SEQ_H, Ls, generator=g, device=device))
    dy = torch.randn(shape, generator=g, device=device).bfloat16()
    call = (lambda *a: lizard_cuda.gla(*a)) if world == 1 else seqpar.gla_seqpar
    chain = lambda *a: seqpar.gla_seqpar(*a, exchange="chain")  # noqa: E731

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / steps], device=device, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.no_grad():
        fwd = timed(lambda: call(fq, fk, v, lg))
    leaves = [t.detach().requires_grad_() for t in (fq, fk, v, lg)]

    def step():
        for t in leaves:
            t.grad = None
        call(*leaves).backward(dy)
    both = timed(step)
    check = None
    chain_res = None
    if world > 1:
        check = seqpar_check(torch, lizard_cuda, dist, world, rank,
                             (fq, fk, v, lg, dy), [t.grad for t in leaves])
        # the same step with the summaries passed rank to rank (NCCL send / recv,
        # P - 1 dependent hops per direction) instead of one all_gather
        ref = [leaves[0].grad.clone(), leaves[1].grad.clone(), leaves[2].grad.clone(),
               leaves[3].grad.clone()]
        with torch.no_grad():
            y_ag = call(fq, fk, v, lg)
            fwd_c = timed(lambda: chain(fq, fk, v, lg))
            y_c = chain(fq, fk, v, lg)

        def step_c():
            for t in leaves:
                t.grad = None
            chain(*leaves).backward(dy)
        both_c = timed(step_c)
        diffs = [(a.float() - b.float()).abs().max() / b.float().abs().max().clamp_min(1e-30)
                 for a, b in zip([y_c] + [t.grad for t in leaves], [y_ag] + ref)]
        dmax = torch.stack(diffs).double().max().reshape(1)
        dist.all_reduce(dmax, op=dist.ReduceOp.MAX)
        chain_res = {"exchange": "NCCL send / recv chain, P - 1 hops per direction",
                     "fwd_ms": fwd_c, "fwd_bwd_ms": both_c,
                     "max_rel_vs_all_gather": float(dmax.item())}
    # the same forward+backward replayed from one CUDA graph (the collectives
    # inside it): the device time of the sharded step without the host's
    # per-call work, captured and replayed by every rank in the same order
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    both_graph = timed(graph.replay)
    del graph
    return {"workload": f"gla config 4 long sequence: B=1 L={SEQ_L} H={SEQ_H} F=D={SEQ_FD}, "
                        f"per-head gate, {world} rank(s) x {Ls} tokens",
            "check": check,
            "exchange": "none" if world == 1 else "one NCCL all_gather of the chunk-state "
                                                  "summaries per direction",
            "fwd_ms": fwd, "fwd_tokens_per_s": SEQ_L / (fwd / 1e3),
            "fwd_bwd_ms": both, "fwd_bwd_tokens_per_s": SEQ_L / (both / 1e3),
            "fwd_bwd_ms_graph": both_graph,
            "fwd_bwd_tokens_per_s_graph": SEQ_L / (both_graph / 1e3),
            "chain": chain_res}


SEQ_CHECK_HEADS = (0, 17)
SEQ_CHECK_LIMIT = 1e-2


def seqpar_check(torch, lizard_cuda, dist, world, rank, inputs, grads):
    """Correctness of the timed sequence-parallel call at N ranks: two sampled
    heads of its output and of all four gradients (from the last timed step)
    against one single-GPU gla call over the whole sequence of those heads,
    whose inputs every rank gathers from the others. Each rank compares its
    own slice; the result is max|err| / max|ref| over every compared tensor,
    reduced as a max over ranks."""
    from lizard_cuda import seqpar
    hs = list(SEQ_CHECK_HEADS)
    fq, fk, v, lg, dy = inputs
    Ls = fq.shape[2]
    full = []
    for t in inputs:
        part = t[:, hs].contiguous()
        bufs = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(bufs, part)
        full.append(torch.cat(bufs, dim=2))
    with torch.no_grad():
        y = seqpar.gla_seqpar(fq, fk, v, lg)[:, hs]
    ref_leaves = [t.detach().clone().requires_grad_() for t in full[:4]]
    ref_y = lizard_cuda.gla(*ref_leaves)
    ref_y.backward(full[4])
    a, b = rank * Ls, (rank + 1) * Ls
    pairs = [("y", y, ref_y[:, :, a:b])]
    for name, g, r in zip(("dfq", "dfk", "dv", "dlog_gamma"), grads, ref_leaves):
        pairs.append((name, g[:, hs], r.grad[:, :, a:b]))
    worst = {}
    for name, got, ref in pairs:
        err = (got.float() - ref.float()).abs().max()
        den = ref.float().abs().max().clamp_min(1e-30)
        worst[name] = err / den
    vals = torch.stack([worst[n] for n, _, _ in pairs]).double()
    dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    per = {n: float(x) for (n, _, _), x in zip(pairs, vals.tolist())}
    mx = max(per.values())
    return {"heads": hs, "max_rel": mx, "per_tensor": per, "limit": SEQ_CHECK_LIMIT,
            "ok": mx <= SEQ_CHECK_LIMIT,
            "against": "single-GPU lizard_cuda.gla over the whole sequence of the sampled heads"}


def length_sweep(torch, lizard_cuda, device, lengths=(512, 1024, 2048, 4096, 8192, 16384),
                 steps=5, warmup=3):
    """Config 4 sweep: B=16, H=32, F=D=128, per-head gate; device ms of the
    forward (no grad) and of forward+backward at each L (inputs >= 67 MB per
    tensor; from L=1024 on every tensor is larger than L2)."""
    import torch.nn.functional as F
    out = {}
    for Lx in lengths:
        g = torch.Generator(device=device).manual_seed(99)
        shape = (16, 32, Lx, 128)
        fq = (F.softplus(torch.randn(shape, generator=g, device=device)) / math.sqrt(128)).bfloat16()
        fk = (F.softplus(torch.randn(shape, generator=g, device=device)) / math.sqrt(128)).bfloat16()
        v = torch.randn(shape, generator=g, device=device).bfloat16()
        lg = F.logsigmoid(3 + 1.5 * torch.randn(16, 32, Lx, generator=g, device=device))
        dy = torch.randn(shape, generator=g, device=device).bfloat16()
        leaves = [t.detach().requires_grad_() for t in (fq, fk, v, lg)]

        def timed(fn):
            for _ in range(warmup):
                fn()
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(steps):
                fn()
            e.record()
            torch.cuda.synchronize()
            return s.elapsed_time(e) / steps

        with torch.no_grad():
            fwd = timed(lambda: lizard_cuda.gla(fq, fk, v, lg))

        def step():
            for t in leaves:
                t.grad = None
            lizard_cuda.gla(*leaves).backward(dy)
        both = timed(step)
        tok = 16 * Lx
        out[f"L{Lx}"] = {"fwd_ms": fwd, "fwd_tokens_per_s": tok / (fwd / 1e3),
                         "fwd_bwd_ms": both, "fwd_bwd_tokens_per_s": tok / (both / 1e3)}
        del fq, fk, v, lg, dy, leaves
        torch.cuda.empty_cache()
    return out


def prologue_measure(torch, lizard_cuda, device, steps=20, warmup=3):
    """GLA prologue: the Hedgehog feature map of one projection at
    the model's head shape (B=4, H=32, L=4096, Dh=64, feature dim 128, fp32
    heads as the layer feeds them), fused kernel against the same torch ops
    (matmul, two softmaxes, concatenation, bf16 cast) on the GPU; forward and
    forward+backward device ms. Bytes moved by the fused forward: fp32 x in,
    bf16 features out."""
    Bp, Hp, Lp, Dh, Fd = 4, 32, 4096, 64, 128
    g = torch.Generator(device=device).manual_seed(11)
    x = torch.randn(Bp, Hp, Lp, Dh, generator=g, device=device)
    w = 0.05 * torch.randn(Fd, Dh, generator=g, device=device)
    df = torch.randn(Bp, Hp, Lp, 2 * Fd, generator=g, device=device).bfloat16()

    def torch_hh(xx, ww):
        xw = xx @ ww.T
        return torch.cat([xw.softmax(-1), (-xw).softmax(-1)], -1).bfloat16()

    def timed(fn):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            fn()
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / steps

    out = {"workload": f"hedgehog x [{Bp},{Hp},{Lp},{Dh}] fp32, W [{Fd},{Dh}] -> bf16 [.., {2 * Fd}]"}
    with torch.no_grad():
        out["fused_fwd_ms"] = timed(lambda: lizard_cuda.hedgehog(x, w))
        out["torch_fwd_ms"] = timed(lambda: torch_hh(x, w))
    xl, wl = x.clone().requires_grad_(), w.clone().requires_grad_()

    def fb(fn):
        def step():
            xl.grad = wl.grad = None
            fn(xl, wl).backward(df)
        return step
    out["fused_fwd_bwd_ms"] = timed(fb(lizard_cuda.hedgehog))
    out["torch_fwd_bwd_ms"] = timed(fb(torch_hh))
    rows = Bp * Hp * Lp
    out["fused_fwd_gbs"] = rows * (4 * Dh + 2 * 2 * Fd) / (out["fused_fwd_ms"] / 1e3) / 1e9
    return out


# Lizard-Llama-3.2-1B shape (config 5): the public Llama 3.2 1B architecture numbers.
LLAMA_1B = dict(hidden_size=2048, intermediate_size=8192, num_hidden_layers=16,
                num_attention_heads=32, num_key_value_heads=8, vocab_size=128256,
                rope_theta=500000.0, max_position_embeddings=131072, tie_word_embeddings=True,
                rms_norm_eps=1e-5,
                rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0,
                              "high_freq_factor": 4.0, "original_max_position_embeddings": 8192})


def prefill_flops_per_token(cfg, Lm, window=64, feature_dim=128):
    """Algorithmic flops per token of the config-5 prefill: 2 x every projection,
    MLP and logit weight (2.47 GFLOP), plus per layer and head the GLA forward
    2(2FD + CF + CD) with C = 64 (F = 2 feature_dim, D = head dim), the SWA
    forward 4 D w (w = mean window size at length Lm) and the two Hedgehog
    feature maps 2 Dh feature_dim (queries on all heads, keys on the KV heads)."""
    h, hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    d = cfg.hidden_size // h
    kv = hkv * d
    per_layer = (2 * cfg.hidden_size * cfg.hidden_size + 2 * cfg.hidden_size * kv
                 + 3 * cfg.hidden_size * cfg.intermediate_size + cfg.hidden_size)
    linear = 2 * (cfg.num_hidden_layers * per_layer + cfg.hidden_size * cfg.vocab_size)
    Fd = 2 * feature_dim
    wbar = sum(min(i + 1, window) for i in range(Lm)) / Lm
    attn = (h * 2 * (2 * Fd * d + 64 * Fd + 64 * d) + h * 4 * d * wbar
            + (h + hkv) * 2 * d * feature_dim)
    return linear + cfg.num_hidden_layers * attn


def model_prefill_measure(torch, lizard_cuda, device, Bm=32, Lm=4096, steps=3, warmup=3,
                          dist=None, world=1, decode=True):
    """Config 5: forward prefill of a random-init bf16 Lizard-Llama-3.2-1B
    (every attention layer swapped by lizard_cuda.model.to_lizard, window 64, 4 sinks,
    feature dim 128 -> F = 256, GQA 32/8 heads) on uniform random token ids, full logits.
    Device ms per step by CUDA events, tokens/s, and the same for one Lizard attention
    layer alone at the model's shape (its share of the step). With N ranks the batch is
    sharded: every rank runs Bm sequences (Bm = 32 / N from the caller), the ranks
    start together after a barrier and the step time is the max over ranks; tokens/s
    counts all ranks' tokens. The tensor roofline fraction is the whole step's
    algorithmic flops over the sustained bf16 peak (a step of several hundred ms
    runs under the power cap)."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from lizard_cuda.model import to_lizard
    cfg = LlamaConfig(**LLAMA_1B)
    torch.manual_seed(0)
    with torch.device(device):
        model = LlamaForCausalLM(cfg).to(torch.bfloat16)
    to_lizard(model, window=64, num_meta=4, feature_dim=128).eval()
    rank = dist.get_rank() if dist is not None else 0
    g = torch.Generator(device=device).manual_seed(3 + rank)
    ids = torch.randint(0, cfg.vocab_size, (Bm, Lm), generator=g, device=device)

    def timed(fn, n, w):
        for _ in range(w):
            fn()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(n):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / n], device=device, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    out = {"workload": f"Lizard-Llama-3.2-1B prefill, random-init bf16, B={Bm * world} L={Lm} "
                       f"({world} rank(s) x B={Bm}, batch sharded), uniform random ids, full "
                       "logits, window 64, 4 sinks, F=256, GQA 32/8",
           "n_gpus": world}
    with torch.no_grad():
        out["ms_per_step"] = timed(lambda: model(ids, use_cache=False).logits, steps, warmup)
        out["tokens_per_s"] = world * Bm * Lm / (out["ms_per_step"] / 1e3)
        x = torch.randn(Bm, Lm, cfg.hidden_size, generator=g, device=device).bfloat16()
        pos = torch.arange(Lm, device=device)[None].expand(Bm, Lm)
        rope = model.model.rotary_emb(x, pos)
        attn = model.model.layers[0].self_attn
        out["attention_layer_ms"] = timed(lambda: attn(x, rope), steps, warmup)
    out["attention_share"] = cfg.num_hidden_layers * out["attention_layer_ms"] / out["ms_per_step"]
    flops = prefill_flops_per_token(cfg, Lm) * Bm * Lm
    tflops = flops / (out["ms_per_step"] / 1e3) / 1e12
    sustained = measured_sustained_tflops()
    out["tensor_roofline"] = {"flops_per_step_per_gpu": flops, "tflops_per_gpu": tflops,
                              "peak_tflops": sustained[0], "peak_source": sustained[1],
                              "frac": tflops / sustained[0]}
    if decode:
        out["decode"] = decode_measure(torch, model, cfg, ids, device, steps=max(4, steps))
    del model
    torch.cuda.empty_cache()
    return out


def measured_sustained_tflops():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        if "bf16_tflops_sustained" in d:
            return float(d["bf16_tflops_sustained"]), "measured sustained (MEASURED_PEAKS.json)"
    return 1400.0, "fallback sustained 1.4 PFLOP/s"


def decode_measure(torch, model, cfg, ids, device, steps=8, warmup=2):
    """Recurrent decode of the config-5 model: the prompt ids [B, L]
    through the full forward into a LizardCache, then one greedy token per step
    for the whole batch (eager, one model call per step). Also the GLA decode
    kernel alone at the model's shape against its state traffic (the fp32 state
    and normaliser read and written once per step)."""
    from lizard_cuda.decode import LizardCache, gla_decode
    Bm, Lm = ids.shape
    out = {"workload": f"greedy decode after a {Lm}-token prompt, B={Bm}, one token per step"}
    with torch.no_grad():
        cache = LizardCache()
        tok = model(ids, lizard_cache=cache, use_cache=False,
                    logits_to_keep=1).logits[:, -1].argmax(-1, keepdim=True)
        pos = torch.full((Bm, 1), Lm, dtype=torch.long, device=device)

        def step():
            nonlocal tok
            tok = model(tok, position_ids=pos, lizard_cache=cache,
                        use_cache=False).logits[:, -1].argmax(-1, keepdim=True)
            pos.add_(1)
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            step()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / steps
        out["ms_per_step"] = ms
        out["tokens_per_s"] = Bm / (ms / 1e3)
        # the same step as one CUDA graph launch (lizard_cuda.model.GraphedDecoder)
        from lizard_cuda.model import GraphedDecoder
        dec = GraphedDecoder(model, cache, tok, pos)
        for _ in range(warmup):
            dec.step()
        torch.cuda.synchronize()
        s.record()
        for _ in range(steps):
            dec.step()
        e.record()
        torch.cuda.synchronize()
        gms = s.elapsed_time(e) / steps
        out["graph_ms_per_step"] = gms
        out["graph_tokens_per_s"] = Bm / (gms / 1e3)
        del dec
        c0 = cache[0]
        Hs, F, D = c0.state.shape[1:]
        H = cfg.num_attention_heads
        g = torch.Generator(device=device).manual_seed(9)
        fq = torch.rand(Bm, H, F, generator=g, device=device).bfloat16()
        fk = torch.rand(Bm, Hs, F, generator=g, device=device).bfloat16()
        v = torch.randn(Bm, Hs, D, generator=g, device=device).bfloat16()
        lg = -torch.rand(Bm, generator=g, device=device)
        # five state copies (5 x 34 MB > the 126 MB L2) taken in turn, so every call
        # reads its state from HBM as a layer's decode step does; 50 launches
        # replayed from one graph, so the timing sees the kernel and not the Python
        # call around it
        sts = [(c0.state.clone(), c0.zstate.clone()) for _ in range(5)]
        st, zs = sts[0]
        for _ in range(3):
            gla_decode(fq, fk, v, lg, st, zs)
        torch.cuda.synchronize()
        n = 50
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(n):
                gla_decode(fq, fk, v, lg, *sts[i % 5])
        graph.replay()
        torch.cuda.synchronize()
        s.record()
        graph.replay()
        e.record()
        torch.cuda.synchronize()
        del graph, sts
        us = s.elapsed_time(e) / n * 1e3
        state_bytes = 2 * (st.numel() + zs.numel()) * 4
        out["gla_decode_kernel_us"] = us
        out["gla_decode_state_bytes"] = state_bytes
        out["gla_decode_gbs"] = state_bytes / (us / 1e6) / 1e9
    return out


def secondary(torch, lizard_cuda, device, steps=50, warmup=5):
    """Config 3 (B=1, L=2048, H=32, F=D=64): GLA fwd+bwd with a per-token gate
    and SWA fwd+bwd (window 64, 4 sinks; also window 128, the reference's
    training setting); device ms per step.

    "ms" is eager (one Python call per step, host launch overhead included);
    "ms_graph" replays the same step captured in a CUDA graph, which shows the
    device time without the host in the way (back to back: the 8 MB inputs stay
    in L2); "ms_graph_l2_flushed" flushes L2 before every replay."""
    import torch.nn.functional as F
    g = torch.Generator(device=device).manual_seed(7)
    Bs, Hs, Ls, Ds = 1, 32, 2048, 64

    def leaf(t):
        return t.detach().requires_grad_()
    fq = leaf((F.softplus(torch.randn(Bs, Hs, Ls, Ds, generator=g, device=device)) / 8).bfloat16())
    fk = leaf((F.softplus(torch.randn(Bs, Hs, Ls, Ds, generator=g, device=device)) / 8).bfloat16())
    v = leaf(torch.randn(Bs, Hs, Ls, Ds, generator=g, device=device).bfloat16())
    lg = leaf(F.logsigmoid(3 + 1.5 * torch.randn(Bs, Ls, generator=g, device=device)))
    q = leaf(torch.randn(Bs, Hs, Ls, Ds, generator=g, device=device).bfloat16())
    k = leaf(torch.randn(Bs, Hs, Ls, Ds, generator=g, device=device).bfloat16())
    meta = leaf(torch.randn(4, generator=g, device=device))
    dy = torch.randn(Bs, Hs, Ls, Ds, generator=g, device=device).bfloat16()
    out = {}

    def timed(name, fn, leaves):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0 = lizard_cuda.launch_count()
        s.record()
        for _ in range(steps):
            for t in leaves:
                t.grad = None
            fn()
        e.record()
        torch.cuda.synchronize()
        ms = s.elapsed_time(e) / steps
        launches = (lizard_cuda.launch_count() - n0) / steps

        def step():
            for t in leaves:
                t.grad = None
            fn()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(3):
                step()
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        for _ in range(warmup):
            graph.replay()
        torch.cuda.synchronize()
        s.record()
        for _ in range(steps):
            graph.replay()
        e.record()
        torch.cuda.synchronize()
        msg = s.elapsed_time(e) / steps
        # the same replays with L2 flushed before each (a 256 MB write, untimed)
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
        tot = 0.0
        for _ in range(steps):
            flush.fill_(1)
            s.record()
            graph.replay()
            e.record()
            e.synchronize()
            tot += s.elapsed_time(e)
        del graph, flush
        msf = tot / steps
        out[name] = {"ms": ms, "tokens_per_s": Bs * Ls / (ms / 1e3), "ms_graph": msg,
                     "tokens_per_s_graph": Bs * Ls / (msg / 1e3), "ms_graph_l2_flushed": msf,
                     "launches_per_step": launches}

    timed("gla_fwd_bwd_cfg3", lambda: lizard_cuda.gla(fq, fk, v, lg).backward(dy),
          (fq, fk, v, lg))
    timed("swa_fwd_bwd_cfg3", lambda: lizard_cuda.swa(q, k, v, meta, 64).backward(dy),
          (q, k, v, meta))
    # the reference's training configs use window 128 (configs/lizard-1b*.yaml)
    timed("swa_fwd_bwd_cfg3_w128", lambda: lizard_cuda.swa(q, k, v, meta, 128).backward(dy),
          (q, k, v, meta))
    with torch.no_grad():
        timed("gla_fwd_cfg3", lambda: lizard_cuda.gla(fq, fk, v, lg), ())
        timed("swa_fwd_cfg3", lambda: lizard_cuda.swa(q, k, v, meta, 64), ())
        timed("swa_fwd_cfg3_w128", lambda: lizard_cuda.swa(q, k, v, meta, 128), ())
    return out


REF_DIR = ROOT / "baseline" / "_ref"


def median_ms(torch, fn, leaves=(), reps=20, warmup=3):
    """Median device ms of one call: CUDA events around each call, L2 flushed
    (a 256 MB write) before each, gradients of `leaves` reset; the procedure of
    the reference's own harness (triton.testing.do_bench with
    return_mode="median", src/benchmark.py:57-66), written out here so every
    implementation below is timed by the same code."""
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        for t in leaves:
            t.grad = None
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    out = []
    for _ in range(reps):
        for t in leaves:
            t.grad = None
        flush.zero_()
        s.record()
        fn()
        e.record()
        e.synchronize()
        out.append(s.elapsed_time(e))
    del flush
    return statistics.median(out)


def reference_gpu_measure(torch, lizard_cuda, device, budget_s=420.0):
    """Same-box timing of the reference's own GPU kernels: the Triton kernels.gla
    and kernels.swa of src/kernels/ (installed unmodified in baseline/_ref), JIT
    compiled here for sm_100, and flash-linear-attention's chunk_gla /
    chunk_simple_gla when the fla package imports (the comparators of
    src/benchmark.py:44-54). Every workload is timed for lizard_cuda and the
    reference on the same inputs with median_ms; `ratio` = reference ms / our ms
    (above 1: lizard_cuda is faster). Synthetic inputs with the BASELINE
    distributions; FLA takes [B, L, H, D] and computes an unnormalised GLA, so
    it is a speed comparator only."""
    import torch.nn.functional as F
    if not (REF_DIR / "kernels" / "__init__.py").exists():
        return {"unavailable": "baseline/_ref/kernels is not installed"}
    sys.path.insert(0, str(REF_DIR))
    try:
        import kernels as ref_kernels  # the reference's src/kernels package
    except Exception as exc:  # noqa: BLE001 - report why the comparator is missing
        return {"unavailable": f"import of the reference kernels failed: {exc!r}"}
    try:
        from fla.ops.gla import chunk_gla
        from fla.ops.simple_gla import chunk_simple_gla
    except Exception as exc:  # noqa: BLE001
        chunk_gla = chunk_simple_gla = None
        fla_note = f"fla not importable: {exc!r}"
    else:
        fla_note = "fla-core chunk_gla / chunk_simple_gla, scale 1.0"
    t_start = time.perf_counter()
    g = torch.Generator(device=device).manual_seed(77)

    def feats(*shape):
        return (F.softplus(torch.randn(shape, generator=g, device=device))
                / math.sqrt(shape[-1])).bfloat16()

    def gate(*shape):
        return F.logsigmoid(3 + 1.5 * torch.randn(shape, generator=g, device=device))

    out = {"harness": "median of per-call CUDA events, L2 flushed before each call, "
                      "20 calls after 3 warm-ups",
           "fla": fla_note, "workloads": {}}

    def record(name, desc, ours_fn, ref_fn, leaves_ours=(), leaves_ref=(), fla=None):
        if time.perf_counter() - t_start > budget_s:
            out["workloads"][name] = {"skipped": f"time budget of {budget_s:.0f} s spent"}
            return
        row = {"workload": desc}
        row["ours_ms"] = median_ms(torch, ours_fn, leaves_ours)
        try:
            row["reference_triton_ms"] = median_ms(torch, ref_fn, leaves_ref)
            row["ratio"] = row["reference_triton_ms"] / row["ours_ms"]
        except Exception as exc:  # noqa: BLE001 - e.g. out of memory in the reference
            row["reference_triton_ms"] = None
            row["reference_error"] = repr(exc)[:200]
        if fla is not None:
            for key, fn in fla.items():
                try:
                    row[key] = median_ms(torch, fn)
                except Exception as exc:  # noqa: BLE001
                    row[key] = None
                    row[key + "_error"] = repr(exc)[:200]
        out["workloads"][name] = row
        torch.cuda.empty_cache()

    def gla_case(name, Bc, Hc, Lc, FDc, per_head, train, with_fla=False):
        fq, fk = feats(Bc, Hc, Lc, FDc), feats(Bc, Hc, Lc, FDc)
        v = torch.randn(Bc, Hc, Lc, FDc, generator=g, device=device).bfloat16()
        lg = gate(Bc, Hc, Lc) if per_head else gate(Bc, Lc)
        desc = (f"gla {'fwd+bwd' if train else 'fwd'} B={Bc} H={Hc} L={Lc} F=D={FDc}, "
                f"{'per-head' if per_head else 'per-token'} gate")
        fla = None
        if with_fla and chunk_gla is not None and not train:
            qf, kf, vf = (t.transpose(1, 2).contiguous() for t in (fq, fk, v))
            gf = lg.transpose(1, 2).contiguous() if per_head else lg
            ge = gf[..., None].expand(*qf.shape).contiguous()
            fla = {"fla_chunk_gla_ms": lambda: chunk_gla(qf, kf, vf, ge, scale=1.0)[0],
                   "fla_chunk_simple_gla_ms": lambda: chunk_simple_gla(qf, kf, vf, gf,
                                                                      scale=1.0)[0]}
        if not train:
            def ours():
                with torch.no_grad():
                    lizard_cuda.gla(fq, fk, v, lg)

            def ref():
                with torch.no_grad():
                    ref_kernels.gla(fq, fk, v, lg)
            record(name, desc, ours, ref, fla=fla)
            return
        dy = torch.randn(Bc, Hc, Lc, FDc, generator=g, device=device).bfloat16()
        lo = [t.detach().clone().requires_grad_() for t in (fq, fk, v, lg)]
        lr = [t.detach().clone().requires_grad_() for t in (fq, fk, v, lg)]
        record(name, desc, lambda: lizard_cuda.gla(*lo).backward(dy),
               lambda: ref_kernels.gla(*lr).backward(dy), lo, lr)

    gla_case("cfg2_fwd", 8, 32, 2048, 128, True, False, with_fla=True)
    gla_case("cfg3_gla_fwd_bwd", 1, 32, 2048, 64, False, True)
    gla_case("cfg3_gla_fwd", 1, 32, 2048, 64, False, False)
    # config 3 SWA on the same shape: window 64, 4 sinks
    q, k = (torch.randn(1, 32, 2048, 64, generator=g, device=device).bfloat16()
            for _ in range(2))
    v = torch.randn(1, 32, 2048, 64, generator=g, device=device).bfloat16()
    meta = torch.randn(4, generator=g, device=device)
    dy = torch.randn(1, 32, 2048, 64, generator=g, device=device).bfloat16()
    lo = [t.detach().clone().requires_grad_() for t in (q, k, v, meta)]
    lr = [t.detach().clone().requires_grad_() for t in (q, k, v, meta)]
    record("cfg3_swa_fwd_bwd", "swa fwd+bwd B=1 H=32 L=2048 D=64, window 64, 4 sinks",
           lambda: lizard_cuda.swa(*lo, 64).backward(dy),
           lambda: ref_kernels.swa(*lr, 64).backward(dy), lo, lr)

    def swa_fwd_ours():
        with torch.no_grad():
            lizard_cuda.swa(q, k, v, meta, 64)

    def swa_fwd_ref():
        with torch.no_grad():
            ref_kernels.swa(q, k, v, meta, 64)
    record("cfg3_swa_fwd", "swa fwd B=1 H=32 L=2048 D=64, window 64, 4 sinks",
           swa_fwd_ours, swa_fwd_ref)
    # window 128, the reference's training configs (configs/lizard-1b*.yaml)
    record("cfg3_swa_w128_fwd_bwd", "swa fwd+bwd B=1 H=32 L=2048 D=64, window 128, 4 sinks",
           lambda: lizard_cuda.swa(*lo, 128).backward(dy),
           lambda: ref_kernels.swa(*lr, 128).backward(dy), lo, lr)

    def swa128_fwd_ours():
        with torch.no_grad():
            lizard_cuda.swa(q, k, v, meta, 128)

    def swa128_fwd_ref():
        with torch.no_grad():
            ref_kernels.swa(q, k, v, meta, 128)
    record("cfg3_swa_w128_fwd", "swa fwd B=1 H=32 L=2048 D=64, window 128, 4 sinks",
           swa128_fwd_ours, swa128_fwd_ref)
    del q, k, v, meta, dy, lo, lr
    gla_case("cfg4_L2048_fwd_bwd", 16, 32, 2048, 128, True, True)
    gla_case("cfg4_L8192_fwd_bwd", 16, 32, 8192, 128, True, True)
    # the reference's own Table-3 forward shapes (src/benchmark.py:8-9), H=32, D=128
    for Bt, Lt in ((16, 2048), (16, 4096), (16, 8192), (32, 8192)):
        gla_case(f"table3_B{Bt}_L{Lt}_fwd", Bt, 32, Lt, 128, True, False, with_fla=True)
    out["seconds"] = time.perf_counter() - t_start
    return out


def run_ours(args, torch):
    import lizard_cuda
    rank, local, world = env_rank()
    if args.gpus != world:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=device)
    lizard_cuda.load()

    def barrier():
        if dist is not None:
            dist.barrier()

    fq, fk, v, lg = make_inputs(torch, device, seed=1234 + rank)
    stream = torch.cuda.current_stream(device)
    sampler = ClockSampler(physical_gpu(local)) if rank == 0 else None
    with torch.no_grad():
        for _ in range(args.warmup):
            lizard_cuda.gla(fq, fk, v, lg)
        # untimed soak of about one second so the clock sampler sees the load
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < 1.0:
            for _ in range(20):
                lizard_cuda.gla(fq, fk, v, lg)
            torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0 = lizard_cuda.launch_count()
        start.record(stream)
        for _ in range(args.steps):
            y = lizard_cuda.gla(fq, fk, v, lg)
        end.record(stream)
        torch.cuda.synchronize()
        launches = lizard_cuda.launch_count() - n0
        barrier()
    clocks = sampler.stop() if sampler else None
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    del y

    # end to end through the public API: every step copies its inputs from pinned host
    # memory and its output back. Inputs and outputs are double-buffered: the inputs
    # go up on one stream, y comes back on another, so step n + 1's host-to-device
    # copy overlaps step n's compute and device-to-host copy (the two directions
    # use separate copy engines).
    host = [x.cpu().pin_memory() for x in (fq, fk, v, lg)]
    y_host = [torch.empty(B, H, L, D, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    dev_in = [[torch.empty_like(x) for x in (fq, fk, v, lg)] for _ in range(2)]
    h2d = sum(x.numel() * x.element_size() for x in host)
    d2h = y_host[0].numel() * y_host[0].element_size()
    e2e_steps = max(3, min(args.steps, 50))
    up, down = torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]
    ev_y = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(i):
        k = i % 2
        with torch.cuda.stream(up):
            up.wait_event(ev_free[k])  # step i - 2 has read this input buffer
            for dst, src in zip(dev_in[k], host):
                dst.copy_(src, non_blocking=True)
            ev_in[k].record(up)
        stream.wait_event(ev_in[k])
        y = lizard_cuda.gla(*dev_in[k])
        ev_free[k].record(stream)
        ev_y[k].record(stream)
        with torch.cuda.stream(down):
            down.wait_event(ev_y[k])
            y_host[k].copy_(y, non_blocking=True)
            y.record_stream(down)

    with torch.no_grad():
        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(stream)
        up.wait_event(s2)
        for i in range(e2e_steps):
            e2e_step(i)
        stream.wait_stream(down)
        e2.record(stream)
        torch.cuda.synchronize()
        barrier()
    t2 = torch.tensor([s2.elapsed_time(e2)], device=device, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t2, op=dist.ReduceOp.MAX)
    e2e_ms = float(t2.item())

    side = None
    seq = None
    if not args.no_secondary:
        seq = seqpar_measure(torch, lizard_cuda, device, dist, world, rank)
        model = None
        if 32 % world == 0:  # config 5, batch sharded over every rank
            model = model_prefill_measure(torch, lizard_cuda, device, Bm=32 // world,
                                          dist=dist, world=world, decode=(world == 1))
        if rank == 0:
            side = secondary(torch, lizard_cuda, device)
            side["cfg5_model_prefill"] = model
            if world == 1:
                side["cfg4_length_sweep"] = length_sweep(torch, lizard_cuda, device)
                side["prologue_hedgehog"] = prologue_measure(torch, lizard_cuda, device)
                side["reference_gpu"] = reference_gpu_measure(torch, lizard_cuda, device)

    cpu = None
    if rank == 0 and world == 1:
        rate, runs, dt = cpu_oracle_rate(torch, fq, fk, v, lg, H, 10.0)
        cpu = {"value": rate, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"dense fp32 torch oracle, batch row 0 (32 heads x {L} tokens) of the "
                         f"config-2 workload, {runs} runs in {dt:.1f} s"}

    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    hbm_peak, tc_peak, src = measured_peaks()
    tokens_per_step = B * L * world
    ms_step = ms_max / args.steps
    kernel_ms = ms / max(1, launches)  # rank 0: one forward launch per step
    alg_bytes = B * H * L * BYTES_PER_TOKEN_HEAD
    alg_flops = B * H * L * FLOPS_PER_TOKEN_HEAD
    achieved = alg_bytes / (kernel_ms / 1e3) / 1e9
    traffic = profiled_traffic()
    line = {
        "metric": METRIC,
        "value": tokens_per_step * args.steps / (ms_max / 1e3),
        "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": dict(CONFIG, parallelism=f"dp{world} (batch*head shards, no collective)"),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "traffic": traffic,
                     "peak_source": f"{src} (MEASURED_PEAKS.json hbm_gbs)" if src == "measured"
                     else "fallback 6.65 TB/s",
                     "alg_bytes_per_launch": alg_bytes,
                     "tensor_tflops": alg_flops / (kernel_ms / 1e3) / 1e12,
                     "tensor_frac": alg_flops / (kernel_ms / 1e3) / 1e12 / tc_peak},
        "e2e": {"value": tokens_per_step * e2e_steps / (e2e_ms / 1e3), "unit": UNIT,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": e2e_steps},
        "gpu_launches": launches,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    if side:
        line["secondary"] = side
    if seq:
        line["seqpar"] = seq
    print(json.dumps(line), flush=True)
    if seq and seq.get("check") and not seq["check"]["ok"]:
        raise SystemExit(f"sequence-parallel check failed: max_rel {seq['check']['max_rel']:.3e} "
                         f"> {SEQ_CHECK_LIMIT}")


def run_case(args, torch):
    """One named workload, K steps after W warm-up steps, device time by CUDA events."""
    import torch.nn.functional as F
    import lizard_cuda
    lizard_cuda.load()
    name = args.case
    Bc, Hc, Lc, FDc, per_head, train, op = CASES[name]
    Bc, Lc = args.B or Bc, args.L or Lc
    if op == "seqpar":  # launched like the main bench: torchrun for N > 1
        rank, local, world = env_rank()
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        dist = None
        if world > 1:
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        res = seqpar_measure(torch, lizard_cuda, dev, dist, world, rank,
                             steps=max(1, args.steps), warmup=args.warmup)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"case": name, "n_gpus": world, **res}), flush=True)
            if res.get("check") and not res["check"]["ok"]:
                raise SystemExit("sequence-parallel check failed")
        return
    dev = torch.device("cuda", 0)
    if op == "model":
        res = model_prefill_measure(torch, lizard_cuda, dev, Bc, Lc, max(1, args.steps),
                                    args.warmup)
        print(json.dumps({"case": name, "B": Bc, "L": Lc, **res}), flush=True)
        return
    if op == "reference_gpu":
        res = reference_gpu_measure(torch, lizard_cuda, dev)
        print(json.dumps({"case": name, **res}), flush=True)
        return
    from lizard_cuda import _lib
    _lib.set_schedule(args.schedule)
    g = torch.Generator(device=dev).manual_seed(5)
    shape = (Bc, Hc, Lc, FDc)
    a = (F.softplus(torch.randn(shape, generator=g, device=dev)) / math.sqrt(FDc)).bfloat16()
    b = (F.softplus(torch.randn(shape, generator=g, device=dev)) / math.sqrt(FDc)).bfloat16()
    v = torch.randn(shape, generator=g, device=dev).bfloat16()
    lg = F.logsigmoid(3 + 1.5 * torch.randn((Bc, Hc, Lc) if per_head else (Bc, Lc),
                                            generator=g, device=dev))
    meta = torch.randn(4, generator=g, device=dev)
    dy = torch.randn(shape, generator=g, device=dev).bfloat16()
    if op == "gla":
        args_in = [a, b, v, lg]
        call = lizard_cuda.gla
    elif op == "gla_gqa":  # config-5 GLA: D = 64 values, 8 key/value heads, per-token gate
        Hkv, Dv = 8, 64
        fk = (F.softplus(torch.randn(Bc, Hkv, Lc, FDc, generator=g, device=dev))
              / math.sqrt(FDc)).bfloat16()
        vv = torch.randn(Bc, Hkv, Lc, Dv, generator=g, device=dev).bfloat16()
        args_in = [a, fk, vv, lg]
        call = lizard_cuda.gla
        dy = torch.randn(Bc, Hc, Lc, Dv, generator=g, device=dev).bfloat16()
    elif op == "hedgehog_bf16":
        xp = torch.randn(Bc, Lc, Hc * FDc, generator=g, device=dev).bfloat16()
        args_in = [xp.view(Bc, Lc, Hc, FDc).transpose(1, 2),
                   0.05 * torch.randn(128, FDc, generator=g, device=dev)]
        call = lizard_cuda.hedgehog
    elif op == "blend":
        args_in = [torch.randn(shape, generator=g, device=dev).bfloat16(),
                   torch.randn(shape, generator=g, device=dev).bfloat16(),
                   torch.tensor(0.7, device=dev)]
        call = lambda a_, b_, al: lizard_cuda.blend(a_, b_, al, torch.bfloat16)  # noqa: E731
    elif op == "decode":
        from lizard_cuda.decode import gla_decode, swa_decode
        Hkv, Dv, W = 8, 64, 64
        st = torch.zeros(Bc, Hkv, FDc, Dv, device=dev)
        zs = torch.zeros(Bc, Hkv, FDc, device=dev)
        kr = torch.zeros(Bc, Hkv, W, Dv, device=dev)
        vr = torch.zeros_like(kr)
        pos = torch.full((Bc,), Lc, dtype=torch.int32, device=dev)
        fq1 = torch.rand(Bc, Hc, FDc, generator=g, device=dev).bfloat16()
        fk1 = torch.rand(Bc, Hkv, FDc, generator=g, device=dev).bfloat16()
        q1 = torch.randn(Bc, Hc, Dv, generator=g, device=dev).bfloat16()
        k1 = torch.randn(Bc, Hkv, Dv, generator=g, device=dev).bfloat16()
        v1 = torch.randn(Bc, Hkv, Dv, generator=g, device=dev).bfloat16()
        c1 = torch.ones(1, Dv, device=dev)
        s1 = torch.zeros(1, Dv, device=dev)
        lg1 = -torch.rand(Bc, generator=g, device=dev)
        args_in = []

        def call():
            gla_decode(fq1, fk1, v1, lg1, st, zs)
            swa_decode(q1, k1, v1, c1, s1, meta, kr, vr, pos)
    elif op == "swa_rope":  # projections [B, L, heads * 64] read in place as heads
        Hkv = 8
        qp = torch.randn(Bc, Lc, Hc * FDc, generator=g, device=dev).bfloat16()
        kp = torch.randn(Bc, Lc, Hkv * FDc, generator=g, device=dev).bfloat16()
        vp = torch.randn(Bc, Lc, Hkv * FDc, generator=g, device=dev).bfloat16()
        inv = 1.0 / (5e5 ** (torch.arange(0, FDc, 2, device=dev).float() / FDc))
        ang = torch.arange(Lc, device=dev).float()[:, None] * inv
        emb = torch.cat([ang, ang], -1)[None]
        cos, sin = emb.cos().bfloat16(), emb.sin().bfloat16()
        args_in = [qp.view(Bc, Lc, Hc, FDc).transpose(1, 2),
                   kp.view(Bc, Lc, Hkv, FDc).transpose(1, 2),
                   vp.view(Bc, Lc, Hkv, FDc).transpose(1, 2), meta]
        call = lambda q, k, vv_, m: lizard_cuda.swa_rope(q, k, vv_, cos, sin, m, 64)  # noqa: E731
    elif op == "hedgehog":
        args_in = [torch.randn(shape, generator=g, device=dev),
                   0.05 * torch.randn(128, FDc, generator=g, device=dev)]
        call = lizard_cuda.hedgehog
        dy = torch.randn(Bc, Hc, Lc, 256, generator=g, device=dev).bfloat16()
    else:
        args_in = [torch.randn(shape, generator=g, device=dev).bfloat16(),
                   torch.randn(shape, generator=g, device=dev).bfloat16(), v, meta]
        call = lambda q, k, vv, m: lizard_cuda.swa(q, k, vv, m, args.window)  # noqa: E731
    leaves = [t.detach().requires_grad_() for t in args_in] if train else args_in

    def step():
        if train:
            for t in leaves:
                t.grad = None
            call(*leaves).backward(dy)
        else:
            with torch.no_grad():
                call(*leaves)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        step()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / max(1, args.steps)
    print(json.dumps({"case": name, "B": Bc, "H": Hc, "L": Lc, "F=D": FDc, "train": train,
                      "steps": args.steps, "ms_per_step": ms}), flush=True)


def main():
    args = parse()
    import torch
    if args.case:
        run_case(args, torch)
        return
    if args.impl == "reference":
        run_reference(args, torch)
    else:
        run_ours(args, torch)


if __name__ == "__main__":
    main()
