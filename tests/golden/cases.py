"""Seeded input builders shared by make_golden.py and the tests.

Each builder returns a dict of CPU tensors. Shapes and distributions follow the
reference's own kernel tests (tests/test_kernels.py:45-52, 73-76, 137-148 of
mahdikhashan/lizard-reproduction) and BASELINE config 1 (a single Lizard layer,
B=1, L=256, hidden 256, 4 heads, window 64, 4 sinks, RoPE base 5e5).
"""
import torch
import torch.nn.functional as F

BF = torch.bfloat16


def gla_case(length, gates=(), shift=0.0, batch=2, heads=3, features=24, dim=20, seed=0):
    """tests/test_kernels.py:45-52: softmax features, N(0,1) values, z = 2N + shift."""
    torch.manual_seed(seed)
    fq = torch.randn(batch, heads, length, features).softmax(-1).to(BF)
    fk = torch.randn(batch, heads, length, features).softmax(-1).to(BF)
    v = torch.randn(batch, heads, length, dim).to(BF)
    z = 2 * torch.randn(batch, *gates, length) + shift
    dy = torch.randn(batch, heads, length, dim)
    return dict(fq=fq, fk=fk, v=v, log_gamma=F.logsigmoid(z), dy=dy)


def swa_case(length, batch=2, heads=3, dim=20, sinks=4, seed=0):
    """tests/test_kernels.py:73-76: N(0,1) bf16 q, k, v and N(0,1) sinks."""
    torch.manual_seed(seed)
    q, k, v = (torch.randn(batch, heads, length, dim).to(BF) for _ in range(3))
    meta = torch.randn(sinks)
    dy = torch.randn(batch, heads, length, dim)
    return dict(q=q, k=k, v=v, meta=meta, dy=dy)


# name -> (builder, kwargs); SWA cases also carry the window
GLA_CASES = {
    "gla_L1": dict(length=1),
    "gla_L77": dict(length=77),
    "gla_L150": dict(length=150),
    "gla_perhead_L100": dict(length=100, gates=(3,)),
    "gla_strong_L200": dict(length=200, shift=-6.0),
    "gla_F64_D64_L130": dict(length=130, features=64, dim=64, heads=2),
}

SWA_CASES = {
    "swa_L1_W8": (dict(length=1), 8),
    "swa_L77_W32": (dict(length=77), 32),
    "swa_L150_W128": (dict(length=150), 128),
    "swa_L130_D64_W64": (dict(length=130, dim=64, heads=2), 64),
    "swa_nosink_L40_W16": (dict(length=40, sinks=0), 16),
}

# Layer cases: hidden, heads, kv_heads, window, num_meta, feature_dim, rope theta,
# batch, length, init ("perturb" = every parameter N(0, 0.3) as in
# tests/test_kernels.py:140-142; "cfg1" = the layer's own init with a random
# gate projection and random sinks so gates and sinks are not constant).
LAYER_CASES = {
    "layer_tiny": dict(hidden=128, heads=4, kv_heads=2, window=16, num_meta=4,
                       feature_dim=8, theta=10000.0, batch=2, length=40, init="perturb"),
    "layer_cfg1": dict(hidden=256, heads=4, kv_heads=4, window=64, num_meta=4,
                       feature_dim=128, theta=500000.0, batch=1, length=256, init="cfg1"),
}


def init_layer_params(layer, init, seed=0):
    """Deterministic parameter init for a layer whose parameters are named like
    the reference's LizardAttention (src/lizard_attention.py:60-68)."""
    torch.manual_seed(seed)
    with torch.no_grad():
        if init == "perturb":
            for _, p in sorted(layer.named_parameters()):
                p.normal_(0, 0.3)
        else:
            hidden = layer.q_proj.weight.shape[1]
            for name in ("q_proj", "k_proj", "v_proj", "o_proj"):
                w = getattr(layer, name).weight
                w.normal_(0, hidden ** -0.5)
            layer.phi_q.weight.normal_(0, 0.02 * 8)
            layer.phi_k.weight.normal_(0, 0.02 * 8)
            layer.W_gamma.weight.normal_(0, 3.0 * hidden ** -0.5)
            layer.meta_tokens.normal_(0, 1.0)
            layer.alpha_blend.fill_(0.7)


def layer_inputs(case, seed=1):
    torch.manual_seed(seed)
    x = torch.randn(case["batch"], case["length"], case["hidden"])
    grad = torch.randn(case["batch"], case["length"], case["hidden"])
    return x, grad


def checksum(t):
    t = t.detach().double()
    return torch.tensor([t.sum().item(), t.abs().sum().item(), (t * t).sum().item()],
                        dtype=torch.float64)
