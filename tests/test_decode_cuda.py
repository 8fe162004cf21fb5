"""Recurrent decode (one token at a time against a cached state) against the
full-sequence results: the CPU oracle's dense attention (the reference's
torch backend restated) at every decoded position, the layer's own full
forward, and a small Lizard-Llama's logits."""
import copy
from types import SimpleNamespace

import pytest
import torch

import lizard_oracle as orc
from parity import assert_output

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib(built_lib):
    import lizard_cuda
    lizard_cuda.load()


def _rep(x, grp):
    return x.repeat_interleave(grp, dim=1)


@pytest.mark.parametrize("B,H,Hkv,F,D,L0,T,per_head", [
    (2, 4, 2, 64, 64, 100, 40, False),   # shared gate: Hkv states for 4 query heads
    (1, 4, 4, 256, 64, 0, 30, False),    # from an empty state, the model's F = 256
    (2, 4, 2, 32, 48, 70, 20, True),     # per-head gate: one state per query head
    (1, 8, 1, 128, 128, 129, 16, False),  # 8 query heads on one state
])
def test_gla_decode_matches_dense_oracle(B, H, Hkv, F, D, L0, T, per_head):
    from lizard_cuda.decode import gla_decode, gla_state
    g = torch.Generator(device=DEV).manual_seed(L0 + T + F)
    L = L0 + T
    sp = torch.nn.functional.softplus
    fq = (sp(torch.randn(B, H, L, F, generator=g, device=DEV)) / F ** 0.5).bfloat16()
    fk = (sp(torch.randn(B, Hkv, L, F, generator=g, device=DEV)) / F ** 0.5).bfloat16()
    v = torch.randn(B, Hkv, L, D, generator=g, device=DEV).bfloat16()
    lg = torch.nn.functional.logsigmoid(
        3 + 1.5 * torch.randn(*((B, H, L) if per_head else (B, L)), generator=g, device=DEV))
    Hs = H if per_head else Hkv
    if L0:
        sfk, sv = (_rep(fk[:, :, :L0], H // Hkv), _rep(v[:, :, :L0], H // Hkv)) if per_head \
            else (fk[:, :, :L0], v[:, :, :L0])
        state, zstate = gla_state(sfk, sv, lg[..., :L0])
    else:
        state = torch.zeros(B, Hs, F, D, device=DEV)
        zstate = torch.zeros(B, Hs, F, device=DEV)
    ys = [gla_decode(fq[:, :, t], fk[:, :, t], v[:, :, t], lg[..., t], state, zstate)
          for t in range(L0, L)]
    got = torch.stack(ys, 2)
    ref = orc.gla(fq.double().cpu(), _rep(fk, H // Hkv).double().cpu(),
                  _rep(v, H // Hkv).double().cpu(), lg.double().cpu())[:, :, L0:]
    assert_output(got, ref.float(), f"gla decode {B},{H},{Hkv},{F},{D},{L0},{T}")


@pytest.mark.parametrize("H,Hkv,W,L0,T,dtype,D", [
    (4, 2, 16, 40, 30, torch.float32, 64),
    (4, 4, 64, 10, 70, torch.bfloat16, 64),   # the ring fills during the decode
    (6, 2, 8, 0, 20, torch.float32, 64),
    (4, 1, 5, 3, 12, torch.float32, 32),      # odd window: ring rows staged in shared memory
    (2, 2, 24, 30, 6, torch.bfloat16, 128),
    (8, 2, 512, 520, 8, torch.bfloat16, 64),  # rings too large to stage: read from HBM
    (4, 1, 1024, 1030, 4, torch.bfloat16, 64),  # the largest window the decode step takes
])
def test_swa_decode_matches_dense_oracle(H, Hkv, W, L0, T, dtype, D):
    from lizard_cuda.decode import swa_decode, swa_ring
    g = torch.Generator(device=DEV).manual_seed(W + T)
    B, L = 2, L0 + T
    q = torch.randn(B, H, L, D, generator=g, device=DEV).to(dtype)
    k = torch.randn(B, Hkv, L, D, generator=g, device=DEV).to(dtype)
    v = torch.randn(B, Hkv, L, D, generator=g, device=DEV).to(dtype)
    meta = torch.randn(4, generator=g, device=DEV)
    cos, sin = (t.to(DEV).expand(B, L, D) for t in orc.rotary_tables(L, D, 5e5))
    if L0:
        k_ring, v_ring = swa_ring(k[:, :, :L0], v[:, :, :L0], cos[:, :L0], sin[:, :L0], W)
    else:
        k_ring = torch.zeros(B, Hkv, W, D, device=DEV)
        v_ring = torch.zeros_like(k_ring)
    pos = torch.full((B,), L0, dtype=torch.int32, device=DEV)
    ys = []
    for t in range(L0, L):
        ys.append(swa_decode(q[:, :, t], k[:, :, t], v[:, :, t], cos[:, t], sin[:, t], meta,
                             k_ring, v_ring, pos))
        pos += 1
    got = torch.stack(ys, 2)
    c, s = cos.cpu(), sin.cpu()
    qr, kr = orc.rope(q.double().cpu(), c.double(), s.double()), \
        orc.rope(k.double().cpu(), c.double(), s.double())
    ref = orc.awa(qr, _rep(kr, H // Hkv), _rep(v.double().cpu(), H // Hkv), meta.double().cpu(),
                  W)[:, :, L0:]
    assert_output(got, ref.float(), f"swa decode {H},{Hkv},{W},{L0},{T}")


def _layer(hidden=256, heads=4, kv=2, window=16, feature_dim=32, dtype=torch.bfloat16):
    from lizard_cuda.layer import LizardAttention
    cfg = SimpleNamespace(hidden_size=hidden, num_attention_heads=heads, num_key_value_heads=kv)
    torch.manual_seed(0)
    layer = LizardAttention(cfg, 0, window=window, num_meta=4, feature_dim=feature_dim)
    with torch.no_grad():
        for p in layer.parameters():
            p.normal_(0, 0.3)
    return layer.to(DEV).to(dtype)


def _rope(B, L, D):
    cos, sin = orc.rotary_tables(L, D, 5e5)
    return cos.to(DEV).expand(B, L, D), sin.to(DEV).expand(B, L, D)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_layer_decode_matches_full_forward(dtype):
    from lizard_cuda.decode import LizardCache
    layer = _layer(dtype=dtype)
    B, L0, T = 2, 50, 25
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(B, L0 + T, 256, generator=g, device=DEV).to(dtype)
    cos, sin = _rope(B, L0 + T, 64)
    with torch.no_grad():
        full = layer(x, (cos, sin))[0]
        cache = LizardCache()
        pre = layer(x[:, :L0], (cos[:, :L0], sin[:, :L0]), lizard_cache=cache)[0]
        steps = [layer(x[:, t:t + 1], (cos[:, t:t + 1], sin[:, t:t + 1]), lizard_cache=cache)[0]
                 for t in range(L0, L0 + T - 5)]
        # several tokens in one call decode one at a time
        steps.append(layer(x[:, L0 + T - 5:], (cos[:, L0 + T - 5:], sin[:, L0 + T - 5:]),
                           lizard_cache=cache)[0])
    assert_output(pre, full[:, :L0], f"layer prefill {dtype}", layer=True)
    got = torch.cat(steps, 1)
    assert_output(got, full[:, L0:], f"layer decode {dtype}", layer=True)
    assert int(cache[0].pos[0]) == L0 + T
    # and against the dense oracle layer (the reference's torch backend) in the
    # layer's dtype: a bf16 layer rounds its projections to bf16 as the
    # reference's does, an fp32 one is compared with float64
    odt = torch.float64 if dtype == torch.float32 else dtype
    dense = orc.LizardAttention(256, 4, 2, window=16, num_meta=4, feature_dim=32).to(odt)
    dense.load_state_dict({k: t.to(odt).cpu() for k, t in layer.state_dict().items()})
    with torch.no_grad():
        ref = dense(x.to(odt).cpu(), (cos.to(odt).cpu(), sin.to(odt).cpu()))[0][:, L0:]
    assert_output(got, ref.float(), f"layer decode vs oracle {dtype}", layer=True)


def test_model_decode_logits_match_full_forward():
    from test_model import tiny_llama
    from lizard_cuda.decode import LizardCache
    from lizard_cuda.model import greedy_generate, to_lizard
    model = to_lizard(tiny_llama(layers=2), window=16, num_meta=4, feature_dim=16)
    torch.manual_seed(1)
    with torch.no_grad():
        for block in model.model.layers:
            for n, p in block.self_attn.named_parameters():
                if not n.endswith("proj.weight"):
                    p.normal_(0, 0.3)
    model = model.to(DEV).eval()
    B, L0, T = 2, 40, 12
    ids = torch.randint(0, 97, (B, L0 + T), generator=torch.Generator().manual_seed(2)).to(DEV)
    with torch.no_grad():
        full = model(ids, use_cache=False).logits
        cache = LizardCache()
        model(ids[:, :L0], lizard_cache=cache, use_cache=False)
        got = []
        for t in range(L0, L0 + T):
            pos = torch.full((B, 1), t, dtype=torch.long, device=DEV)
            got.append(model(ids[:, t:t + 1], position_ids=pos, lizard_cache=cache,
                             use_cache=False).logits)
    assert_output(torch.cat(got, 1), full[:, L0:], "model decode logits", layer=True)
    toks, cache2 = greedy_generate(model, ids[:, :L0], 6)
    assert toks.shape == (B, 6) and int(cache2[0].pos[0]) == L0 + 5
    with torch.no_grad():  # the first generated token is the prompt's argmax
        assert torch.equal(toks[:, 0], full[:, L0 - 1].argmax(-1))
    # a decode step replayed from a CUDA graph runs the same kernels on the same data
    gtoks, gcache = greedy_generate(model, ids[:, :L0], 6, graph=True)
    assert torch.equal(gtoks, toks)
    assert torch.equal(gcache[1].state, cache2[1].state)
