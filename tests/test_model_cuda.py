"""A small Lizard-Llama on the cuda backend against the same model with the
oracle's dense layer (the reference's torch backend restated): logits and the
gradients of every Lizard parameter after a backward through the whole model."""
import copy

import pytest
import torch

import lizard_oracle as orc
from parity import assert_grad, assert_output

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_check_kernels_on_the_gpu(built_lib):
    from types import SimpleNamespace
    from lizard_cuda.model import check_kernels
    msg = check_kernels(None, SimpleNamespace(lizard=SimpleNamespace(backend="cuda")))
    assert msg.startswith("lizard_cuda ABI 3 on ")


def test_lizard_llama_matches_dense_oracle_model(built_lib):
    from test_model import tiny_llama
    from lizard_cuda.model import to_lizard
    base = tiny_llama(layers=2)
    ours = to_lizard(copy.deepcopy(base), window=16, num_meta=4, feature_dim=16)
    torch.manual_seed(1)
    with torch.no_grad():  # non-trivial gates, sinks and blend (the init makes them constant)
        for block in ours.model.layers:
            a = block.self_attn
            a.W_gamma.weight.normal_(0, 0.3)
            a.meta_tokens.normal_(0, 1.0)
            a.alpha_blend.fill_(0.7)
            a.phi_q.weight.normal_(0, 0.3)
            a.phi_k.weight.normal_(0, 0.3)
    ref = copy.deepcopy(base)
    cfg = base.config
    for block, mine in zip(ref.model.layers, ours.model.layers):
        dense = orc.LizardAttention(cfg.hidden_size, cfg.num_attention_heads,
                                    cfg.num_key_value_heads, window=16, num_meta=4,
                                    feature_dim=16)
        dense.load_state_dict(mine.self_attn.state_dict())
        block.self_attn = dense
    ours, ref = ours.to(DEV), ref.double()
    ids = torch.randint(0, cfg.vocab_size, (2, 96), generator=torch.Generator().manual_seed(2))
    out = ours(ids.to(DEV), use_cache=False).logits
    rout = ref(ids, use_cache=False).logits
    assert_output(out, rout.float(), "model logits", layer=True)
    g = torch.randn(out.shape, generator=torch.Generator().manual_seed(3))
    out.backward(g.to(DEV))
    rout.backward(g.double())
    names = ("phi_q.weight", "phi_k.weight", "W_gamma.weight", "meta_tokens", "alpha_blend",
             "q_proj.weight", "k_proj.weight", "v_proj.weight")
    for i, (mb, rb) in enumerate(zip(ours.model.layers, ref.model.layers)):
        mp, rp = dict(mb.self_attn.named_parameters()), dict(rb.self_attn.named_parameters())
        for n in names:
            assert_grad(mp[n].grad.float(), rp[n].grad.float(), f"layer {i} d{n}")
