"""Model-level integration on the CPU: to_lizard swaps every block's attention
(src/train.py:35-39) and check_kernels reports the backend (src/check.py:39-45).
No kernel runs here."""
from types import SimpleNamespace

import pytest
import torch


def tiny_llama(layers=2):
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=128, intermediate_size=256, num_hidden_layers=layers,
                      num_attention_heads=4, num_key_value_heads=2, vocab_size=97,
                      rope_theta=500000.0, max_position_embeddings=512)
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg)


def test_to_lizard_swaps_every_block_and_copies_projections():
    from lizard_cuda.layer import LizardAttention
    from lizard_cuda.model import to_lizard
    model = tiny_llama()
    before = [{n: getattr(b.self_attn, n).weight.clone() for n in ("q_proj", "k_proj",
                                                                    "v_proj", "o_proj")}
              for b in model.model.layers]
    out = to_lizard(model, window=16, num_meta=4, feature_dim=8)
    assert out is model
    for i, (block, w) in enumerate(zip(model.model.layers, before)):
        attn = block.self_attn
        assert isinstance(attn, LizardAttention)
        assert attn.layer_idx == i and attn.window == 16 and attn.backend == "cuda"
        assert attn.kv_heads == 2 and attn.heads == 4
        assert attn.phi_q.weight.shape == (8, 32) and attn.meta_tokens.shape == (4,)
        for n, t in w.items():
            assert torch.equal(getattr(attn, n).weight, t), (i, n)


def test_to_lizard_rejects_other_backends():
    from lizard_cuda.model import to_lizard
    with pytest.raises(ValueError, match="cuda backend only"):
        to_lizard(tiny_llama(1), backend="triton")


def _cfg(backend):
    return SimpleNamespace(lizard=SimpleNamespace(backend=backend))


def test_check_kernels_skips_other_backends():
    from lizard_cuda.model import check_kernels
    assert check_kernels(None, _cfg("torch")) == "skipped, backend torch"
    assert check_kernels(None, _cfg("triton")) == "skipped, backend triton"


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU branch")
def test_check_kernels_fails_without_a_gpu():
    from lizard_cuda.model import check_kernels
    with pytest.raises(RuntimeError, match="needs a CUDA GPU"):
        check_kernels(None, _cfg("cuda"))
