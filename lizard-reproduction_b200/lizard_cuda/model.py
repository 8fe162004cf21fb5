"""Model-level integration of the cuda backend.

to_lizard(model, ...) replaces every decoder block's self-attention of a
Hugging Face Llama model by LizardAttention with the `cuda` backend, copying
the q / k / v / o projections, as the reference's training script does
(src/train.py:35-39 with from_llama, src/lizard_attention.py:100-107). The
Lizard parameters (phi_q, phi_k, W_gamma, meta_tokens, alpha_blend) start from
the layer's own init, as in the reference.

check_kernels(api, cfg) is the reference's pre-flight check
(src/check.py:39-45) with a branch for the `cuda` backend: it loads
liblizard_cuda.so (which verifies its ABI revision) and checks that the GPU
is a compute capability 10.0 part, the one the library is built for.
"""
from .layer import LizardAttention, from_llama  # noqa: F401
from . import _lib

OPTIONS = ("window", "num_meta", "feature_dim", "backend")


def to_lizard(model, window=128, num_meta=4, feature_dim=128, backend="cuda"):
    """Swap model.model.layers[i].self_attn for LizardAttention in place and
    return the model (src/train.py:35-39). The keyword arguments are the
    reference config's `lizard` section (src/config.py:10-15)."""
    options = dict(window=window, num_meta=num_meta, feature_dim=feature_dim, backend=backend)
    for block in model.model.layers:
        block.self_attn = from_llama(block.self_attn, model.config, **options)
    return model


def check_kernels(api, cfg):
    """Pre-flight check of the kernel backend named by cfg.lizard.backend.
    Returns a one-line status; raises when the backend cannot run here (the
    reference's check runner reports the exception as a failed check)."""
    backend = cfg.lizard.backend
    if backend != "cuda":
        return f"skipped, backend {backend}"
    import torch
    assert torch.cuda.is_available(), "the cuda backend needs a CUDA GPU"
    lib = _lib.load()
    major, minor = torch.cuda.get_device_capability()
    assert (major, minor) == (10, 0), (
        f"liblizard_cuda.so is built for sm_100a; this GPU is sm_{major}{minor}")
    return f"lizard_cuda ABI {lib.lz_abi_version()} on {torch.cuda.get_device_name()}"
