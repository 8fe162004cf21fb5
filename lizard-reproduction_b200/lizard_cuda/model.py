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

greedy_generate(model, input_ids, steps) decodes with the recurrent cache
(lizard_cuda.decode): one full forward over the prompt, then one token per
step at O(1) cost per layer (the reference has no cache and would recompute
the whole sequence for every new token); GraphedDecoder replays a captured
decode step as one CUDA graph launch.
"""
import torch

from .decode import LizardCache
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
    Returns a one-line status; raises RuntimeError when the backend cannot run
    here (the reference's check runner reports any exception as a failed check,
    src/check.py:39-45, where the triton branch asserts instead; a raised error
    also survives python -O)."""
    backend = cfg.lizard.backend
    if backend != "cuda":
        return f"skipped, backend {backend}"
    if not torch.cuda.is_available():
        raise RuntimeError("the cuda backend needs a CUDA GPU")
    lib = _lib.load()
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        raise RuntimeError(
            f"liblizard_cuda.so is built for sm_100a; this GPU is sm_{major}{minor}")
    return f"lizard_cuda ABI {lib.lz_abi_version()} on {torch.cuda.get_device_name()}"


class GraphedDecoder:
    """One greedy decode step of the whole model for a fixed batch, captured
    as a CUDA graph: a step is one graph launch instead of several hundred
    kernel launches from Python. The step reads the token and position
    buffers, advances every layer's cache in place (the cache tensors are the
    graph's static buffers) and writes the next token and position back.

    Construction runs one eager step (which also prepares every kernel's
    launch attributes) and then captures the next; `tokens` / `position`
    ([B, 1], the last token and its position) are copied into the static
    buffers. step() replays the graph and returns the new tokens [B, 1]."""

    def __init__(self, model, cache, tokens, position):
        self.model, self.cache = model, cache
        self.tok = tokens.clone()
        self.pos = position.clone()
        self._step()  # eager: the kernels' one-time setup happens outside the capture
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()

    def _step(self):
        logits = self.model(self.tok, position_ids=self.pos, lizard_cache=self.cache,
                            use_cache=False).logits
        self.tok.copy_(logits[:, -1].argmax(-1, keepdim=True))
        self.pos.add_(1)

    def step(self):
        self.graph.replay()
        return self.tok


@torch.no_grad()
def greedy_generate(model, input_ids, steps, graph=False):
    """Greedy continuation of input_ids [B, L] by `steps` tokens with a
    LizardCache: the prompt runs through the full forward (which stores every
    layer's state), each new token through the layers' decode path, eagerly or
    (graph=True) as replays of a GraphedDecoder. Returns the new token ids
    [B, steps] and the cache."""
    cache = LizardCache()
    B, L = input_ids.shape
    logits = model(input_ids, lizard_cache=cache, use_cache=False, logits_to_keep=1).logits
    tokens = [logits[:, -1].argmax(-1, keepdim=True)]
    pos = torch.full((B, 1), L, dtype=torch.long, device=input_ids.device)
    if graph and steps > 2:
        dec = GraphedDecoder(model, cache, tokens[-1], pos)  # runs step 2 eagerly
        tokens.append(dec.tok.clone())
        for _ in range(2, steps):
            tokens.append(dec.step().clone())
        return torch.cat(tokens, 1), cache
    for _ in range(1, steps):
        logits = model(tokens[-1], position_ids=pos, lizard_cache=cache, use_cache=False).logits
        tokens.append(logits[:, -1].argmax(-1, keepdim=True))
        pos = pos + 1
    return torch.cat(tokens, 1), cache
