"""lizard_cuda: B200 (sm_100a) kernels for Lizard's attention branches.

Drop-in for the reference's `kernels` package (src/kernels/__init__.py):
    import lizard_cuda as kernels
    kernels.gla(fq, fk, v, log_gamma, chunk=64)
    kernels.swa(q, k, v, meta, window, fwd_blocks=(64, 64), bwd_blocks=(64, 64))
Everything runs in liblizard_cuda.so through its C ABI; there is no CPU path.
Beyond the reference's two entry points: grouped-query k / v (fewer heads than
q) in gla and swa, swa_rope (RoPE fused into the SWA operand pass) and hedgehog
(the fused feature map) and blend (the layer's output blend).
"""
from ._lib import launch_count, load  # noqa: F401
from .blend import blend
from .gla import gla
from .hedgehog import hedgehog
from .rope import swa_rope
from .swa import swa

__all__ = ["gla", "swa", "swa_rope", "hedgehog", "blend", "load", "launch_count"]
