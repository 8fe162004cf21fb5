"""lizard_cuda: B200 (sm_100a) kernels for Lizard's attention branches.

Drop-in for the reference's `kernels` package (src/kernels/__init__.py):
    import lizard_cuda as kernels
    kernels.gla(fq, fk, v, log_gamma, chunk=64)
    kernels.swa(q, k, v, meta, window, fwd_blocks=(64, 64), bwd_blocks=(64, 64))
Everything runs in liblizard_cuda.so through its C ABI; there is no CPU path.
"""
from ._lib import launch_count, load  # noqa: F401
from .gla import gla
from .hedgehog import hedgehog
from .swa import swa

__all__ = ["gla", "swa", "hedgehog", "load", "launch_count"]
