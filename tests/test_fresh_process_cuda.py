"""The first backward of a process on the tensor-core kernels. PyTorch runs it
on its autograd worker thread; with a bf16 contiguous dy and every tensor from
the caching allocator's cache, no CUDA runtime call has touched that thread yet,
so no context is current there when the library encodes its tensor maps (a
driver call). The library makes the primary context current first; before it
did, this sequence failed with CUDA_ERROR_INVALID_CONTEXT. Each case runs in a
fresh interpreter, since any earlier CUDA work on the thread would hide it."""
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

SCRIPT = r"""
import sys
sys.path.insert(0, {pkg!r})
import torch
import torch.nn.functional as F
import lizard_cuda
from lizard_cuda import _lib
dev = torch.device("cuda:0")
g = torch.Generator(device=dev).manual_seed(0)
B, H, L, D = 1, 4, 2048, {dim}
feats = lambda: (F.softplus(torch.randn(B, H, L, D, generator=g, device=dev)) / D ** 0.5).bfloat16()
if {gla}:
    _lib.set_schedule("walk")
    leaves = [t.requires_grad_() for t in (feats(), feats(),
              torch.randn(B, H, L, D, generator=g, device=dev).bfloat16(),
              F.logsigmoid(3 + torch.randn(B, H, L, generator=g, device=dev)))]
    y = lizard_cuda.gla(*leaves)
else:
    leaves = [t.requires_grad_() for t in (torch.randn(B, H, L, D, generator=g, device=dev).bfloat16(),
              torch.randn(B, H, L, D, generator=g, device=dev).bfloat16(),
              torch.randn(B, H, L, D, generator=g, device=dev).bfloat16(),
              torch.randn(4, generator=g, device=dev))]
    y = lizard_cuda.swa(*leaves, 128)
y.backward(torch.randn(B, H, L, D, generator=g, device=dev).bfloat16())
torch.cuda.synchronize()
assert all(torch.isfinite(t.grad).all() for t in leaves)
print("ok")
"""


@pytest.mark.parametrize("gla,dim", [(True, 128), (False, 64)], ids=["gla_f128_walk", "swa_w128"])
def test_first_backward_in_a_fresh_process(gla, dim):
    code = SCRIPT.format(pkg=str(ROOT / "lizard-reproduction_b200"), dim=dim, gla=gla)
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         timeout=300)
    assert res.returncode == 0 and res.stdout.strip().endswith("ok"), res.stderr[-2000:]
