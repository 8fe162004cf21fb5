"""Generate the golden fixtures in this directory from the reference itself.

Runs the reference's own torch backend (src/lizard_attention.py of
mahdikhashan/lizard-reproduction: gla, awa, LizardAttention) in fp32 on the
seeded inputs of cases.py and stores outputs and gradients, the latter both
for the fp32 upstream gradient and for its bf16 rounding (keys ending in _b),
which is what a bf16-output kernel receives from autograd. This is exactly
how the reference checks its kernels (tests/test_kernels.py:32-42, 61-70,
121-122, 137-156). Needs a checkout of the reference; the path comes from
LIZARD_REFERENCE_SRC when it is set, else from baseline/_ref at the root of
this repository (where the reference's src/ modules are installed, unmodified,
for the same-box timing). The fixtures are committed; the tests never need the
reference.

    LIZARD_REFERENCE_SRC=<reference checkout>/src python tests/golden/make_golden.py
"""
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import cases  # noqa: E402

def _reference_src():
    env = os.environ.get("LIZARD_REFERENCE_SRC")
    if env:
        return env
    local = HERE.parents[1] / "baseline" / "_ref"
    if (local / "lizard_attention.py").exists():
        return str(local)
    raise SystemExit("set LIZARD_REFERENCE_SRC to the reference's src/ directory "
                     "(or install the reference into baseline/_ref)")


def reference():
    sys.path.insert(0, _reference_src())
    import lizard_attention as lz  # the reference module
    return lz


def gla_run(lz, inp, dy):
    fq, fk, v = (inp[n].float().requires_grad_() for n in ("fq", "fk", "v"))
    lg = inp["log_gamma"].clone().requires_grad_()
    gamma = lg.exp()
    if lg.dim() == 2:
        y = lz.gla(fq, fk, v, gamma)
    else:  # per-head gate: fold batch*heads (tests/test_kernels.py:66-70)
        b, h, n, _ = fq.shape

        def fold(t):
            return t.reshape(b * h, 1, n, -1)
        y = lz.gla(fold(fq), fold(fk), fold(v), gamma.reshape(b * h, n)).reshape(b, h, n, -1)
    y.backward(dy)
    return y.detach(), (fq.grad, fk.grad, v.grad, lg.grad)


def gla_golden(lz, name, kw):
    inp = cases.gla_case(**kw)
    y, (dfq, dfk, dv, dlg) = gla_run(lz, inp, inp["dy"])
    # the kernels return bf16, so autograd hands them bf16(dy): the reference's
    # gradients for that upstream gradient (suffix _b)
    _, (dfq_b, dfk_b, dv_b, dlg_b) = gla_run(lz, inp, inp["dy"].bfloat16().float())
    return dict(kind="gla", kw=kw, inputs=inp, y=y, dfq=dfq, dfk=dfk, dv=dv, dlog_gamma=dlg,
                dfq_b=dfq_b, dfk_b=dfk_b, dv_b=dv_b, dlog_gamma_b=dlg_b)


def swa_run(lz, inp, window, dy):
    q, k, v = (inp[n].float().requires_grad_() for n in ("q", "k", "v"))
    meta = inp["meta"].clone().requires_grad_()
    if meta.numel() == 0:  # no sinks: the reference evaluates it with a -1e4 sink
        ref_meta = torch.full((1,), -1e4)  # (tests/test_kernels.py:127-134)
    else:
        ref_meta = meta
    y = lz.awa(q, k, v, ref_meta, window)
    y.backward(dy)
    dmeta = meta.grad if meta.numel() else torch.zeros(0)
    return y.detach(), (q.grad, k.grad, v.grad, dmeta)


def swa_golden(lz, name, kw, window):
    inp = cases.swa_case(**kw)
    y, (dq, dk, dv, dmeta) = swa_run(lz, inp, window, inp["dy"])
    _, (dq_b, dk_b, dv_b, dmeta_b) = swa_run(lz, inp, window, inp["dy"].bfloat16().float())
    return dict(kind="swa", kw=kw, window=window, inputs=inp, y=y, dq=dq, dk=dk, dv=dv,
                dmeta=dmeta, dq_b=dq_b, dk_b=dk_b, dv_b=dv_b, dmeta_b=dmeta_b)


def layer_golden(lz, name, case):
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    config = LlamaConfig(hidden_size=case["hidden"], intermediate_size=2 * case["hidden"],
                         num_hidden_layers=1, num_attention_heads=case["heads"],
                         num_key_value_heads=case["kv_heads"], vocab_size=100,
                         rope_theta=case["theta"], attn_implementation="eager")
    layer = lz.LizardAttention(config, 0, window=case["window"], num_meta=case["num_meta"],
                               feature_dim=case["feature_dim"], backend="torch")
    cases.init_layer_params(layer, case["init"])
    x, grad = cases.layer_inputs(case)
    positions = torch.arange(case["length"])[None]
    cos, sin = LlamaRotaryEmbedding(config)(x, positions)
    y = layer(x, (cos, sin))[0]
    y.backward(grad)
    grads = {n: p.grad.detach().clone() for n, p in layer.named_parameters()}
    params = {n: cases.checksum(p) for n, p in layer.named_parameters()}
    return dict(kind="layer", case=case, x_sum=cases.checksum(x), grad_sum=cases.checksum(grad),
                param_sums=params, cos=cos.float(), sin=sin.float(), y=y.detach(), grads=grads)


def main():
    lz = reference()
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    for name, kw in cases.GLA_CASES.items():
        torch.save(gla_golden(lz, name, kw), HERE / f"{name}.pt")
        print("wrote", name)
    for name, (kw, window) in cases.SWA_CASES.items():
        torch.save(swa_golden(lz, name, kw, window), HERE / f"{name}.pt")
        print("wrote", name)
    for name, case in cases.LAYER_CASES.items():
        torch.save(layer_golden(lz, name, case), HERE / f"{name}.pt")
        print("wrote", name)


if __name__ == "__main__":
    main()
