"""Fused gated output norm of the mixer (``gated_rms_norm``).

It replaces ``SophiaKDA.forward``'s ``self.output_norm(o) * sigmoid(gate)``
(``ml/runtime/model/attention.py:416-419``; ``RMSNorm`` is
``torch.nn.functional.rms_norm`` with a fp32 weight, ``ml/runtime/model/ops.py:
49-64``).  The GPU tests compare the CUDA kernels, forward and all three
gradients, with the same formula evaluated by torch in float64 on the same
inputs.

Tolerances: fp32 inputs 2e-5 relative per element (+1e-6 absolute; the kernel
uses rsqrt.approx and ex2.approx); bf16 inputs and outputs one bf16 rounding,
8e-3 relative (+1e-3 absolute), and relative Frobenius error 4e-3.  The weight
gradient is a fp32 sum over rows either way: 1e-4 relative Frobenius.
"""

from __future__ import annotations

import pytest
import torch

import sophia_b200
from sophia_b200.ops import HEAD_DIM


def _reference(o, g, w, eps, dy):
    o64, g64, w64 = (t.detach().double().requires_grad_(True) for t in (o, g, w))
    y = o64 * torch.rsqrt(o64.pow(2).mean(-1, keepdim=True) + eps) * w64 * torch.sigmoid(g64)
    y.backward(dy.double())
    return y.detach(), o64.grad, g64.grad, w64.grad


def _rel(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 1, 1), (2, 37, 3), (4, 256, 16), (0, 5, 2)])
def test_gated_norm_matches_torch(dtype, shape):
    gen = torch.Generator(device="cuda").manual_seed(7)
    o = (torch.randn(*shape, HEAD_DIM, device="cuda", generator=gen) * 1.7).to(dtype).requires_grad_(True)
    g = (torch.randn(*shape, HEAD_DIM, device="cuda", generator=gen) * 2.0).to(dtype).requires_grad_(True)
    w = (torch.rand(HEAD_DIM, device="cuda", generator=gen) + 0.5).requires_grad_(True)
    dy = torch.randn(*shape, HEAD_DIM, device="cuda", generator=gen).to(dtype)
    eps = 1e-5
    y = sophia_b200.gated_rms_norm(o, g, w, eps)
    assert y.dtype == dtype and y.shape == o.shape
    y.backward(dy)
    ry, ro, rg, rw = _reference(o, g, w, eps, dy)
    if o.numel() == 0:
        assert torch.all(w.grad == 0)
        return
    for got, ref in ((y, ry), (o.grad, ro), (g.grad, rg)):
        err = (got.double() - ref).abs()
        if dtype == torch.float32:
            assert torch.all(err <= 2e-5 * ref.abs() + 1e-6), float(err.max())
        else:
            assert torch.all(err <= 8e-3 * ref.abs() + 1e-3), float(err.max())
            assert _rel(got, ref) <= 4e-3
    assert _rel(w.grad, rw) <= 1e-4


@pytest.mark.gpu
def test_gated_norm_weight_gradient_is_deterministic():
    gen = torch.Generator(device="cuda").manual_seed(3)
    o = torch.randn(8, 512, 16, HEAD_DIM, device="cuda", generator=gen).bfloat16()
    g = torch.randn(8, 512, 16, HEAD_DIM, device="cuda", generator=gen).bfloat16()
    w = torch.rand(HEAD_DIM, device="cuda", generator=gen) + 0.5
    dy = torch.randn(8, 512, 16, HEAD_DIM, device="cuda", generator=gen).bfloat16()
    grads = []
    for _ in range(2):
        ww = w.clone().requires_grad_(True)
        sophia_b200.gated_rms_norm(o, g, ww).backward(dy)
        grads.append(ww.grad.clone())
    assert torch.equal(grads[0], grads[1])


def test_gated_norm_rejects_bad_shapes_and_cpu_tensors():
    o = torch.zeros(2, 3, HEAD_DIM)
    with pytest.raises(ValueError):
        sophia_b200.gated_rms_norm(o, torch.zeros(2, 3, 64), torch.ones(HEAD_DIM))
    with pytest.raises(ValueError):
        sophia_b200.gated_rms_norm(o, o, torch.ones(64))
    with pytest.raises(RuntimeError):
        sophia_b200.gated_rms_norm(o, o, torch.ones(HEAD_DIM))
