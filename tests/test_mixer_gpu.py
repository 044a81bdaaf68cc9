"""The mixer block (``sophia_b200.mixer.KDAMixerBlock``) against its oracle.

The oracle is the same block computed on the CPU in float64 from torch ops
and the restated reference recurrence (``oracle.kda_oracle.kda_layer``, which
follows ``ml/runtime/model/attention.py:24-60,260-294``), with the output
RMSNorm and gate of ``attention.py:416-419``.  Compared: the block output and
the gradients of the input and of every parameter, as relative Frobenius
errors.

Tolerance 2e-2 (as the module-level integration test): the kernels take their
inputs in bf16, as the reference's CUDA path does.
"""

from __future__ import annotations

import os
import sys

import pytest
import torch
from torch.nn import functional as F

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from oracle.kda_oracle import kda_layer as oracle_layer  # noqa: E402

pytestmark = pytest.mark.gpu
REL_TOL = 2e-2


def _oracle_block(m, x):
    p = {n: t.detach().double().requires_grad_(True) for n, t in m.named_parameters()}
    xx = x.detach().double().requires_grad_(True)
    B, T, dim = xx.shape
    H, D = m.heads, 128
    h = F.rms_norm(xx, (dim,), p["in_norm"], m.eps)
    q, k, v, gate = F.linear(h, p["w_qkvg"]).split(H * D, dim=-1)
    decay = F.linear(F.linear(h, p["decay_down"]), p["decay_up"])
    beta = F.linear(h, p["beta_proj"])
    o = oracle_layer(q.reshape(B, T, H, D), k.reshape(B, T, H, D), v.reshape(B, T, H, D),
                     decay.reshape(B, T, H, D), beta, p["A_log"], p["dt_bias"],
                     conv_weights=[p["conv_q"], p["conv_k"], p["conv_v"]], lower_bound=m.lower_bound,
                     compute_dtype=torch.float64).o
    y = F.rms_norm(o, (D,), p["out_norm"], m.eps) * torch.sigmoid(gate.reshape(B, T, H, D))
    out = F.linear(y.reshape(B, T, H * D), p["o_proj"])
    return out, xx, p


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def test_mixer_block_matches_oracle():
    from sophia_b200.mixer import KDAMixerBlock
    gen = torch.Generator().manual_seed(11)
    m = KDAMixerBlock(dim=256, heads=2, decay_rank=32, std=0.05, generator=gen)
    x = torch.randn(2, 96, 256, generator=gen)
    dout = torch.randn(2, 96, 256, generator=gen)
    ref_out, ref_x, ref_p = _oracle_block(m, x)
    (ref_out * dout.double()).sum().backward()

    mc = m.cuda()
    xc = x.cuda().requires_grad_(True)
    out = mc(xc)
    (out * dout.cuda()).sum().backward()
    errs = {"out": _rel(out.detach(), ref_out.detach()), "d_x": _rel(xc.grad, ref_x.grad)}
    for n, prm in mc.named_parameters():
        errs["d_" + n] = _rel(prm.grad, ref_p[n].grad)
    bad = {k: v for k, v in errs.items() if not v <= REL_TOL}
    assert not bad, {k: f"{v:.2e}" for k, v in sorted(errs.items())}


def test_mixer_block_bf16_autocast_runs_and_is_finite():
    from sophia_b200.mixer import KDAMixerBlock
    gen = torch.Generator().manual_seed(5)
    m = KDAMixerBlock(generator=gen).cuda()
    x = torch.randn(1, 200, 1536, generator=gen).cuda().bfloat16().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = m(x)
    assert out.dtype == torch.bfloat16 and out.shape == x.shape
    out.float().square().mean().backward()
    assert torch.isfinite(x.grad).all()
    assert all(torch.isfinite(p.grad).all() for p in m.parameters())
