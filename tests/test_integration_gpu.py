"""install() end to end on the GPU.

``SophiaKDA.forward`` (``ml/runtime/model/attention.py:373-420``) replaced by
``sophia_b200.install`` against the reference module's own fp32 output and
gradients (``golden/module_forward.npz``, written by ``make_golden.py`` from
Sophia's ``SophiaKDA`` with the reference backend: two rows of 70 tokens, the
second left-padded by 6 tokens through the pad mask).

The GPU box has no reference checkout, so the module is rebuilt here as a
stand-in class of the same name holding the same submodules and weights.  The
patched forward only uses those submodules -- the projections, the ShortConv
weights, the decay and beta projections, the output gate, the output norm
(``torch.nn.functional.rms_norm`` as ``ml/runtime/model/ops.py:49-64``) and
``o_proj`` -- plus this package's fused ``kda_layer``.

Tolerance: relative Frobenius error 2e-2 for the output and every gradient.
The reference runs in fp32 end to end, while the layer's inputs (post-projection
q, k, v, decay and beta logits) enter the kernels in bf16, as in the
reference's own CUDA path.
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch
from torch import nn

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "module_forward.npz")
REL_TOL = 2e-2


class _Conv(nn.Module):
    def __init__(self, channels: int, kernel: int) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.empty(channels, kernel))


class _RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return nn.functional.rms_norm(x, (int(x.size(-1)),), self.weight, float(self.eps))


class SophiaKDA(nn.Module):
    """Stand-in with the attributes the patched forward reads."""

    def __init__(self, dim: int, H: int, D: int, decay_rank: int) -> None:
        super().__init__()
        self.num_heads, self.head_dim, self.inner_dim = H, D, H * D
        self.output_gate_full_rank = True
        self.lower_bound = -5.0
        self.backend = "fla"
        self.use_cache = False
        self.conv_kernel = 4
        self.A_log = nn.Parameter(torch.zeros(H))
        self.dt_bias = nn.Parameter(torch.zeros(H * D))
        self.q_proj = nn.Linear(dim, H * D, bias=False)
        self.k_proj = nn.Linear(dim, H * D, bias=False)
        self.v_proj = nn.Linear(dim, H * D, bias=False)
        self.q_conv, self.k_conv, self.v_conv = (_Conv(H * D, 4) for _ in range(3))
        self.decay_down = nn.Linear(dim, decay_rank, bias=False)
        self.decay_up = nn.Linear(decay_rank, H * D, bias=False)
        self.beta_proj = nn.Linear(dim, H, bias=False)
        self.output_gate = nn.Linear(dim, H * D, bias=False)
        self.output_norm = _RMSNorm(D, 1e-5)
        self.o_proj = nn.Linear(H * D, dim, bias=False)

    def _run_kda(self, *args, **kwargs):
        raise RuntimeError("the stand-in has no recurrence of its own")

    def forward(self, x: torch.Tensor, *, start_pos: int = 0) -> torch.Tensor:
        raise RuntimeError("the stand-in is only run through install()")


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def test_installed_forward_matches_reference_module():
    import sophia_b200
    gold = np.load(GOLDEN)
    dim = gold["x"].shape[-1]
    H = gold["param.A_log"].shape[0]
    mod = SophiaKDA(dim, H, 128, gold["param.decay_down.weight"].shape[0])
    with torch.no_grad():
        for name, prm in mod.named_parameters():
            prm.copy_(torch.from_numpy(gold["param." + name]))
    mod = mod.cuda()
    report = sophia_b200.install(mod)
    assert report["kda_modules"] == 1
    assert mod._fla_chunk_kda() is sophia_b200.chunk_kda
    assert mod._fla_fused_recurrent_kda() is sophia_b200.fused_recurrent_kda
    mod._pad_mask = torch.from_numpy(gold["mask"]).cuda()
    x = torch.from_numpy(gold["x"]).cuda().requires_grad_(True)
    out = mod(x)
    (out * torch.from_numpy(gold["dout"]).cuda()).sum().backward()
    errs = {"out": _rel(out.detach(), torch.from_numpy(gold["out"])),
            "d_x": _rel(x.grad, torch.from_numpy(gold["d_x"]))}
    for name, prm in mod.named_parameters():
        ref = torch.from_numpy(gold["grad." + name])
        if ref.abs().max() > 0:
            errs["d_" + name] = _rel(prm.grad, ref)
    bad = {k: v for k, v in errs.items() if not v <= REL_TOL}
    assert not bad, {k: f"{v:.2e}" for k, v in sorted(errs.items())}
