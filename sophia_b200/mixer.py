"""The KDA mixer block on the B200 kernels (the configuration-2 shape).

RMSNorm of the block input -> one fused q/k/v/gate projection -> low-rank
decay and beta projections -> ShortConv(+SiLU), L2 norms, gate and the chunked
delta rule (``kda_layer``) -> gated output RMSNorm (``gated_rms_norm``) ->
out-projection.  It follows ``SophiaKDA`` (``ml/runtime/model/attention.py:
62-420``: projections ``:107-125``, ``forward`` ``:373-420``) with its
``args`` defaults (``ml/runtime/model/config.py``: decay rank 128, dt in
[1e-3, 1e-1] floored at 1e-4, ``A_log`` = 0, norm eps 1e-5, lower bound -5)
and adds the block's input RMSNorm in front.  The q/k/v/gate weights are one
[4 x 2048, 1536] parameter; its four row blocks are four GEMMs, whose outputs
are the contiguous [B, T, 2048] operands the kernels read (one GEMM's output
would need four strided copies first).

The projections are plain cuBLAS GEMMs (``torch.nn.functional.linear``); the
recurrence and the output norm run on this package's kernels.  Parameters are
fp32; run it under ``torch.autocast("cuda", torch.bfloat16)`` for the bf16
training step.
"""

from __future__ import annotations

import math

import torch
from torch import nn
from torch.nn import functional as F

from .ops import HEAD_DIM, gated_rms_norm, kda_layer


def _inverse_softplus(x: torch.Tensor) -> torch.Tensor:
    return x + torch.log(-torch.expm1(-x))


class KDAMixerBlock(nn.Module):
    def __init__(self, dim: int = 1536, heads: int = 16, decay_rank: int = 128, conv_kernel: int = 4,
                 eps: float = 1e-5, lower_bound: float = -5.0, dt_min: float = 1e-3, dt_max: float = 1e-1,
                 dt_floor: float = 1e-4, std: float = 0.02, generator: torch.Generator | None = None,
                 device: torch.device | str | None = None) -> None:
        super().__init__()
        if conv_kernel != 4:
            raise ValueError("the fused ShortConv has kernel size 4")
        self.dim, self.heads, self.eps, self.lower_bound = dim, heads, eps, lower_bound
        inner = heads * HEAD_DIM
        kw = {"device": device, "dtype": torch.float32}

        def normal(*shape):
            return nn.Parameter(torch.randn(*shape, generator=generator, **kw) * std)

        self.in_norm = nn.Parameter(torch.ones(dim, **kw))
        self.w_qkvg = normal(4 * inner, dim)          # q, k, v, output gate
        self.decay_down = normal(decay_rank, dim)
        self.decay_up = normal(inner, decay_rank)
        self.beta_proj = normal(heads, dim)
        self.conv_q, self.conv_k, self.conv_v = normal(inner, 4), normal(inner, 4), normal(inner, 4)
        self.A_log = nn.Parameter(torch.zeros(heads, **kw))
        u = torch.rand(inner, generator=generator, **kw)
        dt = torch.exp(u * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min)).clamp_min(dt_floor)
        self.dt_bias = nn.Parameter(_inverse_softplus(dt))
        self.out_norm = nn.Parameter(torch.ones(HEAD_DIM, **kw))
        self.o_proj = normal(dim, inner)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x [B, T, dim] -> [B, T, dim]."""
        B, T, _ = x.shape
        H, D = self.heads, HEAD_DIM
        h = F.rms_norm(x, (self.dim,), self.in_norm.to(x.dtype), self.eps)
        # four GEMMs from row blocks of the one weight: each output is a
        # contiguous [B, T, H*D] tensor, so the kernels read it without a copy
        q, k, v, gate = (F.linear(h, w) for w in self.w_qkvg.split(H * D, dim=0))
        decay = F.linear(F.linear(h, self.decay_down), self.decay_up)
        beta = F.linear(h, self.beta_proj)
        o, _ = kda_layer(q.reshape(B, T, H, D), k.reshape(B, T, H, D), v.reshape(B, T, H, D),
                         decay.reshape(B, T, H, D), beta, self.A_log, self.dt_bias,
                         self.conv_q, self.conv_k, self.conv_v, lower_bound=self.lower_bound)
        y = gated_rms_norm(o, gate.reshape(B, T, H, D), self.out_norm, self.eps)
        return F.linear(y.reshape(B, T, H * D), self.o_proj)
