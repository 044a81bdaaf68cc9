"""CPU oracle for the KDA layer hot path (TEST INFRASTRUCTURE ONLY).

This module restates, in plain PyTorch on the CPU, what Sophia's reference KDA
layer computes. It is the checker the parity tests, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg compare the CUDA path against. Nothing in
the product package imports it: the product fails loudly when its CUDA
extension is missing instead of falling back to this file.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
modules (``ml.runtime.model.attention``) on seeded inputs and commits their
outputs and autograd gradients under ``tests/golden/``; ``tests/test_oracle.py``
checks this restatement against those fixtures.

Reference semantics restated here (paths relative to the Sophia repository):

* ``CausalDepthwiseConv1d.forward`` -- ``ml/runtime/model/attention.py:32-60``:
  left zero history of ``K-1`` positions, depthwise ``conv1d`` with weight
  ``[C, K]``, then SiLU.
* ``SophiaKDA._reference_kda`` -- ``ml/runtime/model/attention.py:260-294``:
  ``q <- normalize(q) * D**-0.5``, ``k <- normalize(k)``,
  ``g = lower_bound * sigmoid(exp(A_log) * (logits + dt_bias))``,
  ``beta = sigmoid(beta_logits)`` and the per-token delta rule
  ``S <- S * exp(g)``; ``S <- S + k (beta (v - k^T S))^T``; ``o = S^T q``.
* ``SophiaKDA._run_kda`` -- ``ml/runtime/model/attention.py:314-371``: the
  module seam; ``scale`` defaults to ``D**-0.5``
  (``fla/ops/kda/chunk.py:386-387`` of flash-linear-attention 0.5.x).
* Packed sequences (``cu_seqlens``): the reference itself never packs; the
  chunked CUDA path it calls (flash-linear-attention ``chunk_kda``) resets the
  recurrent state at every boundary, and the ShortConv seam's CUDA
  replacement (causal-conv1d with ``seq_idx``) resets the convolution history.
  The oracle therefore runs each document as an independent unpacked sequence
  with zero conv history and its own initial state.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

__all__ = [
    "shortconv_silu",
    "kda_gate",
    "reference_kda",
    "kda_layer",
    "KdaOutputs",
]


def shortconv_silu(x: torch.Tensor, weight: torch.Tensor,
                   history: torch.Tensor | None = None):
    """Causal depthwise conv + SiLU (``attention.py:32-60``).

    x: ``[B, T, C]``; weight: ``[C, K]``; history: ``[B, C, K-1]`` or None
    (zeros).  Returns ``(silu(conv(x)), next_history)``.
    """
    B, T, C = x.shape
    K = weight.shape[1]
    xc = x.transpose(1, 2)
    if K > 1:
        if history is None:
            history = xc.new_zeros(B, C, K - 1)
        seq = torch.cat((history.to(x.dtype), xc), dim=-1)
    else:
        seq = xc
    out = F.conv1d(seq, weight.to(x.dtype).unsqueeze(1), groups=C).transpose(1, 2)
    nxt = seq[..., -(K - 1):] if K > 1 else seq[..., :0]
    return F.silu(out), nxt


def kda_gate(g_logits: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor,
             lower_bound: float) -> torch.Tensor:
    """Per-channel log decay ``lb * sigmoid(exp(A_log) * (x + dt_bias))``
    (``attention.py:275-280``); g_logits ``[B, T, H, D]``."""
    H, D = g_logits.shape[-2:]
    scale = torch.exp(A_log.to(g_logits.dtype)).view(1, 1, H, 1)
    bias = dt_bias.to(g_logits.dtype).view(1, 1, H, D)
    return lower_bound * torch.sigmoid(scale * (g_logits + bias))


def reference_kda(q, k, v, g_logits, beta_logits, A_log, dt_bias, *,
                  lower_bound: float = -5.0, scale: float | None = None,
                  initial_state: torch.Tensor | None = None,
                  compute_dtype: torch.dtype = torch.float64):
    """Per-token gated delta rule of ``_reference_kda`` (``attention.py:260-294``).

    q, k, v, g_logits: ``[B, T, H, D]`` (post-conv, pre-norm); beta_logits
    ``[B, T, H]``; initial_state ``[B, H, D, D]``.  Everything is computed in
    ``compute_dtype``; returns ``(o [B,T,H,D] in compute_dtype, S [B,H,D,D])``.
    """
    B, T, H, D = q.shape
    if scale is None:
        scale = D ** -0.5
    cd = compute_dtype
    qn = F.normalize(q.to(cd), p=2.0, dim=-1) * scale
    kn = F.normalize(k.to(cd), p=2.0, dim=-1)
    vv = v.to(cd)
    alpha = torch.exp(kda_gate(g_logits.to(cd), A_log.to(cd), dt_bias.to(cd), lower_bound))
    beta = torch.sigmoid(beta_logits.to(cd))
    state = (qn.new_zeros(B, H, D, vv.shape[-1]) if initial_state is None
             else initial_state.to(cd))
    outs = []
    for t in range(T):
        state = state * alpha[:, t].unsqueeze(-1)
        pred = torch.einsum("bhd,bhdv->bhv", kn[:, t], state)
        corr = (vv[:, t] - pred) * beta[:, t].unsqueeze(-1)
        state = state + kn[:, t].unsqueeze(-1) * corr.unsqueeze(-2)
        outs.append(torch.einsum("bhd,bhdv->bhv", qn[:, t], state))
    if T == 0:
        o = vv.new_zeros(B, 0, H, vv.shape[-1])
    else:
        o = torch.stack(outs, dim=1)
    return o, state


@dataclass
class KdaOutputs:
    o: torch.Tensor           # [B, T, H, D]
    final_state: torch.Tensor  # [N, H, D, D]


def kda_layer(q_pre, k_pre, v_pre, g_logits, beta_logits, A_log, dt_bias, *,
              conv_weights=None, lower_bound: float = -5.0,
              scale: float | None = None, initial_state=None, cu_seqlens=None,
              compute_dtype: torch.dtype = torch.float64) -> KdaOutputs:
    """ShortConv(+SiLU) on q/k/v (when ``conv_weights`` is given) followed by
    the reference recurrence, per document when ``cu_seqlens`` is given.

    q_pre/k_pre/v_pre: ``[B, T, H, D]``; conv_weights: three ``[H*D, 4]``
    tensors (q, k, v) or None (inputs are already post-conv).
    cu_seqlens: 1-D int tensor ``[N+1]`` (requires ``B == 1``).
    Differentiable w.r.t. every floating input.
    """
    B, T, H, D = q_pre.shape
    cd = compute_dtype

    def run(qp, kp, vp, gl, bl, h0):
        if conv_weights is not None:
            outs = []
            for x, w in zip((qp, kp, vp), conv_weights):
                b, t = x.shape[:2]
                y, _ = shortconv_silu(x.to(cd).reshape(b, t, H * D), w.to(cd))
                outs.append(y.reshape(b, t, H, D))
            qp, kp, vp = outs
        return reference_kda(qp, kp, vp, gl, bl, A_log, dt_bias,
                             lower_bound=lower_bound, scale=scale,
                             initial_state=h0, compute_dtype=cd)

    if cu_seqlens is None:
        o, S = run(q_pre, k_pre, v_pre, g_logits, beta_logits, initial_state)
        return KdaOutputs(o, S)
    if B != 1:
        raise ValueError("cu_seqlens requires batch size 1")
    cu = [int(x) for x in cu_seqlens.tolist()]
    outs, states = [], []
    for n, (bos, eos) in enumerate(zip(cu[:-1], cu[1:])):
        h0 = None if initial_state is None else initial_state[n:n + 1]
        sl = slice(bos, eos)
        o, S = run(q_pre[:, sl], k_pre[:, sl], v_pre[:, sl], g_logits[:, sl],
                   beta_logits[:, sl], h0)
        outs.append(o)
        states.append(S)
    o = torch.cat(outs, dim=1) if outs else q_pre.new_zeros(1, 0, H, D, dtype=cd)
    return KdaOutputs(o, torch.cat(states, dim=0))


def inverse_softplus(x: torch.Tensor) -> torch.Tensor:
    """``attention.py:20-21``."""
    return x + torch.log(-torch.expm1(-x))


def dt_bias_init(n: int, generator: torch.Generator, dt_min=1e-3, dt_max=1e-1,
                 dt_floor=1e-4) -> torch.Tensor:
    """``dt_bias`` initialisation of ``attention.py:101-106``."""
    dt = torch.exp(torch.rand(n, generator=generator, dtype=torch.float32)
                   * (math.log(dt_max) - math.log(dt_min)) + math.log(dt_min)
                   ).clamp_min(dt_floor)
    return inverse_softplus(dt)
