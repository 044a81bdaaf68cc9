"""Runs the CPU oracle on a golden case and returns outputs and gradients.

Shared by the CPU oracle tests and the GPU parity tests.  The gradients are
torch autograd of ``sum(o * dO) + sum(S * dS)`` through the oracle, the same
loss the golden generator uses with the reference modules.
"""

from __future__ import annotations

import torch

from cases import Case, make_inputs
from oracle.kda_oracle import kda_layer

GRAD_KEYS = ("q", "k", "v", "g", "beta", "conv_q", "conv_k", "conv_v",
             "A_log", "dt_bias", "h0")


def run_oracle(case: Case, inputs: dict | None = None,
               dtype: torch.dtype = torch.float64, grads: bool = True) -> dict:
    inp = make_inputs(case) if inputs is None else inputs
    leaves = {k: inp[k].to(dtype).clone().requires_grad_(grads) for k in GRAD_KEYS}
    cu = None if case.cu_seqlens is None else torch.tensor(case.cu_seqlens)
    out = kda_layer(
        leaves["q"], leaves["k"], leaves["v"], leaves["g"], leaves["beta"],
        leaves["A_log"], leaves["dt_bias"],
        conv_weights=(leaves["conv_q"], leaves["conv_k"], leaves["conv_v"]) if case.conv else None,
        lower_bound=case.lower_bound,
        initial_state=leaves["h0"] if case.h0 else None,
        cu_seqlens=cu, compute_dtype=dtype)
    res = {"o": out.o.detach(), "final_state": out.final_state.detach()}
    if grads:
        loss = (out.o * inp["do"].to(dtype)).sum()
        if case.final_state_grad:
            loss = loss + (out.final_state * inp["dht"].to(dtype)).sum()
        loss.backward()
        for k, v in leaves.items():
            res["d_" + k] = (v.grad if v.grad is not None else torch.zeros_like(v)).detach()
        if not case.conv:
            for k in ("conv_q", "conv_k", "conv_v"):
                res["d_" + k] = torch.zeros_like(leaves[k])
        if not case.h0:
            res["d_h0"] = torch.zeros_like(leaves["h0"])
    return res
