"""The reference's own CUDA path for the KDA layer, for accuracy comparison
(TEST INFRASTRUCTURE ONLY).

On CUDA, Sophia's ``SophiaKDA`` runs ``CausalDepthwiseConv1d`` as a bf16
``conv1d`` + SiLU under autocast (``ml/runtime/model/attention.py:32-60``) and
the recurrence through flash-linear-attention's Triton ``chunk_kda``
(``attention.py:349-365``).  This module runs exactly that pair on the same
inputs as ``kda_cuda_runner.run_cuda`` so the two CUDA paths can be held to the
same oracle.  FLA's alternative backends are disabled so its default Triton
kernels run.
"""

from __future__ import annotations

import os

os.environ.setdefault("FLA_DISABLE_BACKEND_DISPATCH", "1")

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

from cases import Case, make_inputs  # noqa: E402
from oracle_runner import GRAD_KEYS  # noqa: E402


def fla_available() -> bool:
    try:
        import fla.ops.kda  # noqa: F401
        return True
    except Exception:
        return False


def _conv_bf16(x, w):
    """attention.py:38-60 with history None, in the input dtype."""
    B, T, C = x.shape
    xc = x.transpose(1, 2)
    seq = torch.cat((xc.new_zeros(B, C, 3), xc), dim=-1)
    out = F.conv1d(seq, w.to(x.dtype).unsqueeze(1), groups=C).transpose(1, 2)
    return F.silu(out)


def run_fla(case: Case, inputs: dict | None = None, grads: bool = True) -> dict:
    from fla.ops.kda import chunk_kda
    inp = make_inputs(case) if inputs is None else inputs
    dev = "cuda"
    t = {}
    for k in GRAD_KEYS:
        dt = torch.bfloat16 if k in ("q", "k", "v", "g", "beta") else torch.float32
        t[k] = inp[k].to(device=dev, dtype=dt).clone().requires_grad_(grads)
    B, T, H, D = t["q"].shape
    cu = None if case.cu_seqlens is None else torch.tensor(case.cu_seqlens, dtype=torch.int64, device=dev)
    xs = [t["q"], t["k"], t["v"]]
    if case.conv:
        post = []
        for x, w in zip(xs, (t["conv_q"], t["conv_k"], t["conv_v"])):
            if cu is None:
                y = _conv_bf16(x.reshape(B, T, H * D), w)
            else:  # per document, zero history at every boundary
                cuts = case.cu_seqlens
                y = torch.cat([_conv_bf16(x.reshape(B, T, H * D)[:, cuts[n]:cuts[n + 1]], w)
                               for n in range(len(cuts) - 1)], dim=1)
            post.append(y.reshape(B, T, H, D))
        xs = post
    o, ht = chunk_kda(xs[0], xs[1], xs[2], t["g"], t["beta"],
                      initial_state=t["h0"] if case.h0 else None, output_final_state=True,
                      use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True,
                      use_beta_sigmoid_in_kernel=True, safe_gate=True, lower_bound=case.lower_bound,
                      A_log=t["A_log"], dt_bias=t["dt_bias"], cu_seqlens=cu)
    res = {"o": o.detach().float().cpu(), "final_state": ht.detach().float().cpu()}
    if grads:
        loss = (o.float() * inp["do"].to(dev)).sum()
        if case.final_state_grad:
            loss = loss + (ht * inp["dht"].to(dev)).sum()
        loss.backward()
        for k in GRAD_KEYS:
            g = t[k].grad
            res["d_" + k] = (torch.zeros_like(t[k]) if g is None else g).detach().float().cpu()
    torch.cuda.synchronize()
    return res
