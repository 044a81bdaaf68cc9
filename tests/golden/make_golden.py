"""Generates the KDA golden fixtures from Sophia's own reference modules.

Usage::

    python tests/golden/make_golden.py --reference <path to the Sophia checkout>

The script imports ``ml.runtime.model.attention`` from the given checkout and
runs, for every case of ``cases.py``:

* ``CausalDepthwiseConv1d.forward`` (``attention.py:32-60``) on q/k/v unless
  the case is post-conv,
* ``SophiaKDA._reference_kda`` (``attention.py:260-294``) -- the reference's
  own per-token recurrence, float32 inside,
* torch autograd of ``sum(o * dO) + sum(S * dS)`` for every gradient,

one document at a time for packed cases (state and conv history reset at each
boundary).  Results go to ``tests/golden/<case>.npz``; configuration 0 of the
benchmark (the full projections, T=512) goes to ``tests/golden/cfg0.npz`` as
strided slices plus whole-tensor sums; ``SophiaKDA.forward`` end to end goes to
``module_forward.npz`` and its cached prefill / continuation / decode path to
``module_cache.npz``.  The fixtures are small enough to
commit; the reference checkout is only needed to regenerate them.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from cases import CASES, CFG0, make_cfg0_inputs, make_inputs  # noqa: E402


def _module(reference_root: str, H: int, D: int, lower_bound: float):
    sys.path.insert(0, reference_root)
    from ml.runtime.model.attention import CausalDepthwiseConv1d, SophiaKDA
    from ml.runtime.model.config import ModelArgs

    args = ModelArgs(dim=64, num_heads=H, head_dim=D, kda_decay_rank=16,
                     kda_output_gate_rank=16, mla_q_rank=16, mla_kv_rank=16,
                     kda_backend="reference", use_cache=False,
                     kda_decay_lower_bound=lower_bound, vocab_size=128,
                     ffn_hidden=128, n_layers=4, max_batch_size=2)
    return SophiaKDA(args), CausalDepthwiseConv1d


def _input_sums(inputs: dict[str, torch.Tensor]) -> dict[str, float]:
    return {k: float(v.double().sum()) for k, v in inputs.items()}


def run_case(reference_root: str, case) -> dict[str, np.ndarray]:
    inp = make_inputs(case)
    mod, Conv = _module(reference_root, case.H, case.D, case.lower_bound)
    HD = case.H * case.D
    leaves = {k: v.clone().requires_grad_(True) for k, v in inp.items()
              if k not in ("do", "dht")}
    # the module's own parameters are the differentiable leaves
    mod.A_log = torch.nn.Parameter(inp["A_log"].clone())
    mod.dt_bias = torch.nn.Parameter(inp["dt_bias"].clone())
    leaves["A_log"], leaves["dt_bias"] = mod.A_log, mod.dt_bias
    convs = []
    for name in ("conv_q", "conv_k", "conv_v"):
        c = Conv(HD, 4)
        c.weight = torch.nn.Parameter(inp[name].clone())
        leaves[name] = c.weight
        convs.append(c)

    B = case.B
    if case.cu_seqlens is None:
        docs = [(b, 0, case.T) for b in range(B)]
    else:
        cu = case.cu_seqlens
        docs = [(0, cu[n], cu[n + 1]) for n in range(len(cu) - 1)]
    o_full = torch.zeros(B, case.T, case.H, case.D)
    states = []
    loss = torch.zeros((), dtype=torch.float32)
    for n, (b, bos, eos) in enumerate(docs):
        sl = slice(bos, eos)
        xs = [leaves[k][b:b + 1, sl] for k in ("q", "k", "v")]
        if case.conv:
            post = []
            for x, c in zip(xs, convs):
                y, _ = c(x.reshape(1, eos - bos, HD))
                post.append(y.reshape(1, eos - bos, case.H, case.D))
            xs = post
        h0 = leaves["h0"][n:n + 1] if case.h0 else None
        o, S = mod._reference_kda(xs[0], xs[1], xs[2], leaves["g"][b:b + 1, sl],
                                  leaves["beta"][b:b + 1, sl], h0)
        loss = loss + (o * inp["do"][b:b + 1, sl]).sum()
        if case.final_state_grad:
            loss = loss + (S * inp["dht"][n:n + 1]).sum()
        o_full[b:b + 1, sl] = o.detach()
        states.append(S.detach())
    loss.backward()
    out = {"o": o_full.numpy(), "final_state": torch.cat(states).numpy()}
    for k, v in leaves.items():
        grad = v.grad if v.grad is not None else torch.zeros_like(v)
        out["d_" + k] = grad.detach().numpy()
    out["input_sums"] = np.array(json.dumps(_input_sums(inp)))
    return out


def run_cfg0(reference_root: str) -> dict[str, np.ndarray]:
    inp = make_cfg0_inputs()
    c = CFG0
    mod, Conv = _module(reference_root, c["H"], c["D"], -5.0)
    with torch.no_grad():
        mod.A_log.zero_()
        mod.dt_bias.zero_()
        HD = c["H"] * c["D"]
        post = []
        for name, key in (("conv_q", "q"), ("conv_k", "k"), ("conv_v", "v")):
            conv = Conv(HD, 4)
            conv.weight.copy_(inp[name])
            y, _ = conv(inp[key].reshape(c["B"], c["T"], HD))
            post.append(y.reshape(c["B"], c["T"], c["H"], c["D"]))
        o, S = mod._reference_kda(post[0], post[1], post[2], inp["g"], inp["beta"], None)
    o64, S64 = o.double(), S.double()
    return {
        "o_slice": o[:, ::16].numpy(),
        "state_slice": S[:, :, ::4].numpy(),
        "o_stats": np.array([o64.sum(), o64.abs().sum(), (o64 ** 2).sum()]),
        "state_stats": np.array([S64.sum(), S64.abs().sum(), (S64 ** 2).sum()]),
        "input_sums": np.array(json.dumps(_input_sums(inp))),
    }


MODULE_CFG = dict(B=2, T=70, dim=64, H=2, D=128, pad=6, seed=2024)


def run_module(reference_root: str) -> dict[str, np.ndarray]:
    """SophiaKDA.forward end to end (attention.py:373-420, fp32, reference
    backend): projections, ShortConv, decay/beta logits with a left-padded row
    (pad mask), the recurrence, gated output norm and o_proj; then the
    backward of <out, dout> for the input and every parameter."""
    c = MODULE_CFG
    torch.manual_seed(c["seed"])
    mod, _ = _module(reference_root, c["H"], c["D"], -5.0)
    gen = torch.Generator().manual_seed(c["seed"])
    with torch.no_grad():
        for name in ("q_proj", "k_proj", "v_proj", "decay_down", "beta_proj"):
            w = getattr(mod, name).weight
            w.copy_(torch.randn(w.shape, generator=gen) * 0.15)
        w = mod.decay_up.weight
        w.copy_(torch.randn(w.shape, generator=gen) * 0.3)
        for name in ("q_conv", "k_conv", "v_conv"):
            w = getattr(mod, name).weight
            w.copy_(torch.randn(w.shape, generator=gen) * 0.5)
    x = torch.randn(c["B"], c["T"], c["dim"], generator=gen).requires_grad_(True)
    mask = torch.ones(c["B"], c["T"], dtype=torch.bool)
    mask[1, :c["pad"]] = False
    mod._pad_mask = mask
    out = mod(x)
    dout = torch.randn(out.shape, generator=gen)
    (out * dout).sum().backward()
    res = {"x": x.detach().numpy(), "mask": mask.numpy(), "dout": dout.numpy(), "out": out.detach().numpy(),
           "d_x": x.grad.numpy()}
    for name, prm in mod.named_parameters():
        res["param." + name] = prm.detach().numpy()
        res["grad." + name] = (prm.grad if prm.grad is not None else torch.zeros_like(prm)).numpy()
    return res


CACHE_CFG = dict(B=2, dim=64, H=2, D=128, pad=5, prefill=70, chunk=9, decode=4, seed=2025)


def _cache_module(reference_root: str, use_cache: bool):
    sys.path.insert(0, reference_root)
    from ml.runtime.model.attention import SophiaKDA
    from ml.runtime.model.config import ModelArgs

    c = CACHE_CFG
    args = ModelArgs(dim=c["dim"], num_heads=c["H"], head_dim=c["D"], kda_decay_rank=16,
                     kda_output_gate_rank=16, mla_q_rank=16, mla_kv_rank=16, kda_backend="reference",
                     use_cache=use_cache, kda_decay_lower_bound=-5.0, vocab_size=128, ffn_hidden=128,
                     n_layers=4, max_batch_size=c["B"])
    return SophiaKDA(args)


def run_cache(reference_root: str) -> dict[str, np.ndarray]:
    """The cached path of SophiaKDA.forward (attention.py:373-420 with
    use_cache): a left-padded prefill (start_pos 0, pad mask), a 9-token
    continuation (start_pos 70: conv history from conv_state, initial state from
    recurrent_state) and four one-token decode steps, fp32, reference backend;
    plus the same 83 tokens in one uncached call.  Records every call's output
    and the two cache buffers after the prefill and at the end."""
    c = CACHE_CFG
    torch.manual_seed(c["seed"])
    mod = _cache_module(reference_root, True)
    gen = torch.Generator().manual_seed(c["seed"])
    with torch.no_grad():
        for name, prm in mod.named_parameters():
            if name in ("A_log", "dt_bias"):
                continue
            prm.copy_(torch.randn(prm.shape, generator=gen) * (0.5 if "conv" in name else 0.15))
        mod.A_log.copy_(torch.randn(mod.A_log.shape, generator=gen) * 0.5)
    total = c["prefill"] + c["chunk"] + c["decode"]
    x = torch.randn(c["B"], total, c["dim"], generator=gen)
    mask = torch.ones(c["B"], total, dtype=torch.bool)
    mask[1, :c["pad"]] = False
    res = {"x": x.numpy(), "mask": mask.numpy()}
    for name, prm in mod.named_parameters():
        res["param." + name] = prm.detach().numpy()
    with torch.no_grad():
        mod._pad_mask = mask
        p0 = c["prefill"]
        res["out.prefill"] = mod(x[:, :p0], start_pos=0).numpy()
        res["state.prefill.recurrent"] = mod.recurrent_state.clone().numpy()
        res["state.prefill.conv"] = mod.conv_state.clone().numpy()
        res["out.chunk"] = mod(x[:, p0:p0 + c["chunk"]], start_pos=p0).numpy()
        outs = []
        for i in range(c["decode"]):
            pos = p0 + c["chunk"] + i
            outs.append(mod(x[:, pos:pos + 1], start_pos=pos))
        res["out.decode"] = torch.cat(outs, dim=1).numpy()
        res["state.final.recurrent"] = mod.recurrent_state.clone().numpy()
        res["state.final.conv"] = mod.conv_state.clone().numpy()
        full = _cache_module(reference_root, False)
        full.load_state_dict(mod.state_dict(), strict=False)
        full._pad_mask = mask
        res["out.full"] = full(x, start_pos=0).numpy()
    cached = np.concatenate([res["out.prefill"], res["out.chunk"], res["out.decode"]], axis=1)
    np.testing.assert_allclose(cached, res["out.full"], rtol=1e-4, atol=1e-5)  # the reference's own invariant
    return res


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of the Sophia checkout (contains ml/)")
    ap.add_argument("--out", default=str(HERE))
    a = ap.parse_args()
    torch.set_num_threads(max(1, torch.get_num_threads()))
    for name, case in CASES.items():
        np.savez_compressed(Path(a.out) / f"{name}.npz", **run_case(a.reference, case))
        print("wrote", name)
    np.savez_compressed(Path(a.out) / "cfg0.npz", **run_cfg0(a.reference))
    print("wrote cfg0")
    np.savez_compressed(Path(a.out) / "module_forward.npz", **run_module(a.reference))
    print("wrote module_forward")
    np.savez_compressed(Path(a.out) / "module_cache.npz", **run_cache(a.reference))
    print("wrote module_cache")


if __name__ == "__main__":
    main()
