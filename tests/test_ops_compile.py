"""The custom-op boundary of the layer, without a GPU: under ``torch.compile``
every kernel call is a ``torch.library.custom_op`` with a fake implementation
and an autograd formula, so the seam traces with ``fullgraph=True`` (no graph
break) and shapes, dtypes and gradients propagate on meta tensors (Sophia
compiles its training model, ``ml/training/pretrain/engine/
sm120_graph_runner.py:71-75``).  Eager calls take a plain autograd.Function
over the same implementation (checked on the GPU)."""

from __future__ import annotations

import pytest
import torch

from sophia_b200 import ops

B, T, H, D = 2, 100, 2, 128


def _mk(*shape, dt=torch.bfloat16):
    return torch.empty(*shape, device="meta", dtype=dt).requires_grad_(True)


def _inputs(dt=torch.bfloat16):
    x = {n: _mk(B, T, H, D, dt=dt) for n in ("q", "k", "v", "g")}
    x["beta"] = _mk(B, T, H, dt=dt)
    x["A_log"] = _mk(H, dt=torch.float32)
    x["dt_bias"] = _mk(H * D, dt=torch.float32)
    for n in ("conv_q", "conv_k", "conv_v"):
        x[n] = _mk(H * D, 4, dt=torch.float32)
    x["h0"] = _mk(B, H, D, D, dt=torch.float32)
    return x


ARGS = ("q", "k", "v", "g", "beta", "A_log", "dt_bias", "conv_q", "conv_k", "conv_v", "h0")


def _traced(fn):
    return torch.compile(fn, backend="eager", fullgraph=True)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_layer_shapes_and_gradients_propagate(dt):
    x = _inputs(dt)
    o, ht = _traced(lambda *a: ops._layer(*a, None, D ** -0.5, -5.0, True))(*(x[n] for n in ARGS))
    assert o.shape == (B, T, H, D) and o.dtype == dt
    assert ht.shape == (B, H, D, D) and ht.dtype == torch.float32
    (o.float().sum() + ht.sum()).backward()
    for n in ARGS:
        assert x[n].grad is not None and x[n].grad.shape == x[n].shape and x[n].grad.dtype == x[n].dtype, n


def test_packed_and_inference_calls():
    x = _inputs()
    q1 = {n: _mk(1, 150, H, D) for n in ("q", "k", "v", "g")}
    cu = torch.empty(4, device="meta", dtype=torch.int32)
    h0 = _mk(3, H, D, D, dt=torch.float32)
    packed = _traced(lambda q, k, v, g, b, A, dtb, h, c: ops._layer(q, k, v, g, b, A, dtb, None, None, None, h, c,
                                                                    D ** -0.5, -5.0, True))
    o, ht = packed(q1["q"], q1["k"], q1["v"], q1["g"], _mk(1, 150, H), x["A_log"], x["dt_bias"], h0, cu)
    assert ht.shape == (3, H, D, D)
    o.float().sum().backward()
    assert h0.grad.shape == h0.shape and q1["q"].grad.shape == q1["q"].shape
    with torch.no_grad():  # no saved buffer when nothing needs gradients
        o, ht = _traced(lambda *a: ops._layer(*a, None, D ** -0.5, -5.0, False))(*(x[n] for n in ARGS))
    assert ht is None and o.shape == (B, T, H, D)


def test_compile_fullgraph_traces_the_seam():
    x = _inputs()

    def step(q, k, v, g, beta, A_log, dt_bias, cq, ck, cv, h0):
        o, ht = ops._layer(q, k, v, g, beta, A_log, dt_bias, cq, ck, cv, h0, None, D ** -0.5, -5.0, True)
        y = ops._gated_norm_fwd(o, g, torch.ones(D, device=q.device), 1e-5)
        return y.float().sum() + ht.sum()

    loss = torch.compile(step, backend="aot_eager", fullgraph=True)(*(x[n] for n in ARGS))
    loss.backward()
    for n in ARGS:
        assert x[n].grad is not None and x[n].grad.shape == x[n].shape, n


def test_decode_op_shapes():
    q = torch.empty(3, 1, H, D, device="meta", dtype=torch.float32)
    b = torch.empty(3, 1, H, device="meta", dtype=torch.float32)
    A = torch.empty(H, device="meta")
    dtb = torch.empty(H * D, device="meta")
    o, ht = ops._kda_recurrent(q, q, q, q, b, A, dtb, None, None, D ** -0.5, -5.0, True)  # the custom op itself
    assert o.shape == q.shape and o.dtype == torch.float32 and ht.shape == (3, H, D, D)
