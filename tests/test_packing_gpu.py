"""Capture-safe document resets for packed pretraining windows
(``sophia_b200.document_cu_seqlens``): the device-built table follows the
boundary rule (a document starts at every window start and after every EOS),
and a whole packed fwd+bwd step -- table, layer, backward -- captured in one
CUDA graph and replayed on new token windows gives the eager step's bits."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

EOS = 2


def _expected(tokens: np.ndarray, eos: int, cap: int):
    """The boundary rule restated: starts at t % window == 0 or after an EOS."""
    W = tokens.shape[-1]
    flat = tokens.reshape(-1)
    starts = [t for t in range(flat.size) if t % W == 0 or flat[t - 1] == eos]
    kept = starts[:cap]
    return kept + [flat.size] * (cap + 1 - len(kept)), len(starts)


def _windows(gen, n, W, mean_doc):
    tok = gen.integers(3, 1000, size=(n, W)).astype(np.int32)
    mask = gen.random((n, W)) < 1.0 / mean_doc
    tok[mask] = EOS
    return tok


@pytest.mark.parametrize("n,W,mean_doc,cap", [(1, 4096, 300, 64), (16, 4096, 500, 256), (3, 1000, 7, 50),
                                              (2, 777, 40, 1)])
def test_document_bounds_follow_the_rule(n, W, mean_doc, cap):
    from sophia_b200 import document_cu_seqlens
    gen = np.random.default_rng(n * 1000 + W)
    tok = _windows(gen, n, W, mean_doc)
    tok[0, -1] = EOS          # an EOS closing a window
    tok[-1, 5:8] = EOS        # one-token documents
    cu, nd = document_cu_seqlens(torch.from_numpy(tok).cuda(), EOS, cap)
    want, count = _expected(tok, EOS, cap)
    assert cu.cpu().tolist() == want
    assert int(nd.item()) == count


def test_graph_captured_packed_step_equals_eager():
    from sophia_b200 import _lib, document_cu_seqlens, kda_layer
    n, W, H, cap = 2, 1024, 2, 64
    TT = n * W
    gen = torch.Generator().manual_seed(7)
    dev = "cuda"
    mk = lambda *s, std=1.0: (torch.randn(*s, generator=gen) * std).to(dev)  # noqa: E731
    leaves = {"q": mk(1, TT, H, 128).bfloat16(), "k": mk(1, TT, H, 128).bfloat16(),
              "v": mk(1, TT, H, 128).bfloat16(), "g": mk(1, TT, H, 128).bfloat16(), "beta": mk(1, TT, H).bfloat16(),
              "A_log": mk(H, std=0.5), "dt_bias": mk(H * 128, std=0.1), "conv_q": mk(H * 128, 4, std=0.5),
              "conv_k": mk(H * 128, 4, std=0.5), "conv_v": mk(H * 128, 4, std=0.5)}
    for t in leaves.values():
        t.requires_grad_(True)
    do = mk(1, TT, H, 128).bfloat16()
    rng = np.random.default_rng(3)
    tok_a, tok_b = _windows(rng, n, W, 150), _windows(rng, n, W, 90)
    tokens = torch.from_numpy(tok_a).to(dev)
    names = ("q", "k", "v", "g", "beta", "A_log", "dt_bias", "conv_q", "conv_k", "conv_v")

    def step(tok):
        cu, _ = document_cu_seqlens(tok, EOS, cap)
        o, ht = kda_layer(*(leaves[k] for k in names[:5]), *(leaves[k] for k in names[5:]), cu_seqlens=cu,
                          output_final_state=True)
        o.backward(do)
        return o, ht

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            for t in leaves.values():
                t.grad = None
            step(tokens)
    torch.cuda.current_stream().wait_stream(side)
    for t in leaves.values():
        t.grad = None
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        o_g, ht_g = step(tokens)
    static_grads = {k: leaves[k].grad for k in names}  # rewritten by every replay

    eager = {k: v.detach().clone().requires_grad_(True) for k, v in leaves.items()}
    for tok in (tok_a, tok_b):
        tokens.copy_(torch.from_numpy(tok))
        graph.replay()
        torch.cuda.synchronize()
        got = {"o": o_g.clone(), "ht": ht_g.clone(), **{k: static_grads[k].clone() for k in names}}
        for t in eager.values():
            t.grad = None
        cu = torch.tensor(_expected(tok, EOS, cap)[0], dtype=torch.int32, device=dev)
        o, ht = kda_layer(*(eager[k] for k in names[:5]), *(eager[k] for k in names[5:]), cu_seqlens=cu,
                          output_final_state=True)
        o.backward(do)
        want = {"o": o.detach(), "ht": ht.detach(), **{k: eager[k].grad.clone() for k in names}}
        for k in want:
            assert torch.equal(got[k], want[k]), k
    assert _lib.device_error(reset=True) == 0
    del graph
