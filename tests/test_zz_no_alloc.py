"""The forward entry point that allocates nothing (kda_b200_fwd_noalloc).

Some callers cannot allocate device memory: a host binding (cgo, JNI, a C
serving loop) with no device allocator of its own, or a process that reserves
all device memory at start-up and forbids later allocations.  For them the
library keeps a static 64 MiB device scratch array.  These tests call that
entry point through the C ABI and check it against kda_b200_fwd (which gets a
caller-provided workspace) on two calls in a row, with the tolerance of the
other parity tests.  The file is named to be collected last.
"""

from __future__ import annotations

import pytest
import torch

from kda_cuda_runner import ATOL, RTOL

pytestmark = pytest.mark.gpu


def _inputs(B, T, H, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rn = lambda *s, std=1.0: torch.randn(*s, device="cuda", generator=g) * std  # noqa: E731
    x = {k: rn(B, T, H, 128).to(torch.bfloat16).contiguous() for k in ("q", "k", "v", "g")}
    x["beta"] = rn(B, T, H).to(torch.bfloat16).contiguous()
    x["A_log"] = rn(H, std=0.5)
    x["dt_bias"] = rn(H * 128, std=0.5)
    for c in ("conv_q", "conv_k", "conv_v"):
        x[c] = rn(H * 128, 4, std=0.5)
    x["h0"] = rn(B, H, 128, 128, std=0.1)
    return x


def _args(x, B, T, H):
    p = lambda t: t.data_ptr()  # noqa: E731
    return [p(x["q"]), p(x["k"]), p(x["v"]), p(x["g"]), p(x["beta"]), p(x["A_log"]), p(x["dt_bias"]),
            p(x["conv_q"]), p(x["conv_k"]), p(x["conv_v"]), p(x["h0"]), None, B, T, H, 128, B, 128 ** -0.5, -5.0]


def _close(a, b):
    torch.testing.assert_close(a.float(), b.float(), rtol=RTOL, atol=ATOL)


def test_noalloc_forward_matches_workspace_forward_twice():
    from sophia_b200 import _lib
    lib = _lib.load()
    B, T, H = 2, 200, 4
    x = _inputs(B, T, H, seed=5)
    stream = torch.cuda.current_stream().cuda_stream
    o_ref = torch.empty_like(x["q"])
    ht_ref = torch.empty(B, H, 128, 128, device="cuda")
    ws = torch.empty(lib.kda_b200_fwd_workspace_bytes(B * T, H, B, 0, 0), device="cuda", dtype=torch.uint8)
    _lib.check(lib.kda_b200_fwd(*_args(x, B, T, H), o_ref.data_ptr(), ht_ref.data_ptr(), None, 0,
                                ws.data_ptr(), ws.numel(), stream))
    for _ in range(2):
        o = torch.full_like(x["q"], float("nan"))
        ht = torch.full((B, H, 128, 128), float("nan"), device="cuda")
        _lib.check(lib.kda_b200_fwd_noalloc(*_args(x, B, T, H), o.data_ptr(), ht.data_ptr(), stream))
        torch.cuda.synchronize()
        _close(o, o_ref)
        _close(ht, ht_ref)
    assert _lib.device_error(reset=True) == 0


def test_noalloc_rejects_problems_beyond_the_static_scratch():
    from sophia_b200 import _lib
    lib = _lib.load()
    B, T, H = 8, 4096, 16  # needs far more than the 64 MiB scratch
    x = _inputs(1, 64, 1, seed=6)
    args = _args(x, B, T, H)
    rc = lib.kda_b200_fwd_noalloc(*args, x["q"].data_ptr(), None, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.KDA_ERR_INVALID
    assert b"static scratch" in lib.kda_b200_last_error()


def test_noalloc_packed_forward_matches_workspace_forward_twice():
    # B = 1 with cu_seqlens over three unequal documents: the chunk table and the
    # chunk-to-sequence map are carved from the static scratch as well
    from sophia_b200 import _lib
    lib = _lib.load()
    H, bounds = 4, [0, 37, 150, 290]
    N, T = len(bounds) - 1, bounds[-1]
    x = _inputs(1, T, H, seed=7)
    x["h0"] = (torch.randn(N, H, 128, 128, device="cuda", generator=torch.Generator(device="cuda").manual_seed(8))
               * 0.1)
    cu = torch.tensor(bounds, device="cuda", dtype=torch.int32)
    args = _args(x, 1, T, H)
    args[11], args[16] = cu.data_ptr(), N
    stream = torch.cuda.current_stream().cuda_stream
    o_ref = torch.empty_like(x["q"])
    ht_ref = torch.empty(N, H, 128, 128, device="cuda")
    ws = torch.empty(lib.kda_b200_fwd_workspace_bytes(T, H, N, 1, 0), device="cuda", dtype=torch.uint8)
    _lib.check(lib.kda_b200_fwd(*args, o_ref.data_ptr(), ht_ref.data_ptr(), None, 0, ws.data_ptr(), ws.numel(),
                                stream))
    for _ in range(2):
        o = torch.full_like(x["q"], float("nan"))
        ht = torch.full((N, H, 128, 128), float("nan"), device="cuda")
        _lib.check(lib.kda_b200_fwd_noalloc(*args, o.data_ptr(), ht.data_ptr(), stream))
        torch.cuda.synchronize()
        _close(o, o_ref)
        _close(ht, ht_ref)
    assert _lib.device_error(reset=True) == 0
