"""CPU checks of the C ABI: the library loads and exports every symbol the
header declares, and the buffer-size functions are consistent.  No kernel is
launched here (no GPU)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from sophia_b200 import _lib
from sophia_b200.build import build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def lib():
    build()
    return _lib.load()


def _header_symbols():
    text = open(os.path.join(ROOT, "include", "kda_b200.h")).read()
    return sorted(set(re.findall(r"\b(kda_b200_\w+)\s*\(", text)))


def test_header_symbols_are_bound(lib):
    syms = _header_symbols()
    assert syms, "no declarations found"
    assert sorted(_lib.SIGNATURES) == syms
    for name in syms:
        assert getattr(lib, name) is not None


def test_exported_symbols_match_header():
    build()
    cdll = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in _header_symbols():
        assert hasattr(cdll, name), name


def test_version_and_sizes(lib):
    assert b"sm_100a" in lib.kda_b200_version()
    tt, H, N = 8 * 4096, 16, 8
    saved = lib.kda_b200_saved_bytes(tt, H, N, 0)
    # W, U, Qt, Kb (bf16 token rows x128), M (x64); per chunk slot: v_new (64x128 tile),
    # the chunk-start state, the decays, A and L' (bf16 64x64 each) and the prologue
    # products (q, k, v bf16 64x128, the decay cumsum fp32 64x132, beta)
    mc = tt // 64 + N
    lower = tt * H * (4 * 128 + 64) * 2 + mc * H * (64 * 128 * 2 + 128 * 128 * 2 + 128 * 4 + 2 * 64 * 64 * 2 +
                                                    3 * 64 * 128 * 2 + 64 * 132 * 4 + 64 * 4)
    assert lower <= saved <= lower + 64 * 256
    assert lib.kda_b200_fwd_workspace_bytes(tt, H, N, 0, 1) < lib.kda_b200_fwd_workspace_bytes(tt, H, N, 0, 0)
    assert lib.kda_b200_bwd_workspace_bytes(tt, H, N, 0) > tt * H * 128 * 2 * 7


def test_invalid_arguments_are_rejected_without_launch(lib):
    # D != 128 is rejected before any CUDA call
    rc = lib.kda_b200_fwd(*([None] * 12), 1, 64, 2, 64, 1, 0.125, -5.0,
                          None, None, None, 0, None, 0, None)
    assert rc == _lib.KDA_ERR_UNSUPPORTED
    assert b"head dim" in lib.kda_b200_last_error()
    # null inputs
    rc = lib.kda_b200_fwd(*([None] * 12), 1, 64, 2, 128, 1, 0.125, -5.0,
                          None, None, None, 0, None, 0, None)
    assert rc == _lib.KDA_ERR_INVALID
    # lower bound outside [-5, 0)
    rc = lib.kda_b200_fwd(*([None] * 12), 1, 64, 2, 128, 1, 0.125, -6.0,
                          None, None, None, 0, None, 0, None)
    assert rc == _lib.KDA_ERR_INVALID and b"lower_bound" in lib.kda_b200_last_error()
