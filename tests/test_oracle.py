"""Pins the CPU oracle to the golden fixtures made by the reference's modules."""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from cases import CASES, make_cfg0_inputs, make_inputs
from oracle.chunk_index import (chunk_table_with_true_ids, prepare_chunk_indices,
                                prepare_chunk_offsets)
from oracle.kda_oracle import kda_layer
from oracle_runner import run_oracle

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return np.load(os.path.join(GOLDEN, f"{name}.npz"))


@pytest.mark.parametrize("name", sorted(CASES))
def test_inputs_regenerate_bit_identically(name):
    gold = json.loads(str(_load(name)["input_sums"]))
    inp = make_inputs(CASES[name])
    for k, v in gold.items():
        assert float(inp[k].double().sum()) == v, k


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_matches_reference_golden(name):
    gold = _load(name)
    res = run_oracle(CASES[name], dtype=torch.float64)
    for key in ("o", "final_state"):
        np.testing.assert_allclose(res[key].numpy(), gold[key], rtol=1e-4, atol=2e-5,
                                   err_msg=key)
    for key in [k for k in gold.files if k.startswith("d_")]:
        ref = gold[key]
        got = res[key].numpy()
        scale = max(1e-6, float(np.abs(ref).max()))
        np.testing.assert_allclose(got, ref, rtol=1e-3, atol=2e-5 * scale, err_msg=key)


def test_oracle_fp32_mode_matches_golden_to_1e5():
    gold = _load("small")
    res = run_oracle(CASES["small"], dtype=torch.float32, grads=False)
    np.testing.assert_allclose(res["o"].numpy(), gold["o"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(res["final_state"].numpy(), gold["final_state"],
                               rtol=1e-5, atol=1e-5)


def test_oracle_cfg0_matches_reference():
    gold = _load("cfg0")
    inp = make_cfg0_inputs()
    sums = json.loads(str(gold["input_sums"]))
    for k, v in sums.items():
        assert float(inp[k].double().sum()) == v, k
    with torch.no_grad():
        out = kda_layer(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"],
                        inp["A_log"], inp["dt_bias"],
                        conv_weights=(inp["conv_q"], inp["conv_k"], inp["conv_v"]),
                        compute_dtype=torch.float32)
    np.testing.assert_allclose(out.o[:, ::16].numpy(), gold["o_slice"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(out.final_state[:, :, ::4].numpy(), gold["state_slice"],
                               rtol=1e-5, atol=1e-5)
    o64, s64 = out.o.double(), out.final_state.double()
    np.testing.assert_allclose([o64.sum(), o64.abs().sum(), (o64 ** 2).sum()],
                               gold["o_stats"], rtol=1e-4, atol=1e-3)
    np.testing.assert_allclose([s64.sum(), s64.abs().sum(), (s64 ** 2).sum()],
                               gold["state_stats"], rtol=1e-4, atol=1e-3)


def test_packed_oracle_equals_unpacked_runs():
    case = CASES["varlen"]
    inp = make_inputs(case)
    cu = case.cu_seqlens
    packed = kda_layer(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], inp["A_log"],
                       inp["dt_bias"], conv_weights=(inp["conv_q"], inp["conv_k"], inp["conv_v"]),
                       initial_state=inp["h0"], cu_seqlens=torch.tensor(cu))
    for n in range(len(cu) - 1):
        sl = slice(cu[n], cu[n + 1])
        one = kda_layer(inp["q"][:, sl], inp["k"][:, sl], inp["v"][:, sl], inp["g"][:, sl],
                        inp["beta"][:, sl], inp["A_log"], inp["dt_bias"],
                        conv_weights=(inp["conv_q"], inp["conv_k"], inp["conv_v"]),
                        initial_state=inp["h0"][n:n + 1])
        torch.testing.assert_close(packed.o[:, sl], one.o, rtol=0, atol=0)
        torch.testing.assert_close(packed.final_state[n:n + 1], one.final_state, rtol=0, atol=0)


def test_chunk_index_restatement_known_answers():
    cu = [0, 37, 101, 150, 214]
    np.testing.assert_array_equal(prepare_chunk_offsets(cu, 64), [0, 1, 2, 3, 4])
    np.testing.assert_array_equal(prepare_chunk_indices(cu, 64),
                                  [[0, 0], [1, 0], [2, 0], [3, 0]])
    cu = [0, 64, 65, 200]
    np.testing.assert_array_equal(prepare_chunk_offsets(cu, 64), [0, 1, 2, 5])
    np.testing.assert_array_equal(prepare_chunk_indices(cu, 64),
                                  [[0, 0], [1, 0], [2, 0], [2, 1], [2, 2]])
    # an empty sequence owns no chunk; the restated table keeps FLA's id quirk
    cu = [0, 10, 10, 80]
    np.testing.assert_array_equal(prepare_chunk_indices(cu, 64), [[0, 0], [1, 0], [1, 1]])
    np.testing.assert_array_equal(chunk_table_with_true_ids(cu, 64), [[0, 0], [2, 0], [2, 1]])


def test_chunk_index_restatement_matches_fla():
    """The restated integer bookkeeping equals flash-linear-attention's own
    prepare_chunk_indices / prepare_chunk_offsets (fla/ops/utils/index.py:
    138-158, the reference's pinned CUDA dependency) element for element, on
    hand-made tables (empty, one-token, chunk-aligned documents) and random
    ones, for chunk sizes 64 and 32."""
    index = pytest.importorskip("fla.ops.utils.index")
    rng = np.random.default_rng(11)
    tables = [[0, 37, 101, 150, 214], [0, 64, 65, 200], [0, 10, 10, 80], [0, 1], [0, 64], [0, 0, 0, 5],
              [0, 1, 65, 65, 200, 264, 264 + 4096]]
    for _ in range(20):
        lens = rng.integers(0, 300, size=int(rng.integers(1, 60)))
        tables.append([0] + np.cumsum(lens).tolist())
    for cu in tables:
        cu_t = torch.tensor(cu, dtype=torch.long)
        for chunk in (64, 32):
            np.testing.assert_array_equal(prepare_chunk_offsets(cu, chunk),
                                          index.prepare_chunk_offsets(cu_t, chunk).numpy())
            np.testing.assert_array_equal(prepare_chunk_indices(cu, chunk).reshape(-1, 2),
                                          index.prepare_chunk_indices(cu_t, chunk).numpy().reshape(-1, 2))
