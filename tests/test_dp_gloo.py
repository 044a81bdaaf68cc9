"""The data-parallel harness (sophia_b200.dp) on CPU with two gloo ranks.

Each rank runs the CPU oracle of the layer (forward + backward, fp64) on its
shard of a 5-sequence batch, flattens the weight gradients into the bucket and
all-reduces it; the reduced bucket must equal the gradient of the whole batch
computed in one process, and the max-over-ranks timing must agree on every
rank.  Ranks are started with the spawn method."""

from __future__ import annotations

import os
import socket
import sys

import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _inputs():
    sys.path.insert(0, os.path.join(HERE, "golden"))
    from cases import Case, make_case_inputs
    case = Case("dp", B=5, T=40, H=2, random_gate_params=True, seed=77)
    return make_case_inputs(case)


def _layer_grads(inp, rows: slice) -> dict:
    from oracle.kda_oracle import kda_layer
    from sophia_b200 import dp
    leaves = {k: inp[k].double().clone().requires_grad_(True) for k in dp.WEIGHT_KEYS}
    x = {k: inp[k][rows].double() for k in ("q", "k", "v", "g", "beta", "do")}
    out = kda_layer(x["q"], x["k"], x["v"], x["g"], x["beta"], leaves["A_log"], leaves["dt_bias"],
                    conv_weights=(leaves["conv_q"], leaves["conv_k"], leaves["conv_v"]))
    (out.o * x["do"]).sum().backward()
    return leaves


def _rank(rank: int, world: int, port: int, result_dir: str) -> None:
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    from sophia_b200 import dp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        inp = _inputs()
        leaves = _layer_grads(inp, dp.shard(inp["q"].shape[0], rank, world))
        bucket = dp.allreduce_bucket(dp.grad_bucket(leaves, dtype=torch.float64))
        slowest = dp.max_over_ranks(1.0 + rank)
        torch.save({"bucket": bucket, "max": slowest}, os.path.join(result_dir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shards_cover_the_batch_once():
    from sophia_b200 import dp
    for n in (0, 1, 5, 320):
        for world in (1, 2, 3, 8):
            idx = [i for r in range(world) for i in range(n)[dp.shard(n, r, world)]]
            assert idx == list(range(n))
    with pytest.raises(ValueError):
        dp.shard(4, 2, 2)


def test_two_gloo_ranks_reduce_to_the_single_process_gradient(tmp_path):
    from sophia_b200 import dp
    world = 2
    mp.start_processes(_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    full = dp.grad_bucket(_layer_grads(_inputs(), slice(None)), dtype=torch.float64)
    for r in range(world):
        res = torch.load(os.path.join(tmp_path, f"rank{r}.pt"))
        torch.testing.assert_close(res["bucket"], full, rtol=1e-10, atol=1e-12)
        assert res["max"] == float(world)
    # the reduced bucket scatters back into the parameters' gradients
    params = {k: torch.zeros_like(_inputs()[k]).double() for k in dp.WEIGHT_KEYS}
    dp.scatter_bucket(full, params)
    assert torch.equal(dp.grad_bucket(params, dtype=torch.float64), full)
