"""Data-parallel step of the KDA layer: one process per GPU.

Sequences (or packed documents) are independent, so the layer shards by
sequence with no collective on the data path: rank r processes its contiguous
share of the batch.  The only exchange is one sum all-reduce of the layer's
weight gradients -- ShortConv taps (3 x H*128 x 4), ``A_log`` (H) and
``dt_bias`` (H*128), 26,640 floats at 16 heads -- flattened into one fp32
bucket in a fixed order, so every rank issues the same collective.  Step
times are reported as the maximum over ranks.

The reference has no distributed code; these helpers are the whole harness
(``bench.py`` runs them over NCCL, the tests over gloo on CPU).
"""

from __future__ import annotations

import torch

# order of the weight-gradient bucket
WEIGHT_KEYS = ("A_log", "dt_bias", "conv_q", "conv_k", "conv_v")


def shard(n_items: int, rank: int, world: int) -> slice:
    """Contiguous, balanced share of ``n_items`` for ``rank`` (the first
    ``n_items % world`` ranks take one extra item)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return slice(start, start + base + (1 if rank < extra else 0))


def bucket_numel(H: int, head_dim: int = 128) -> int:
    return H + H * head_dim + 3 * H * head_dim * 4


def grad_bucket(params: dict, out: torch.Tensor | None = None, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Flattens the weight gradients (zeros for a missing one) into one bucket
    (fp32 unless ``dtype`` says otherwise) in ``WEIGHT_KEYS`` order."""
    parts = []
    for k in WEIGHT_KEYS:
        p = params[k]
        g = p.grad if p.grad is not None else torch.zeros_like(p)
        parts.append(g.reshape(-1).to(out.dtype if out is not None else dtype))
    if out is None:
        return torch.cat(parts)
    torch.cat(parts, out=out)
    return out


def allreduce_bucket(bucket: torch.Tensor) -> torch.Tensor:
    """Sum of the bucket over all ranks (in place); a no-op without a process
    group of more than one rank."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(bucket, op=dist.ReduceOp.SUM)
    return bucket


def allreduce_bucket_async(bucket: torch.Tensor):
    """Starts the sum all-reduce of the bucket on the collective's own stream
    and returns its handle (``None`` without a multi-rank group).  The
    caller's stream keeps issuing work (the next micro-batch computes while
    the gradients cross NVLink); ``handle.wait()`` makes the current stream
    wait for the reduction before anything reads or rewrites the bucket."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        return dist.all_reduce(bucket, op=dist.ReduceOp.SUM, async_op=True)
    return None


def scatter_bucket(bucket: torch.Tensor, params: dict) -> None:
    """Writes the (reduced) bucket back into the parameters' ``.grad``."""
    off = 0
    for k in WEIGHT_KEYS:
        p = params[k]
        n = p.numel()
        g = bucket[off:off + n].view_as(p).to(p.dtype)
        if p.grad is None:
            p.grad = g.clone()
        else:
            p.grad.copy_(g)
        off += n


def max_over_ranks(value: float, device: torch.device | str = "cpu") -> float:
    """Maximum of a per-rank scalar (a step time) over all ranks."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1):
        return float(value)
    t = torch.tensor([float(value)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
