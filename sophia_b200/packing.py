"""Document resets for packed pretraining windows, capture-safe.

Sophia's pretraining data path copies fixed ``[1, 4096]`` int32 token windows
into static buffers and replays a captured CUDA graph over them
(``ml/training/pretrain/engine/sm120_graph_runner.py:244-259``); each window
runs as one sequence, so the KDA state flows across document ends.
``document_cu_seqlens`` derives the packed layer's ``cu_seqlens`` from the
tokens on the device -- a document starts at every window start and after
every EOS token -- with a fixed capacity, so the layer call that follows
(``kda_layer(..., cu_seqlens=cu)`` on the flattened windows) has a static
shape and the whole step can be captured once and replayed on new windows.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _lib
from .ops import _stream

__all__ = ["document_cu_seqlens"]


@torch.library.custom_op("sophia_b200::doc_cu_seqlens", mutates_args=(), device_types="cuda")
def _doc_cu_seqlens(tokens: Tensor, window: int, eos_id: int, capacity: int) -> tuple[Tensor, Tensor]:
    tok = tokens.to(torch.int32).contiguous()
    cu = torch.empty(capacity + 1, device=tokens.device, dtype=torch.int32)
    n_docs = torch.empty(1, device=tokens.device, dtype=torch.int32)
    _lib.check(_lib.load().kda_b200_doc_cu_seqlens(tok.data_ptr() if tok.numel() else None, tok.numel(), int(window),
                                                   int(eos_id), int(capacity), cu.data_ptr(), n_docs.data_ptr(),
                                                   _stream()))
    return cu, n_docs


@_doc_cu_seqlens.register_fake
def _(tokens, window, eos_id, capacity):
    return tokens.new_empty((capacity + 1,), dtype=torch.int32), tokens.new_empty((1,), dtype=torch.int32)


def document_cu_seqlens(tokens: Tensor, eos_id: int, capacity: int) -> tuple[Tensor, Tensor]:
    """tokens: int CUDA tensor ``[windows, window_len]`` (or 1-D, one window).
    Returns ``(cu_seqlens [capacity + 1] int32, n_docs [1] int32)``, both on the
    device: document starts in token order over the flattened windows, then
    ``tokens.numel()`` in every unused entry (empty sequences).  ``n_docs`` is
    the true count; documents past the capacity keep no reset of their own.
    No host synchronisation: safe inside CUDA-graph capture."""
    if not tokens.is_cuda:
        raise RuntimeError("document_cu_seqlens runs on the CUDA kernels only")
    if tokens.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"tokens must be an integer tensor, got {tokens.dtype}")
    if capacity < 1:
        raise ValueError("capacity must be >= 1")
    window = tokens.shape[-1] if tokens.dim() > 0 else 1
    return _doc_cu_seqlens(tokens.reshape(-1), int(window), int(eos_id), int(capacity))
