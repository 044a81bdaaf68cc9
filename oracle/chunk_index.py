"""CPU oracle for packed-sequence chunk indexing (TEST INFRASTRUCTURE ONLY).

Restates, in numpy, the integer bookkeeping the reference's CUDA dependency
(flash-linear-attention 0.5.x, pinned 0.5.2 by Sophia's ``requirements.txt:17``)
uses for ``cu_seqlens`` packing:

* ``prepare_chunk_indices`` -- ``fla/ops/utils/index.py:138-149``: one
  ``(sequence id, chunk id within the sequence)`` row per chunk, chunks of
  ``chunk_size`` tokens, the last chunk of a sequence possibly partial.  The
  sequence id is recovered as ``cumsum(chunk_id == 0) - 1``, so a sequence of
  length zero owns no row and shifts no id (ids count non-empty sequences).
* ``prepare_chunk_offsets`` -- ``fla/ops/utils/index.py:152-158``: exclusive
  prefix sum of ``ceil(len / chunk_size)``.

The CUDA path builds the same tables on the device; the tests compare them
element for element.
"""

from __future__ import annotations

import numpy as np


def prepare_lens(cu_seqlens) -> np.ndarray:
    cu = np.asarray(cu_seqlens, dtype=np.int64)
    return cu[1:] - cu[:-1]


def prepare_chunk_offsets(cu_seqlens, chunk_size: int) -> np.ndarray:
    lens = prepare_lens(cu_seqlens)
    n_chunks = (lens + chunk_size - 1) // chunk_size
    return np.concatenate([[0], np.cumsum(n_chunks)]).astype(np.int64)


def prepare_chunk_indices(cu_seqlens, chunk_size: int) -> np.ndarray:
    lens = prepare_lens(cu_seqlens)
    n_chunks = (lens + chunk_size - 1) // chunk_size
    idx = np.concatenate([np.arange(n, dtype=np.int64) for n in n_chunks]
                         + [np.zeros(0, dtype=np.int64)])
    seq = np.cumsum(idx == 0) - 1
    return np.stack([seq, idx], axis=1).astype(np.int64)


def chunk_table_with_true_ids(cu_seqlens, chunk_size: int) -> np.ndarray:
    """``(sequence id, chunk id)`` per chunk where the sequence id is the
    position in ``cu_seqlens`` (empty sequences keep their slot).  Identical to
    ``prepare_chunk_indices`` whenever no sequence is empty."""
    lens = prepare_lens(cu_seqlens)
    rows = [(n, c) for n, L in enumerate(lens)
            for c in range((int(L) + chunk_size - 1) // chunk_size)]
    return np.asarray(rows, dtype=np.int64).reshape(-1, 2)
