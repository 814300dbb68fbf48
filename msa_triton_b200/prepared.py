"""Prepared batch metadata: packed sequence boundaries read to the host once.

Every op of the reference reads ``cu_seqlens`` back to the host on each call
to validate it and to size its launches (layout.py:18-30, index_score.py:
325-355, topk.py:11-47, k2q.py:39-128), which is a device-to-host
synchronisation per op and per layer. ``prepare_batch`` does that read once;
passing the result as ``prepared=`` to ``m3_index_score``, ``m3_topk``,
``m3_sparse_attention`` or ``build_k2q_csr`` skips the per-call reads, so the
ops of every layer that shares the boundaries issue no synchronisation and
the host can run ahead of the GPU. Without ``prepared`` the ops behave as the
reference's do.

The prepared values describe the tensor at preparation time: the caller must
not change ``cu_seqlens`` in place while the prepared batch is in use.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _lib


@dataclass(frozen=True)
class PreparedBatch:
    """Host copy of a ``cu_seqlens`` tensor's boundaries."""

    cu_seqlens: torch.Tensor
    bounds: tuple[int, ...]

    @property
    def lengths(self) -> list[int]:
        return [b - a for a, b in zip(self.bounds[:-1], self.bounds[1:])]

    @property
    def total_tokens(self) -> int:
        return self.bounds[-1]

    @property
    def max_seqlen(self) -> int:
        return max(self.lengths)


def prepare_batch(cu_seqlens: torch.Tensor, bounds=None) -> PreparedBatch:
    """Read (or, with ``bounds``, take from the caller's host copy) the
    boundaries of ``cu_seqlens`` once for all the ops that use it.

    ``bounds`` lets a caller that uploaded ``cu_seqlens`` itself hand over the
    host values it uploaded, so preparing reads nothing from the device."""
    if cu_seqlens.ndim != 1 or cu_seqlens.numel() < 2 or cu_seqlens.dtype != torch.int32:
        raise ValueError("cu_seqlens must be a rank-1 int32 tensor with at least two entries")
    if bounds is None:
        values = _lib.host_ints(cu_seqlens)
    else:
        values = [int(x) for x in bounds]
        if len(values) != cu_seqlens.numel():
            raise ValueError("bounds must have one entry per cu_seqlens element")
    if values[0] != 0 or any(b < a for a, b in zip(values[:-1], values[1:])):
        raise ValueError("cu_seqlens must start at zero and be nondecreasing")
    return PreparedBatch(cu_seqlens, tuple(values))


def host_bounds(cu_seqlens: torch.Tensor, prepared: PreparedBatch | None) -> list[int]:
    """Boundaries of ``cu_seqlens`` on the host: from ``prepared`` when given
    (which must describe this very tensor), else read from the device."""
    if prepared is None:
        return _lib.host_ints(cu_seqlens)
    if not isinstance(prepared, PreparedBatch):
        raise TypeError("prepared must come from prepare_batch")
    src = prepared.cu_seqlens
    if src is not cu_seqlens and (src.device != cu_seqlens.device or src.numel() != cu_seqlens.numel()
                                  or src.data_ptr() != cu_seqlens.data_ptr()):
        raise ValueError("prepared metadata belongs to a different cu_seqlens tensor")
    return list(prepared.bounds)
