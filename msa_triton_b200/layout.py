"""Host-side validation of packed sequence boundaries.

Mirrors layout.py:18-30 of the reference (same checks, same messages). The
boundaries are read to the host once per call, as the reference does.
"""

from __future__ import annotations

import torch


def sequence_lengths(cu_seqlens: torch.Tensor, total_tokens: int, prepared=None) -> list[int]:
    """Validate packed boundaries and return sequence lengths on the host
    (from ``prepared`` when given, else read from the device)."""
    if cu_seqlens.ndim != 1 or cu_seqlens.numel() < 2:
        raise ValueError("cu_seqlens must be a vector with at least two entries")
    if cu_seqlens.dtype != torch.int32:
        raise TypeError("cu_seqlens must be int32")
    from .prepared import host_bounds

    boundaries = host_bounds(cu_seqlens, prepared)
    if boundaries[0] != 0 or boundaries[-1] != total_tokens:
        raise ValueError("cu_seqlens must start at zero and end at total_tokens")
    lengths = [end - start for start, end in zip(boundaries[:-1], boundaries[1:])]
    if min(lengths) < 0:
        raise ValueError("cu_seqlens must be nondecreasing")
    return lengths


def block_prefix(lengths: list[int], block_size: int) -> list[int]:
    """Prefix sum of per-sequence block counts (K2QCSR.cu_block_lens)."""
    out = [0]
    for n in lengths:
        out.append(out[-1] + (n + block_size - 1) // block_size)
    return out
