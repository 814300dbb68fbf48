"""Stage 2: top-k block selection (drop-in for ``msa_triton.triton.topk``).

Validation and output contract follow triton/topk.py:11-47: future blocks are
excluded, the ``local_blocks`` most recent causal blocks are always kept, the
remaining slots go to the highest scores, ids are written in descending rank
with ``-1`` padding. Equal ranks are ordered by ascending block id. The whole
selection (masking, local forcing, ranking) is one warp-per-row CUDA kernel;
no masked copies of the scores are made.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import call, ptr, stream_of
from .prepared import host_bounds


@torch.no_grad()
def m3_topk(scores, cu_seqlens, *, block_size=128, topk_blocks=16, local_blocks=1, prepared=None):
    if scores.ndim != 3 or scores.dtype != torch.float32:
        raise ValueError("scores must be FP32 [T,G,Bmax]")
    if cu_seqlens.ndim != 1 or cu_seqlens.numel() < 2 or cu_seqlens.dtype != torch.int32:
        raise ValueError("cu_seqlens must be an int32 vector with at least two entries")
    if cu_seqlens.device != scores.device:
        raise ValueError("scores and cu_seqlens must share a device")
    if not isinstance(block_size, int) or block_size <= 0:
        raise ValueError("block_size must be a positive integer")
    if not isinstance(topk_blocks, int) or topk_blocks < 0:
        raise ValueError("topk_blocks must be a nonnegative integer")
    if not isinstance(local_blocks, int) or not 0 <= local_blocks <= topk_blocks:
        raise ValueError("local_blocks must satisfy 0 <= local_blocks <= topk_blocks")
    total, groups, blocks = scores.shape
    boundaries = host_bounds(cu_seqlens, prepared)
    if boundaries[0] != 0 or boundaries[-1] != total or any(b < a for a, b in zip(boundaries, boundaries[1:])):
        raise ValueError("cu_seqlens must start at 0, be nondecreasing, and end at T")
    if groups <= 0 or blocks <= 0 or any(b - a > blocks * block_size for a, b in zip(boundaries, boundaries[1:])):
        raise ValueError("scores need positive G and enough block slots for every sequence")
    _lib.require_cuda(scores)
    if torch.compiler.is_compiling():  # traced by torch.compile: the registered operator
        from . import library

        return library.topk(scores, cu_seqlens, boundaries, block_size, topk_blocks, local_blocks)
    return topk_into(scores, cu_seqlens, block_size, topk_blocks, local_blocks)


def topk_into(scores, cu_seqlens, block_size, topk_blocks, local_blocks):
    """Launch the selection kernel on validated arguments; returns int32 ``[T, G, K]``."""
    total, groups, blocks = scores.shape
    result = torch.empty((total, groups, topk_blocks), dtype=torch.int32, device=scores.device)
    if total == 0 or topk_blocks == 0:
        return result.fill_(-1)
    s = scores.contiguous()
    cu = cu_seqlens.contiguous()
    with torch.cuda.device(s.device):
        call("msa_topk", ptr(s), ptr(cu), cu.numel() - 1, total, groups, blocks, block_size, topk_blocks,
             local_blocks, ptr(result), stream_of(s))
    return result
