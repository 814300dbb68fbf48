"""Stage 1: per-group causal block-max index scores (drop-in for
``msa_triton.triton.index_score``).

``m3_index_score`` validates exactly as triton/index_score.py:325-355 and
returns FP32 ``[T, G, ceil(max_seqlen / block_size)]``. Future and
out-of-sequence blocks are ``-inf`` with zero derivative; ties of the block
maximum share the gradient equally (torch.amax). Winners and ties are decided
on float64 dot products of the exact inputs.

Kernel families (no user switch): bf16/f16 inputs with ``Di`` in {64, 128},
``block_size == 128`` and a power-of-two ``G`` compute the public scores with
the tcgen05 GEMM kernel (float32 accumulation of the exact products);
other shapes use the float64 kernel. When a backward is needed the tensor-core
forward also records the winner state (float32 winners where they are clear
of every other key by an error margin, float64 recomputation elsewhere), so
the public scores are the same bits with and without autograd and the
gradients follow the float64 winners; its backward transposes the winner
table without atomics (float64 sums).
"""

from __future__ import annotations

import math

import torch

from . import _dispatch
from . import _lib
from ._lib import DTYPE_CODE, call, ptr, stream_of
from .prepared import host_bounds


def score_forward(index_q, index_k, cu_seqlens, max_seqlen, block_size, scale, save_state):
    """Scores (and, with ``save_state``, the winner state the backward needs) of one call.
    Returns ``(scores, max_val, tie_info, tc)``; the state tensors are None without
    ``save_state``. Shared by the autograd Function and the torch.library operator."""
    q = index_q.contiguous()
    k = index_k.contiguous()
    cu = cu_seqlens.contiguous()
    total, groups, dim = q.shape
    nseq = cu.numel() - 1
    blocks = (max_seqlen + block_size - 1) // block_size
    scores = torch.empty((total, groups, blocks), dtype=torch.float32, device=q.device)
    max_val = tie_info = None
    if save_state:
        max_val = torch.empty((total, groups, blocks), dtype=torch.float64, device=q.device)
        tie_info = torch.empty((total, groups, blocks), dtype=torch.int32, device=q.device)
    tc = _dispatch.score_uses_tc(q, block_size)
    if total:
        with torch.cuda.device(q.device):
            args = (ptr(q), ptr(k), DTYPE_CODE[q.dtype], ptr(cu), nseq, total, groups, dim, blocks, block_size)
            if tc and save_state:  # the tensor-core scores plus the float64-exact winner state
                lib = _lib.load()
                ws_bytes = lib.msa_index_score_state_workspace_size(total, groups)
                ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
                call("msa_index_score_fwd_tc_state", *args, float(scale), ptr(scores), ptr(tie_info),
                     ptr(max_val), ptr(ws), ws_bytes, stream_of(q))
            elif tc:
                call("msa_index_score_fwd_tc", *args, float(scale), 0, total, ptr(scores), stream_of(q))
            else:
                call("msa_index_score_fwd", *args, float(scale), ptr(scores), ptr(max_val), ptr(tie_info),
                     stream_of(q))
    return scores, max_val, tie_info, tc


def score_backward(index_q, index_k, cu_seqlens, max_val, tie_info, grad_scores, block_size, scale, tc, need_q,
                   need_k):
    """(dIQ, dIK) in the inputs' dtypes (None where not requested) through the saved winner state."""
    q = index_q.contiguous()
    k = index_k.contiguous()
    cu = cu_seqlens.contiguous()
    total, groups, dim = q.shape
    nseq = cu.numel() - 1
    blocks = max_val.shape[2]
    ds = grad_scores.to(torch.float32).contiguous()
    dq = torch.empty_like(q) if need_q else None
    dk = torch.empty_like(k) if need_k else None
    if total and (dq is not None or dk is not None):
        with torch.cuda.device(q.device):
            if tc:
                lib = _lib.load()
                ws_bytes = lib.msa_index_score_bwd_tc_workspace_size(total, nseq, groups, dim, blocks)
                ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
                call("msa_index_score_bwd_tc", ptr(q), ptr(k), DTYPE_CODE[q.dtype], ptr(cu), nseq, total, groups,
                     dim, blocks, block_size, scale, ptr(max_val), ptr(tie_info), ptr(ds), ptr(dq), ptr(dk),
                     ptr(ws), ws_bytes, stream_of(q))
            else:
                call("msa_index_score_bwd", ptr(q), ptr(k), DTYPE_CODE[q.dtype], ptr(cu), nseq, total, groups,
                     dim, blocks, block_size, scale, ptr(max_val), ptr(tie_info), ptr(ds), ptr(dq), ptr(dk),
                     stream_of(q))
    return (None if dq is None else dq.to(index_q.dtype), None if dk is None else dk.to(index_k.dtype))


class _IndexScore(torch.autograd.Function):
    @staticmethod
    def forward(ctx, index_q, index_k, cu_seqlens, max_seqlen, block_size, scale, save_state):
        scores, max_val, tie_info, tc = score_forward(index_q, index_k, cu_seqlens, max_seqlen, block_size, scale,
                                                      save_state)
        if save_state:
            ctx.save_for_backward(index_q.contiguous(), index_k.contiguous(), cu_seqlens.contiguous(), max_val,
                                  tie_info)
        ctx.tc = tc
        ctx.meta = (block_size, float(scale))
        return scores

    @staticmethod
    def backward(ctx, grad_scores):
        q, k, cu, max_val, tie_info = ctx.saved_tensors
        block_size, scale = ctx.meta
        dq, dk = score_backward(q, k, cu, max_val, tie_info, grad_scores, block_size, scale, ctx.tc,
                                ctx.needs_input_grad[0], ctx.needs_input_grad[1])
        return dq, dk, None, None, None, None, None


def m3_index_score(
    index_q: torch.Tensor,
    index_k: torch.Tensor,
    cu_seqlens: torch.Tensor,
    max_seqlen: int,
    *,
    block_size: int = 128,
    scale: float = 1.0,
    prepared=None,
) -> torch.Tensor:
    """Return per-group causal block maxima as FP32 ``[T, G, Bmax]``.

    ``index_q`` is ``[T,G,Di]`` and ``index_k`` is ``[T,1,Di]``; blocks are
    relative to the start of each packed sequence. Validation and messages
    follow triton/index_score.py:325-355; CUDA tensors only. ``prepared``
    (from ``prepare_batch``) supplies the boundaries without a device read.
    """
    if index_q.ndim != 3 or index_k.ndim != 3:
        raise ValueError("index_q and index_k must be rank-3 TND tensors")
    total, groups, dim = index_q.shape
    if groups < 1 or dim < 1 or index_k.shape != (total, 1, dim):
        raise ValueError("expected index_q[T,G,Di] and index_k[T,1,Di] with G, Di > 0")
    if index_q.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise TypeError("index_q must have BF16, FP16, or FP32 dtype")
    if index_k.dtype != index_q.dtype or index_k.device != index_q.device:
        raise ValueError("index_q and index_k must share dtype and device")
    if cu_seqlens.ndim != 1 or cu_seqlens.numel() < 2 or cu_seqlens.dtype != torch.int32:
        raise ValueError("cu_seqlens must be a rank-1 int32 tensor with at least two entries")
    if cu_seqlens.device != index_q.device:
        raise ValueError("cu_seqlens must be on the input device")
    if not isinstance(block_size, int) or block_size <= 0:
        raise ValueError("block_size must be a positive integer")
    if not isinstance(max_seqlen, int) or max_seqlen <= 0:
        raise ValueError("max_seqlen must be a positive integer")
    if total > 2147483647 or cu_seqlens.numel() - 1 > 2147483647:
        raise ValueError("packed token and sequence counts must fit int32 metadata")
    if block_size > 2147483647 or max_seqlen > 2147483647:
        raise ValueError("block_size and max_seqlen must fit int32 metadata")
    if not math.isfinite(scale):
        raise ValueError("scale must be finite")
    boundaries = host_bounds(cu_seqlens, prepared)
    lengths = [end - start for start, end in zip(boundaries, boundaries[1:])]
    if boundaries[0] != 0 or boundaries[-1] != total or any(n < 0 for n in lengths):
        raise ValueError("cu_seqlens must span T with nondecreasing boundaries starting at zero")
    if max(lengths) > max_seqlen:
        raise ValueError("max_seqlen is smaller than a packed sequence")
    _lib.require_cuda(index_q)
    save_state = torch.is_grad_enabled() and (index_q.requires_grad or index_k.requires_grad)
    if torch.compiler.is_compiling():  # traced by torch.compile: the registered operator
        from . import library

        return library.index_score(index_q, index_k, cu_seqlens, max_seqlen, block_size, float(scale), save_state)
    return _IndexScore.apply(index_q, index_k, cu_seqlens, max_seqlen, block_size, float(scale), save_state)
