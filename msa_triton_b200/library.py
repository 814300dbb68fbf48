"""The three operators registered with ``torch.library`` (namespace ``msa_b200``).

The reference's review asks for operators that ``torch.compile`` and CUDA-graph
capture can take whole (docs/code_review.md:90-105, A4): each op is a
``torch.library.custom_op`` with a fake (meta) kernel that gives the output
shapes from the arguments alone, and ``register_autograd`` wiring the backward
to a second registered op. The packed boundaries come in as a host list
(``bounds``, from ``prepare_batch``), so nothing inside reads the device.

``m3_index_score``, ``m3_topk`` and ``m3_sparse_attention`` route here by
themselves while ``torch.compile`` traces them (they need ``prepared=`` then);
eager calls keep their ``torch.autograd.Function`` path. Both run the same
launchers (``index_score.score_forward`` / ``score_backward``,
``sparse_attention.attention_forward`` / ``attention_backward``,
``topk.topk_into``) on the same CUDA kernels.

Registered ops (extra outputs carry the state a backward needs and are not
differentiable):

* ``msa_b200::index_score(iq, ik, cu, max_seqlen, block_size, scale, save_state)
  -> (scores, max_val, tie_info)``; ``msa_b200::index_score_backward``.
* ``msa_b200::topk(scores, cu, bounds, block_size, topk_blocks, local_blocks) -> ids``.
* ``msa_b200::sparse_attention(q, k, v, indices, cu, bounds, block_size, scale)
  -> (out, lse, lse64, row_ptr, query_indices, slot_indices, cu_block_lens)``;
  ``msa_b200::sparse_attention_backward``.
"""

from __future__ import annotations

import torch
from torch import Tensor

from . import _dispatch
from . import index_score as _score
from . import sparse_attention as _attn
from . import topk as _topk
from .k2q import K2QCSR
from .layout import block_prefix


def _none_if_empty(t: Tensor, wanted: bool):
    return t if wanted else None


def _empty_like_or(t: Tensor | None, ref: Tensor, dtype=None) -> Tensor:
    return t if t is not None else ref.new_empty((0,), dtype=dtype or ref.dtype)


# ----------------------------------------------------------------------------- index score
@torch.library.custom_op("msa_b200::index_score", mutates_args=(), device_types="cuda")
def _index_score_op(index_q: Tensor, index_k: Tensor, cu_seqlens: Tensor, max_seqlen: int, block_size: int,
                    scale: float, save_state: bool) -> tuple[Tensor, Tensor, Tensor]:
    scores, max_val, tie_info, _ = _score.score_forward(index_q, index_k, cu_seqlens, max_seqlen, block_size, scale,
                                                        save_state)
    return (scores, _empty_like_or(max_val, scores, torch.float64),
            _empty_like_or(tie_info, scores, torch.int32))


@_index_score_op.register_fake
def _(index_q, index_k, cu_seqlens, max_seqlen, block_size, scale, save_state):
    total, groups, _ = index_q.shape
    shape = (total, groups, (max_seqlen + block_size - 1) // block_size)
    state = shape if save_state else (0,)
    return (index_q.new_empty(shape, dtype=torch.float32), index_q.new_empty(state, dtype=torch.float64),
            index_q.new_empty(state, dtype=torch.int32))


@torch.library.custom_op("msa_b200::index_score_backward", mutates_args=(), device_types="cuda")
def _index_score_backward_op(index_q: Tensor, index_k: Tensor, cu_seqlens: Tensor, max_val: Tensor,
                             tie_info: Tensor, grad_scores: Tensor, block_size: int, scale: float, tc: bool,
                             need_q: bool, need_k: bool) -> tuple[Tensor, Tensor]:
    dq, dk = _score.score_backward(index_q, index_k, cu_seqlens, max_val, tie_info, grad_scores, block_size, scale,
                                   tc, need_q, need_k)
    return _empty_like_or(dq, index_q), _empty_like_or(dk, index_k)


@_index_score_backward_op.register_fake
def _(index_q, index_k, cu_seqlens, max_val, tie_info, grad_scores, block_size, scale, tc, need_q, need_k):
    return (torch.empty_like(index_q) if need_q else index_q.new_empty((0,)),
            torch.empty_like(index_k) if need_k else index_k.new_empty((0,)))


def _index_score_setup(ctx, inputs, output):
    index_q, index_k, cu_seqlens, max_seqlen, block_size, scale, save_state = inputs
    _, max_val, tie_info = output
    ctx.save_for_backward(index_q, index_k, cu_seqlens, max_val, tie_info)
    ctx.meta = (block_size, scale, _dispatch.score_uses_tc(index_q, block_size), save_state)


def _index_score_bwd(ctx, grad_scores, _grad_max, _grad_tie):
    index_q, index_k, cu_seqlens, max_val, tie_info = ctx.saved_tensors
    block_size, scale, tc, save_state = ctx.meta
    if not save_state:
        raise RuntimeError("msa_b200::index_score was called with save_state=False; it has no backward state")
    need_q, need_k = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
    dq, dk = torch.ops.msa_b200.index_score_backward(index_q, index_k, cu_seqlens, max_val, tie_info, grad_scores,
                                                     block_size, scale, tc, need_q, need_k)
    return _none_if_empty(dq, need_q), _none_if_empty(dk, need_k), None, None, None, None, None


_index_score_op.register_autograd(_index_score_bwd, setup_context=_index_score_setup)


def index_score(index_q, index_k, cu_seqlens, max_seqlen, block_size, scale, save_state) -> Tensor:
    """The scores of ``msa_b200::index_score`` (arguments already validated)."""
    return torch.ops.msa_b200.index_score(index_q, index_k, cu_seqlens, max_seqlen, block_size, scale, save_state)[0]


# ----------------------------------------------------------------------------- top-k
@torch.library.custom_op("msa_b200::topk", mutates_args=(), device_types="cuda")
def _topk_op(scores: Tensor, cu_seqlens: Tensor, bounds: list[int], block_size: int, topk_blocks: int,
             local_blocks: int) -> Tensor:
    return _topk.topk_into(scores, cu_seqlens, block_size, topk_blocks, local_blocks)


@_topk_op.register_fake
def _(scores, cu_seqlens, bounds, block_size, topk_blocks, local_blocks):
    return scores.new_empty((scores.shape[0], scores.shape[1], topk_blocks), dtype=torch.int32)


def topk(scores, cu_seqlens, bounds, block_size, topk_blocks, local_blocks) -> Tensor:
    return torch.ops.msa_b200.topk(scores, cu_seqlens, list(bounds), block_size, topk_blocks, local_blocks)


# ----------------------------------------------------------------------------- sparse attention
def _csr_sizes(bounds, groups, total, topk_blocks, block_size):
    lengths = [b - a for a, b in zip(bounds[:-1], bounds[1:])]
    blocks = block_prefix(lengths, block_size)
    return blocks[-1] * groups + 1, total * groups * topk_blocks, len(blocks)


@torch.library.custom_op("msa_b200::sparse_attention", mutates_args=(), device_types="cuda")
def _sparse_attention_op(q: Tensor, k: Tensor, v: Tensor, indices: Tensor, cu_seqlens: Tensor, bounds: list[int],
                         block_size: int, scale: float) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor,
                                                                 Tensor]:
    out, lse, lse_saved, _, csr, _ = _attn.attention_forward(q, k, v, indices, cu_seqlens, block_size, scale,
                                                             list(bounds))
    i32 = torch.int32
    if csr is None:  # precise family: float64 LSE saved, CSR built by the backward if K or V needs it
        return out, lse, lse_saved, *(q.new_empty((0,), dtype=i32) for _ in range(4))
    return (out, lse, q.new_empty((0,), dtype=torch.float64), csr.row_ptr, csr.query_indices, csr.slot_indices,
            csr.cu_block_lens)


@_sparse_attention_op.register_fake
def _(q, k, v, indices, cu_seqlens, bounds, block_size, scale):
    total, hq, _ = q.shape
    i32 = torch.int32
    out = torch.empty_like(q)
    lse = q.new_empty((total, hq), dtype=torch.float32)
    if total and _dispatch.attention_uses_tc(q, k, block_size):
        rows, edges, nbl = _csr_sizes(bounds, k.shape[1], total, indices.shape[2], block_size)
        return (out, lse, q.new_empty((0,), dtype=torch.float64), q.new_empty((rows,), dtype=i32),
                q.new_empty((edges,), dtype=i32), q.new_empty((edges,), dtype=i32), q.new_empty((nbl,), dtype=i32))
    return out, lse, q.new_empty((total, hq), dtype=torch.float64), *(q.new_empty((0,), dtype=i32)
                                                                      for _ in range(4))


@torch.library.custom_op("msa_b200::sparse_attention_backward", mutates_args=(), device_types="cuda")
def _sparse_attention_backward_op(q: Tensor, k: Tensor, v: Tensor, indices: Tensor, cu_seqlens: Tensor,
                                  bounds: list[int], block_size: int, scale: float, out: Tensor, lse: Tensor,
                                  lse64: Tensor, row_ptr: Tensor, query_indices: Tensor, slot_indices: Tensor,
                                  cu_block_lens: Tensor, grad_out: Tensor, tc: bool, need_q: bool, need_k: bool,
                                  need_v: bool) -> tuple[Tensor, Tensor, Tensor]:
    csr = K2QCSR(row_ptr, query_indices, slot_indices, cu_block_lens) if tc else None
    dq, dk, dv, _ = _attn.attention_backward(q, k, v, indices, cu_seqlens, lse if tc else lse64, out if tc else None,
                                             csr, block_size, scale, grad_out, need_q, need_k, need_v, list(bounds))
    return _empty_like_or(dq, q), _empty_like_or(dk, k), _empty_like_or(dv, v)


@_sparse_attention_backward_op.register_fake
def _(q, k, v, indices, cu_seqlens, bounds, block_size, scale, out, lse, lse64, row_ptr, query_indices,
      slot_indices, cu_block_lens, grad_out, tc, need_q, need_k, need_v):
    return tuple(torch.empty_like(x) if n else x.new_empty((0,)) for x, n in ((q, need_q), (k, need_k), (v, need_v)))


def _sparse_attention_setup(ctx, inputs, output):
    q, k, v, indices, cu_seqlens, bounds, block_size, scale = inputs
    out, lse, lse64, row_ptr, query_indices, slot_indices, cu_block_lens = output
    ctx.save_for_backward(q, k, v, indices, cu_seqlens, out, lse, lse64, row_ptr, query_indices, slot_indices,
                          cu_block_lens)
    ctx.meta = (list(bounds), block_size, scale, q.shape[0] > 0 and _dispatch.attention_uses_tc(q, k, block_size))


def _sparse_attention_bwd(ctx, grad_out, *_unused):
    q, k, v, indices, cu_seqlens, out, lse, lse64, row_ptr, query_indices, slot_indices, cu_block_lens = \
        ctx.saved_tensors
    bounds, block_size, scale, tc = ctx.meta
    need_q, need_k, need_v = ctx.needs_input_grad[:3]
    dq, dk, dv = torch.ops.msa_b200.sparse_attention_backward(
        q, k, v, indices, cu_seqlens, bounds, block_size, scale, out, lse, lse64, row_ptr, query_indices,
        slot_indices, cu_block_lens, grad_out, tc, need_q, need_k, need_v)
    return (_none_if_empty(dq, need_q), _none_if_empty(dk, need_k), _none_if_empty(dv, need_v), None, None, None,
            None, None)


_sparse_attention_op.register_autograd(_sparse_attention_bwd, setup_context=_sparse_attention_setup)


def sparse_attention(q, k, v, indices, cu_seqlens, bounds, block_size, scale) -> tuple[Tensor, Tensor]:
    """(out, lse) of ``msa_b200::sparse_attention`` (arguments already validated)."""
    res = torch.ops.msa_b200.sparse_attention(q, k, v, indices, cu_seqlens, list(bounds), block_size, scale)
    return res[0], res[1]
