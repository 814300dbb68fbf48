"""Multi-GPU sharding of the three-stage sparse attention (one process per GPU,
``torch.distributed`` for the plumbing: NCCL over NVLink on B200s, gloo in the
CPU tests).

Two layouts, chosen by the caller:

* **Packed batch of many sequences** (``shard_packed_batch``): whole sequences
  go to ranks by longest-processing-time bin packing on their cost (selected
  attention FLOPs forward + backward plus the causal index score). Each rank
  runs the unchanged ``m3_index_score -> m3_topk -> m3_sparse_attention`` on its
  sub-batch with re-based ``cu_seqlens``; no collective touches the data path
  (a sequence's gradients stay on its rank).
* **One long sequence** (``cp_select_blocks``, ``cp_sparse_attention``): query
  tokens split into equal ranges, one per rank. A rank all-gathers ``index_k``,
  K and V, scores and selects blocks for its own queries against every key,
  attends them, and in the backward reduce-scatters its float32 dK/dV partial
  sums back to the ranks owning those keys; dQ stays local. The local kernels
  run on full-length buffers in which only the rank's query rows are real:
  rows of other ranks select no block, so the attention kernels, which walk
  the key-to-query CSR, do no work for them, and the per-row passes (query-
  range entry points) cover only the rank's rows. The K/V all-gathers run
  while the rank's k2q CSR is built.

Collectives are issued in the same order on every rank (forward: K then V;
backward: dK then dV).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _dispatch, _lib
from . import k2q as _k2q_module
from ._lib import DTYPE_CODE, call, ptr, stream_of
from .index_score import m3_index_score
from .prepared import PreparedBatch
from .sparse_attention import tc_backward, tc_forward
from .topk import m3_topk


# --------------------------------------------------------------------------- packed batches
def selected_keys(length: int, block_size: int, topk_blocks: int) -> int:
    """Keys attended by a sequence's tokens summed over its tokens, for distinct
    valid selections: a token at position p sees (p mod B) + 1 keys of its own
    block and B keys of each of min(K, p // B + 1) - 1 earlier blocks."""
    total = 0
    for b in range((length + block_size - 1) // block_size):
        n = min(block_size, length - b * block_size)
        total += n * (n + 1) // 2 + n * block_size * (min(topk_blocks, b + 1) - 1)
    return total


def sequence_cost(length: int, *, q_heads: int, groups: int, dim: int, index_dim: int, block_size: int,
                  topk_blocks: int) -> float:
    """FLOPs of one sequence: attention forward + backward (12 * D per selected
    (query head, key) pair) plus the causal index score (2 * Di * G per pair)."""
    attention = 12 * dim * q_heads * selected_keys(length, block_size, topk_blocks)
    score = 2 * index_dim * groups * length * (length + 1) / 2
    return float(attention + score)


def plan_sequence_shards(costs: list[float], world: int) -> list[list[int]]:
    """Longest-processing-time bin packing: sequences by decreasing cost, each to
    the least-loaded rank (lowest rank on ties). Returns each rank's sequence ids
    in increasing order."""
    if world < 1:
        raise ValueError("world must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    loads = [0.0] * world
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (loads[j], j))
        shards[r].append(i)
        loads[r] += costs[i]
    return [sorted(s) for s in shards]


@dataclass(frozen=True)
class SequenceShard:
    """One rank's part of a packed batch."""

    sequences: tuple[int, ...]  # global sequence ids, in packed order
    token_index: torch.Tensor   # int64 [T_local]: the global token of each local token
    cu_seqlens: torch.Tensor    # int32 [len(sequences) + 1]: local boundaries
    max_seqlen: int


def shard_packed_batch(cu_seqlens: torch.Tensor, world: int, rank: int, *, q_heads: int, groups: int, dim: int,
                       index_dim: int, block_size: int = 128, topk_blocks: int = 16) -> SequenceShard:
    """Whole-sequence shard of a packed batch for `rank` (LPT on `sequence_cost`)."""
    bounds = _lib.host_ints(cu_seqlens)
    lengths = [b - a for a, b in zip(bounds[:-1], bounds[1:])]
    if bounds[0] != 0 or any(n < 0 for n in lengths):
        raise ValueError("cu_seqlens must start at zero and be nondecreasing")
    if not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    costs = [sequence_cost(n, q_heads=q_heads, groups=groups, dim=dim, index_dim=index_dim, block_size=block_size,
                           topk_blocks=topk_blocks) for n in lengths]
    mine = plan_sequence_shards(costs, world)[rank]
    parts = [torch.arange(bounds[s], bounds[s + 1], dtype=torch.int64) for s in mine]
    token_index = torch.cat(parts) if parts else torch.zeros(0, dtype=torch.int64)
    local = [0]
    for s in mine:
        local.append(local[-1] + lengths[s])
    return SequenceShard(tuple(mine), token_index, torch.tensor(local, dtype=torch.int32),
                         max([lengths[s] for s in mine], default=0))


def take_tokens(x: torch.Tensor, shard: SequenceShard) -> torch.Tensor:
    """Rows of a packed TND tensor that belong to `shard`, in local order."""
    return x.index_select(0, shard.token_index.to(x.device))


# --------------------------------------------------------------------------- one long sequence
def context_parallel_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Query tokens [lo, hi) of `rank` when `total` tokens split evenly over `world` ranks."""
    if total % world:
        raise ValueError(f"context parallelism needs T divisible by the world size ({total} % {world} != 0)")
    n = total // world
    return rank * n, (rank + 1) * n


def all_gather_tokens(x: torch.Tensor, group=None) -> torch.Tensor:
    """Concatenation over ranks (in rank order) of equally sized token slices."""
    world = dist.get_world_size(group)
    out = x.new_empty((world * x.shape[0],) + tuple(x.shape[1:]))
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def reduce_scatter_tokens(x: torch.Tensor, group=None) -> torch.Tensor:
    """Sum over ranks of a full-length tensor; each rank keeps its token slice."""
    world = dist.get_world_size(group)
    out = x.new_empty((x.shape[0] // world,) + tuple(x.shape[1:]))
    dist.reduce_scatter_tensor(out, x.contiguous(), op=dist.ReduceOp.SUM, group=group)
    return out


def _cp_scores(iq_full, ik_full, total, lo, hi, block_size, scale):
    """Index scores of query rows [lo, hi) of one sequence of `total` tokens against
    all its keys; rows outside the range are not computed (their content is undefined)."""
    cu = torch.tensor([0, total], dtype=torch.int32, device=iq_full.device)
    if not _dispatch.score_uses_tc(iq_full, block_size):
        return m3_index_score(iq_full, ik_full, cu, total, block_size=block_size, scale=scale)
    groups, dim = iq_full.shape[1], iq_full.shape[2]
    blocks = (total + block_size - 1) // block_size
    scores = torch.empty((total, groups, blocks), dtype=torch.float32, device=iq_full.device)
    with torch.cuda.device(iq_full.device):
        call("msa_index_score_fwd_tc", ptr(iq_full), ptr(ik_full), DTYPE_CODE[iq_full.dtype], ptr(cu), 1, total,
             groups, dim, blocks, block_size, float(scale), lo, hi, ptr(scores), stream_of(iq_full))
    return scores


def _cp_topk(scores_local, lo, total, block_size, topk_blocks, local_blocks):
    """Top-k of the rows of query tokens lo, lo + 1, ... of one sequence: the kernel takes
    positions from cu_seqlens, so a one-sequence cu of [-lo, n] places local row t at
    position lo + t (the selection rule of m3_topk, run on this rank's rows only)."""
    n, groups, blocks = scores_local.shape
    out = torch.empty((n, groups, topk_blocks), dtype=torch.int32, device=scores_local.device)
    if n == 0 or topk_blocks == 0:
        return out.fill_(-1)
    _lib.require_cuda(scores_local)
    cu = torch.tensor([-lo, n], dtype=torch.int32, device=scores_local.device)
    with torch.cuda.device(scores_local.device):
        call("msa_topk", ptr(scores_local.contiguous()), ptr(cu), 1, n, groups, blocks, block_size, topk_blocks,
             local_blocks, ptr(out), stream_of(scores_local))
    return out


@torch.no_grad()
def cp_select_blocks(index_q: torch.Tensor, index_k: torch.Tensor, total: int, *, group=None, block_size: int = 128,
                     topk_blocks: int = 16, local_blocks: int = 1, scale: float = 1.0) -> torch.Tensor:
    """Context-parallel index score + top-k: this rank's query slice
    ``index_q[T/N, G, Di]`` against the all-gathered ``index_k``; returns the rank's
    block ids ``[T/N, G, K]`` (no gradient: the selection is not differentiable).
    Only the rank's rows are scored and ranked."""
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    lo, hi = context_parallel_range(total, world, rank)
    if index_q.shape[0] != hi - lo or index_k.shape[0] != hi - lo:
        raise ValueError("index_q / index_k must hold this rank's T / world tokens")
    ik_full = all_gather_tokens(index_k, group)
    iq_full = index_q.new_empty((total,) + tuple(index_q.shape[1:]))  # rows outside [lo, hi) are never read
    iq_full[lo:hi] = index_q
    scores = _cp_scores(iq_full, ik_full, total, lo, hi, block_size, scale)
    return _cp_topk(scores[lo:hi], lo, total, block_size, topk_blocks, local_blocks)


def _cp_prepare(ids_full, cu, block_size):
    """The k2q CSR of the rank's selection (full-length ids, -1 outside its rows)."""
    return _k2q_module.build_k2q_csr(ids_full, cu, block_size=block_size,
                                     prepared=PreparedBatch(cu, (0, ids_full.shape[0])))


def _cp_forward_local(q_full, k_full, v_full, ids_full, cu, block_size, scale, lo, hi, csr):
    """Tensor-core forward of query rows [lo, hi) on full-length buffers; returns
    (out_full, state for the backward). Rows outside the range are not written."""
    if not _dispatch.attention_uses_tc(q_full, k_full, block_size):
        raise ValueError("context-parallel attention runs the tensor-core kernels: bf16/f16, head_dim 128, "
                         "block_size 128, 4, 8 or 16 query heads per group, at least 8 query heads")
    out_full = torch.empty_like(q_full)
    lse = torch.empty(q_full.shape[:2], dtype=torch.float32, device=q_full.device)
    tc_forward(q_full, k_full, v_full, ids_full, cu, block_size, scale, out_full, lse, [0, q_full.shape[0]],
               query_range=(lo, hi), csr=csr)
    return out_full, (q_full, k_full, v_full, ids_full, cu, lse, out_full, csr, block_size, scale)


def _cp_backward_local(state, grad_full, lo, hi):
    """dQ rows [lo, hi) (input dtype) and float32 dK/dV partial sums over those queries."""
    q, k, v, ids, cu, lse, out, csr, block_size, scale = state
    dq = torch.empty_like(q)
    dk = torch.empty(k.shape, dtype=torch.float32, device=k.device)
    dv = torch.empty(v.shape, dtype=torch.float32, device=v.device)
    tc_backward(q, k, v, ids, cu, lse, out, csr, block_size, scale, grad_full, dq, dk, dv, query_range=(lo, hi))
    return dq, dk, dv


class _ContextParallelAttention(torch.autograd.Function):
    """Rank-local context parallelism. K and V are all-gathered (asynchronously, while the
    k2q CSR of the rank's selection is built); the tensor-core kernels run on full-length
    buffers of which only the rank's query slice is filled, written or passed over
    (query-range entry points: bounds, accumulator zeroing, finalize, delta and dQ
    finalize cover [lo, hi) alone); dK/dV are float32 partial sums over the rank's queries,
    reduce-scattered back to the key owners."""

    @staticmethod
    def forward(ctx, q, k, v, indices, total, block_size, scale, group):
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        lo, hi = context_parallel_range(total, world, rank)
        k_full = k.new_empty((total,) + tuple(k.shape[1:]))
        v_full = v.new_empty((total,) + tuple(v.shape[1:]))
        work = [dist.all_gather_into_tensor(k_full, k.contiguous(), group=group, async_op=True),
                dist.all_gather_into_tensor(v_full, v.contiguous(), group=group, async_op=True)]
        q_full = q.new_empty((total,) + tuple(q.shape[1:]))  # rows outside [lo, hi) are never read
        q_full[lo:hi] = q
        ids_full = indices.new_full((total,) + tuple(indices.shape[1:]), -1)
        ids_full[lo:hi] = indices
        cu = torch.tensor([0, total], dtype=torch.int32, device=q.device)
        csr = _cp_prepare(ids_full, cu, block_size)
        for w_ in work:
            w_.wait()
        out_full, ctx.state = _cp_forward_local(q_full, k_full, v_full, ids_full, cu, block_size, scale, lo, hi, csr)
        ctx.meta = (lo, hi, group, total, k.dtype)
        return out_full[lo:hi].clone()

    @staticmethod
    def backward(ctx, grad_out):
        lo, hi, group, total, kv_dtype = ctx.meta
        grad_full = grad_out.new_empty((total,) + tuple(grad_out.shape[1:]))  # rows outside [lo, hi) unread
        grad_full[lo:hi] = grad_out
        dq_full, dk, dv = _cp_backward_local(ctx.state, grad_full, lo, hi)
        ctx.state = None
        dk = reduce_scatter_tokens(dk, group).to(kv_dtype)
        dv = reduce_scatter_tokens(dv, group).to(kv_dtype)
        return dq_full[lo:hi].clone(), dk, dv, None, None, None, None, None


def cp_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, indices: torch.Tensor, total: int, *,
                        group=None, block_size: int = 128, scale: float | None = None) -> torch.Tensor:
    """Context-parallel ``m3_sparse_attention`` of one causal sequence of `total`
    tokens: this rank holds query/key/value tokens ``[lo, hi)`` (equal slices in
    rank order) and its queries' block ids (sequence-local). Returns the rank's
    output rows; gradients flow to its q, k, v slices."""
    world = dist.get_world_size(group)
    n = total // world
    if q.ndim != 3 or k.ndim != 3 or v.shape != k.shape or q.shape[0] != n or k.shape[0] != n:
        raise ValueError("q/k/v must be this rank's [T / world, H, D] slices")
    if indices.shape[:2] != (n, k.shape[1]) or indices.dtype != torch.int32:
        raise ValueError("indices must be int32 [T / world, G, K]")
    effective = q.shape[-1] ** -0.5 if scale is None else float(scale)
    return _ContextParallelAttention.apply(q, k, v, indices, total, block_size, effective, group)
