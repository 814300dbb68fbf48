"""Decode over a paged KV cache: the three stages for one new token per request.

The reference's notes describe the serving-side layouts (vLLM-Ascend: paged
K/V addressed through a block table, docs/vllm_ascend_k2q.md:22-40) but the
reference implements no decode path. These functions run the same selection
and attention semantics as the prefill operators for a batch of requests, each
contributing its newest token (position ``seq_lens[b] - 1``) as the query:

    scores  = m3_index_score_decode(index_q, index_k_cache, block_table, seq_lens, max_seqlen)
    indices = m3_topk_decode(scores, seq_lens, topk_blocks=16, local_blocks=1)
    out     = m3_sparse_decode(q, k_cache, v_cache, block_table, seq_lens, indices)

Layouts: ``index_q[B,G,Di]``, ``q[B,Hq,D]``; caches ``index_k_cache[P,S,1,Di]``,
``k_cache/v_cache[P,S,G,D]`` (P physical pages of S tokens); ``block_table[B, max_pages]``
int32 physical page of each logical page; ``seq_lens[B]`` int32 keys per request
including the new token. Inference only (no autograd). CUDA tensors only.
"""

from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import DTYPE_CODE, call, ptr, stream_of


def _check_paged(block_table, seq_lens, batch, device):
    if block_table.ndim != 2 or block_table.shape[0] != batch or block_table.dtype != torch.int32:
        raise ValueError("block_table must be int32 [B, max_pages]")
    if seq_lens.ndim != 1 or seq_lens.shape[0] != batch or seq_lens.dtype != torch.int32:
        raise ValueError("seq_lens must be int32 [B]")
    if block_table.device != device or seq_lens.device != device:
        raise ValueError("All inputs must reside on the same device.")


@torch.no_grad()
def m3_index_score_decode(index_q, index_k_cache, block_table, seq_lens, max_seqlen, *, block_size=128, scale=1.0):
    """FP32 ``[B, G, ceil(max_seqlen / block_size)]`` block maxima of the new tokens'
    index logits over their requests' cached index keys (-inf past the query)."""
    if index_q.ndim != 3 or index_k_cache.ndim != 4 or index_k_cache.shape[2] != 1:
        raise ValueError("expected index_q[B,G,Di] and index_k_cache[P,S,1,Di]")
    batch, groups, dim = index_q.shape
    if index_k_cache.shape[3] != dim or index_k_cache.dtype != index_q.dtype:
        raise ValueError("index_q and index_k_cache must share Di and dtype")
    if index_q.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise TypeError("index_q must have BF16, FP16, or FP32 dtype")
    if not isinstance(block_size, int) or block_size <= 0 or not isinstance(max_seqlen, int) or max_seqlen <= 0:
        raise ValueError("block_size and max_seqlen must be positive integers")
    if not math.isfinite(scale):
        raise ValueError("scale must be finite")
    _check_paged(block_table, seq_lens, batch, index_q.device)
    _lib.require_cuda(index_q)
    blocks = (max_seqlen + block_size - 1) // block_size
    scores = torch.empty((batch, groups, blocks), dtype=torch.float32, device=index_q.device)
    iq, ik = index_q.contiguous(), index_k_cache.contiguous()
    with torch.cuda.device(iq.device):
        call("msa_decode_index_score", ptr(iq), ptr(ik), DTYPE_CODE[iq.dtype], ptr(block_table.contiguous()),
             ptr(seq_lens), batch, groups, dim, ik.shape[1], block_table.shape[1], blocks, block_size, float(scale),
             ptr(scores), stream_of(iq))
    return scores


@torch.no_grad()
def m3_topk_decode(scores, seq_lens, *, block_size=128, topk_blocks=16, local_blocks=1):
    """int32 ``[B, G, K]``: the top-k rule of ``m3_topk`` for queries at ``seq_lens - 1``."""
    if scores.ndim != 3 or scores.dtype != torch.float32:
        raise ValueError("scores must be FP32 [B,G,Bmax]")
    if not isinstance(topk_blocks, int) or topk_blocks < 0:
        raise ValueError("topk_blocks must be a nonnegative integer")
    if not isinstance(local_blocks, int) or not 0 <= local_blocks <= topk_blocks:
        raise ValueError("local_blocks must satisfy 0 <= local_blocks <= topk_blocks")
    batch, groups, blocks = scores.shape
    if seq_lens.shape != (batch,) or seq_lens.dtype != torch.int32 or seq_lens.device != scores.device:
        raise ValueError("seq_lens must be int32 [B] on the scores' device")
    _lib.require_cuda(scores)
    out = torch.empty((batch, groups, topk_blocks), dtype=torch.int32, device=scores.device)
    if batch == 0 or topk_blocks == 0:
        return out.fill_(-1)
    positions = (seq_lens - 1).contiguous()
    s = scores.contiguous()
    with torch.cuda.device(s.device):
        call("msa_topk_positions", ptr(s), ptr(positions), batch, groups, blocks, block_size, topk_blocks,
             local_blocks, ptr(out), stream_of(s))
    return out


@torch.no_grad()
def m3_sparse_decode(q, k_cache, v_cache, block_table, seq_lens, indices, *, block_size=128, scale=None,
                     return_lse=False):
    """Sparse attention of each request's new token over its selected cached blocks."""
    if q.ndim != 3 or k_cache.ndim != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("expected q[B,Hq,D] and k_cache/v_cache[P,S,G,D]")
    batch, hq, dim = q.shape
    groups = k_cache.shape[2]
    if k_cache.shape[3] != dim or hq % groups:
        raise ValueError("Hq must be a multiple of G and D must match the cache")
    if q.dtype not in (torch.bfloat16, torch.float16, torch.float32) or k_cache.dtype != q.dtype or \
            v_cache.dtype != q.dtype:
        raise TypeError("q/k/v must share a BF16, FP16, or FP32 dtype.")
    if indices.ndim != 3 or indices.shape[:2] != (batch, groups) or indices.dtype != torch.int32:
        raise ValueError("indices must be int32 [B,G,K].")
    if not isinstance(block_size, int) or block_size <= 0:
        raise ValueError("block_size must be a positive integer.")
    effective = dim ** -0.5 if scale is None else float(scale)
    if not math.isfinite(effective):
        raise ValueError("scale must be finite.")
    _check_paged(block_table, seq_lens, batch, q.device)
    _lib.require_cuda(q)
    out = torch.empty_like(q)
    lse = torch.empty((batch, hq), dtype=torch.float32, device=q.device)
    if batch:
        lib = _lib.load()
        topk = indices.shape[2]
        ws_bytes = lib.msa_decode_attn_workspace_size(batch, hq, dim, topk)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
        qc, kc, vc = q.contiguous(), k_cache.contiguous(), v_cache.contiguous()
        with torch.cuda.device(q.device):
            call("msa_decode_attn", ptr(qc), ptr(kc), ptr(vc), DTYPE_CODE[q.dtype], ptr(block_table.contiguous()),
                 ptr(seq_lens), ptr(indices.contiguous()), batch, hq, groups, dim, kc.shape[1], block_table.shape[1],
                 topk, block_size, effective, ptr(out), ptr(lse), ptr(ws), ws_bytes, stream_of(q))
    return (out, lse) if return_lse else out
