"""Stage 3: causal block-sparse GQA attention (drop-in for
``msa_triton.triton.sparse_attention``).

``m3_sparse_attention`` validates as sparse_attention.py:452-483 and returns
``out`` (q's dtype) and optionally the FP32 natural-log LSE (non-differentiable).
Backward honours each input's ``needs_input_grad``; dK/dV are key-owned
through the k2q CSR and use no floating-point atomics.
``_SparseAttentionAtomicReference`` is the private regression path with
atomic dK/dV (sparse_attention.py:398-426).

Kernel families (no user switch): bf16/f16 with head_dim 128, block_size 128,
4, 8 or 16 query heads per group and at least 8 query heads run the tcgen05
tensor-core kernels
(forward and backward; the backward reuses the forward's k2q CSR, output and
LSE); all other shapes run the float64 precise kernels (dQ query-owned, dK/dV
through the CSR, built only when K or V needs a gradient).
"""

from __future__ import annotations

import math

import torch

from . import _dispatch
from . import _lib
from . import k2q as _k2q_module
from ._lib import DTYPE_CODE, call, ptr, stream_of
from .layout import sequence_lengths
from .prepared import PreparedBatch


def attention_forward(q, k, v, indices, cu_seqlens, block_size, scale, host_bounds=None):
    """One forward call. Returns ``(out, lse, lse_saved, out_saved, csr, workspace)``:
    the tensor-core family saves the float32 LSE and the output for its backward and
    hands over the k2q CSR it built (its work list); the precise family saves a float64
    LSE and no CSR. Shared by the autograd Function and the torch.library operator."""
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    ids = indices.contiguous()
    cu = cu_seqlens.contiguous()
    if host_bounds is None:
        host_bounds = _lib.host_ints(cu)
    total, hq, dim = q.shape
    groups = k.shape[1]
    nseq = cu.numel() - 1
    out = torch.empty_like(q)
    lse = torch.empty((total, hq), dtype=torch.float32, device=q.device)
    csr = workspace = None
    if total and _dispatch.attention_uses_tc(q, k, block_size):
        csr, workspace = tc_forward(q, k, v, ids, cu, block_size, scale, out, lse, host_bounds)
        return out, lse, lse, out, csr, workspace
    lse64 = torch.empty((total, hq), dtype=torch.float64, device=q.device)
    if total:
        with torch.cuda.device(q.device):
            call("msa_attn_fwd", ptr(q), ptr(k), ptr(v), DTYPE_CODE[q.dtype], ptr(ids), ptr(cu), nseq, total,
                 hq, groups, dim, ids.shape[2], block_size, float(scale), ptr(out), ptr(lse), ptr(lse64),
                 stream_of(q))
    return out, lse, lse64, None, None, None


def attention_backward(q, k, v, indices, cu_seqlens, lse_saved, out, csr, block_size, scale, grad_output, need_q,
                       need_k, need_v, host_bounds=None):
    """(dq, dk, dv, workspace) of one backward call; ``csr`` is the tensor-core forward's
    (None selects the precise family, which builds the CSR only when K or V needs a
    gradient, through the module attribute ``k2q.build_k2q_csr``)."""
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    ids = indices.contiguous()
    cu = cu_seqlens.contiguous()
    total, hq, dim = q.shape
    groups = k.shape[1]
    nseq = cu.numel() - 1
    dq = torch.empty_like(q) if need_q else None
    dk = torch.empty_like(k) if need_k else None
    dv = torch.empty_like(v) if need_v else None
    workspace = None
    if csr is not None:
        if need_q or need_k or need_v:
            workspace = tc_backward(q, k, v, ids, cu, lse_saved, out, csr, block_size, scale, grad_output, dq, dk,
                                    dv)
        return dq, dk, dv, workspace
    lse64 = lse_saved
    if total and (need_q or need_k or need_v):
        go = grad_output.to(q.dtype).contiguous()
        common = (DTYPE_CODE[q.dtype],)
        with torch.cuda.device(q.device):
            delta64 = torch.empty((total, hq), dtype=torch.float64, device=q.device) if need_k else None
            if need_q or need_k:
                call("msa_attn_bwd_q", ptr(q), ptr(k), ptr(v), ptr(go), *common, ptr(ids), ptr(cu), nseq, total,
                     hq, groups, dim, ids.shape[2], block_size, scale, ptr(lse64), ptr(dq), ptr(delta64),
                     stream_of(q))
            if need_k or need_v:
                # looked up on the module at call time (the reference's tests patch it)
                prepared = None if host_bounds is None else PreparedBatch(cu_seqlens, tuple(host_bounds))
                csr = _k2q_module.build_k2q_csr(ids, cu_seqlens, block_size=block_size, prepared=prepared)
                call("msa_attn_bwd_kv", ptr(q), ptr(k), ptr(v), ptr(go), *common, ptr(ids), ptr(cu),
                     ptr(csr.cu_block_lens), ptr(csr.row_ptr), ptr(csr.query_indices), ptr(csr.slot_indices),
                     nseq, total, hq, groups, dim, ids.shape[2], block_size, scale, ptr(lse64), ptr(delta64),
                     ptr(dk), ptr(dv), stream_of(q))
    return dq, dk, dv, workspace


class _SparseAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, indices, cu_seqlens, block_size, scale, host_bounds=None):
        out, lse, lse_saved, out_saved, csr, workspace = attention_forward(q, k, v, indices, cu_seqlens, block_size,
                                                                           scale, host_bounds)
        ctx.fwd_workspace = workspace if _dispatch.keep_workspace() else None
        if ctx.fwd_workspace is not None:
            _dispatch.last_fwd_workspace = (workspace, q.shape[0], q.shape[1], csr.row_ptr.numel() - 1)
        ctx.save_for_backward(q.contiguous(), k.contiguous(), v.contiguous(), indices.contiguous(),
                              cu_seqlens.contiguous(), lse_saved, out_saved)
        ctx.tc = csr is not None
        ctx.csr = csr
        ctx.keep_ws = _dispatch.keep_workspace()  # backward runs on autograd's device thread
        ctx.meta = (block_size, float(scale), host_bounds)
        ctx.mark_non_differentiable(lse)
        return out, lse

    @staticmethod
    def backward(ctx, grad_output, grad_lse):
        q, k, v, ids, cu, lse_saved, out = ctx.saved_tensors
        block_size, scale, bounds = ctx.meta
        need_q, need_k, need_v = ctx.needs_input_grad[:3]
        dq, dk, dv, workspace = attention_backward(q, k, v, ids, cu, lse_saved, out, ctx.csr, block_size, scale,
                                                   grad_output, need_q, need_k, need_v, bounds)
        if ctx.keep_ws and workspace is not None:
            _dispatch.last_bwd_workspace = workspace
        return dq, dk, dv, None, None, None, None, None


def tc_forward(q, k, v, ids, cu, block_size, scale, out, lse, bounds=None, query_range=None, csr=None):
    """Tensor-core forward into `out` / `lse`; returns the k2q CSR it built and its workspace.
    `bounds`: host copy of cu's values (saves the k2q build its own device read).
    `query_range` (lo, hi): only those query rows are computed and written (tokens outside
    it must select no block). `csr`: the k2q CSR of `ids` when the caller built it already."""
    total, hq, dim = q.shape
    groups = k.shape[1]
    if csr is None:
        prepared = None if bounds is None else PreparedBatch(cu, tuple(bounds))
        csr = _k2q_module.build_k2q_csr(ids, cu, block_size=block_size, prepared=prepared)
    num_rows = csr.row_ptr.numel() - 1
    lib = _lib.load()
    ws_bytes = lib.msa_attn_fwd_tc_workspace_size(total, hq, num_rows, groups, ids.shape[2])
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    lo, hi = (0, total) if query_range is None else query_range
    with torch.cuda.device(q.device):
        call("msa_attn_fwd_tc_range", ptr(q), ptr(k), ptr(v), DTYPE_CODE[q.dtype], ptr(ids), ptr(cu),
             ptr(csr.cu_block_lens), ptr(csr.row_ptr), ptr(csr.query_indices), cu.numel() - 1, total, hq, groups, dim,
             ids.shape[2], block_size, float(scale), num_rows, lo, hi, ptr(out), ptr(lse), ptr(workspace), ws_bytes,
             stream_of(q))
    return csr, workspace


def tc_backward(q, k, v, ids, cu, lse, out, csr, block_size, scale, grad_output, dq, dk, dv, query_range=None):
    """Tensor-core backward over the forward's k2q CSR into dq / dk / dv (any may be None;
    dk / dv may be float32 buffers: context-parallel partial sums). Returns the workspace.
    `query_range`: as for tc_forward (dq rows outside it are not written)."""
    total, hq, dim = q.shape
    groups = k.shape[1]
    num_rows = csr.row_ptr.numel() - 1
    go = grad_output.to(q.dtype).contiguous()
    kv = dk if dk is not None else dv
    kv_dtype = DTYPE_CODE[kv.dtype] if kv is not None else DTYPE_CODE[q.dtype]
    lib = _lib.load()
    ws_bytes = lib.msa_attn_bwd_tc_workspace_size(total, hq, num_rows, groups, ids.shape[2])
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    lo, hi = (0, total) if query_range is None else query_range
    with torch.cuda.device(q.device):
        call("msa_attn_bwd_tc_range", ptr(q), ptr(k), ptr(v), ptr(out), ptr(go), ptr(lse), DTYPE_CODE[q.dtype],
             ptr(cu), ptr(csr.cu_block_lens), ptr(csr.row_ptr), ptr(csr.query_indices), cu.numel() - 1, total, hq,
             groups, dim, ids.shape[2], block_size, scale, num_rows, lo, hi, ptr(dq), ptr(dk), ptr(dv), kv_dtype,
             ptr(workspace), ws_bytes, stream_of(q))
    return workspace


class _SparseAttentionAtomicReference(_SparseAttention):
    """Private regression reference: query-owned backward with atomic dK/dV."""

    @staticmethod
    def backward(ctx, grad_output, grad_lse):
        q, k, v, ids, cu, lse_saved, _ = ctx.saved_tensors
        lse64 = lse_saved.double() if ctx.tc else lse_saved
        block_size, scale, _ = ctx.meta
        need_q, need_k, need_v = ctx.needs_input_grad[:3]
        total, hq, dim = q.shape
        groups = k.shape[1]
        dq = torch.empty_like(q) if need_q else None
        dk = torch.empty_like(k) if need_k else None
        dv = torch.empty_like(v) if need_v else None
        if total and (need_q or need_k or need_v):
            go = grad_output.to(q.dtype).contiguous()
            dk_acc = torch.empty(k.shape, dtype=torch.float64, device=k.device) if need_k else None
            dv_acc = torch.empty(v.shape, dtype=torch.float64, device=v.device) if need_v else None
            with torch.cuda.device(q.device):
                call("msa_attn_bwd_atomic", ptr(q), ptr(k), ptr(v), ptr(go), DTYPE_CODE[q.dtype], ptr(ids), ptr(cu),
                     cu.numel() - 1, total, hq, groups, dim, ids.shape[2], block_size, scale, ptr(lse64), ptr(dq),
                     ptr(dk_acc), ptr(dv_acc), ptr(dk), ptr(dv), stream_of(q))
        return dq, dk, dv, None, None, None, None, None


def m3_sparse_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    indices: torch.Tensor,
    cu_seqlens: torch.Tensor,
    max_seqlen: int,
    *,
    block_size: int = 128,
    scale: float | None = None,
    return_lse: bool = False,
    prepared=None,
):
    """Apply causal block sparse attention to packed TND tensors.

    ``indices[T, G, K]`` holds distinct sequence-local block ids with ``-1``
    padding; each contiguous group of ``Hq / G`` query heads shares group
    ``g``'s selection. Empty selections produce zero output, ``-inf`` LSE and
    zero gradients. CUDA tensors only. ``prepared`` (from ``prepare_batch``)
    supplies the boundaries of ``cu_seqlens`` without a device read.
    """
    if q.ndim != 3 or k.ndim != 3 or v.shape != k.shape:
        raise ValueError("Expected q[T,Hq,D] and matching k/v[T,G,D].")
    if q.shape[0] != k.shape[0] or q.shape[2] != k.shape[2]:
        raise ValueError("q/k/v must have matching token and head dimensions.")
    if k.shape[1] <= 0 or q.shape[1] <= 0 or q.shape[1] % k.shape[1]:
        raise ValueError("Hq must be a positive multiple of G.")
    if q.shape[2] <= 0:
        raise ValueError("Head dimension must be positive.")
    if q.dtype not in (torch.bfloat16, torch.float16, torch.float32) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q/k/v must share a BF16, FP16, or FP32 dtype.")
    if indices.ndim != 3 or indices.shape[:2] != (q.shape[0], k.shape[1]) or indices.dtype != torch.int32:
        raise ValueError("indices must be int32 [T,G,K].")
    if cu_seqlens.ndim != 1 or cu_seqlens.numel() < 2 or cu_seqlens.dtype != torch.int32:
        raise ValueError("cu_seqlens must be int32 [num_sequences + 1].")
    if any(x.device != q.device for x in (k, v, indices, cu_seqlens)):
        raise ValueError("All inputs must reside on the same device.")
    if not isinstance(block_size, int) or block_size <= 0:
        raise ValueError("block_size must be a positive integer.")
    if not isinstance(max_seqlen, int) or max_seqlen <= 0:
        raise ValueError("max_seqlen must be a positive integer.")
    lengths = sequence_lengths(cu_seqlens, q.shape[0], prepared)
    if max(lengths) > max_seqlen:
        raise ValueError("max_seqlen is smaller than an actual sequence.")
    effective_scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    if not math.isfinite(effective_scale):
        raise ValueError("scale must be finite.")
    _lib.require_cuda(q)
    bounds = [0]
    for n in lengths:
        bounds.append(bounds[-1] + n)
    if torch.compiler.is_compiling():  # traced by torch.compile: the registered operator
        from . import library

        output, lse = library.sparse_attention(q, k, v, indices, cu_seqlens, bounds, block_size, effective_scale)
    else:
        output, lse = _SparseAttention.apply(q, k, v, indices, cu_seqlens, block_size, effective_scale, bounds)
    return (output, lse) if return_lse else output
