"""Index KL loss: the indexer's training objective on the selected tokens.

The reference specifies this loss for training the indexer but does not
implement it (docs/msa_training_flow.md:92-138; docs/implementation_plan.md:
66-69). On the selected causal keys J(t, g) of each (query token, group) pair
-- the same key set the sparse attention uses, without the top-k's local +inf
boost:

* student ``p_s = softmax_J(index_scale * index_q[t,g] . index_k[j])`` (token
  logits of the index projections, not the block scores);
* teacher ``p_T`` = the mean over the group's query heads of the main
  attention's probabilities ``softmax_J(scale * q[t,h] . k[j,g])``, detached;
* ``loss = sum over pairs of KL(p_T || p_s) / (T * G)``; a pair that selects no
  key contributes 0.

Gradients reach ``index_q`` and ``index_k`` only (``q`` and ``k`` are the
teacher's detached views). The main attention's LSE (``return_lse=True``) can be
passed as ``lse`` so the teacher reuses it; otherwise it is computed.

Kernels: the tensor-core family (the attention's shapes: bf16/f16, head dim and
block 128, 4/8/16 query heads per group) computes the teacher on tcgen05 by the
attention forward kernel in its teacher mode; with 16-bit index tensors of dim
64 the student logits come from a key-block-stationary walk of the same k2q CSR
on tcgen05 (128 edges x 128 keys per MMA step), a streaming pass forms the loss
and the logit gradients, and a second tensor-core CSR walk gives both index
gradients (no atomics). Other shapes use a
float64 teacher and per-pair student / key-owned dIK kernels.
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


class _IndexKL(torch.autograd.Function):
    @staticmethod
    def forward(ctx, index_q, index_k, q, k, indices, cu_seqlens, block_size, index_scale, scale, lse, bounds,
                need_grad):
        iq, ik = index_q.contiguous(), index_k.contiguous()
        qd, kd = q.detach().contiguous(), k.detach().contiguous()
        ids, cu = indices.contiguous(), cu_seqlens.contiguous()
        total, groups, index_dim = iq.shape
        hq, dim = qd.shape[1], qd.shape[2]
        topk = ids.shape[2]
        nseq = cu.numel() - 1
        dev = iq.device
        prepared = PreparedBatch(cu_seqlens, tuple(bounds))
        tc = total > 0 and _dispatch.attention_uses_tc(qd, kd, block_size)
        # 16-bit index tensors of dim 64: the student logits come from a key-block-stationary
        # walk of the same CSR, and a streaming pass forms the loss
        fused = tc and iq.dtype in (torch.bfloat16, torch.float16) and index_dim == 64
        csr = None
        lib = _lib.load()
        loss = torch.zeros((), dtype=torch.float64, device=dev)
        diq = None
        with torch.cuda.device(dev):
            if tc:
                from .sparse_attention import attention_forward

                if lse is None:  # the teacher's normaliser: the attention LSE (V does not enter it)
                    _, lse, _, _, csr, _ = attention_forward(qd, kd, kd, ids, cu, block_size, scale, list(bounds))
                else:
                    lse = lse.detach().contiguous()
                if csr is None:
                    csr = _k2q_module.build_k2q_csr(ids, cu_seqlens, block_size=block_size, prepared=prepared)
                num_rows = csr.row_ptr.numel() - 1
                pt = torch.empty(total * groups * topk * block_size, dtype=torch.float32, device=dev)
                sbuf = torch.empty_like(pt) if fused else None
                ws_bytes = lib.msa_index_kl_teacher_tc_workspace_size(total, hq, num_rows, groups, topk)
                ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
                call("msa_index_kl_teacher_tc", ptr(qd), ptr(kd), DTYPE_CODE[qd.dtype], ptr(lse), ptr(cu),
                     ptr(csr.cu_block_lens), ptr(csr.row_ptr), ptr(csr.query_indices), ptr(csr.slot_indices), nseq,
                     total, hq, groups, dim, topk, block_size, float(scale), num_rows, ptr(pt), ptr(ws), ws_bytes,
                     stream_of(qd))
                if fused:
                    call("msa_index_kl_logits_tc", ptr(iq), ptr(ik), DTYPE_CODE[iq.dtype], ptr(cu),
                         ptr(csr.cu_block_lens), ptr(csr.row_ptr), ptr(csr.query_indices), ptr(csr.slot_indices),
                         nseq, total, groups, topk, num_rows // groups, float(index_scale), ptr(sbuf), stream_of(iq))
            else:
                pt = torch.empty(max(total * groups * topk * block_size, 1), dtype=torch.float64, device=dev)
                if total:
                    call("msa_index_kl_teacher", ptr(qd), ptr(kd), DTYPE_CODE[qd.dtype], ptr(ids), ptr(cu), nseq, total,
                         hq, groups, dim, topk, block_size, float(scale), ptr(pt), stream_of(qd))
            ws_bytes = lib.msa_index_kl_student_workspace_size(total, groups)
            ws = torch.empty(max(ws_bytes, 8), dtype=torch.uint8, device=dev)
            if fused:
                call("msa_index_kl_student_tc", ptr(sbuf), ptr(pt), ptr(ids), ptr(cu), nseq, total, groups, topk,
                     float(index_scale), 1 if need_grad else 0, ptr(loss), ptr(ws), ws_bytes, stream_of(iq))
                del sbuf
            else:
                acc_dtype = torch.float32 if tc else torch.float64
                diq = torch.empty((total, groups, index_dim), dtype=acc_dtype, device=dev) if need_grad else None
                if total:
                    call("msa_index_kl_student", ptr(iq), ptr(ik), DTYPE_CODE[iq.dtype], ptr(ids), ptr(cu), nseq,
                         total, groups, index_dim, topk, block_size, float(index_scale), ptr(pt), 0 if tc else 1,
                         1 if need_grad else 0, ptr(loss), ptr(diq), ptr(ws), ws_bytes, stream_of(iq))
        ctx.need_grad = need_grad
        if need_grad:
            ctx.save_for_backward(iq, ik, cu, ids, pt, diq)
            ctx.csr = csr
            ctx.meta = (block_size, tc, fused, tuple(bounds), index_scale)
        return loss.float()

    @staticmethod
    def backward(ctx, grad_loss):
        iq, ik, cu, ids, pt, diq = ctx.saved_tensors
        block_size, tc, fused, bounds, index_scale = ctx.meta
        total, groups, index_dim = iq.shape
        need_q, need_k = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if not (need_q or need_k):
            return (None,) * 12
        lib = _lib.load()
        csr = ctx.csr
        if total and csr is None:
            csr = _k2q_module.build_k2q_csr(ids, cu, block_size=block_size, prepared=PreparedBatch(cu, tuple(bounds)))
        dik_acc = None
        with torch.cuda.device(iq.device):
            if fused:
                diq = torch.zeros((total, groups, index_dim), dtype=torch.float32, device=iq.device)
                dik_acc = torch.zeros((total, 1, index_dim), dtype=torch.float32, device=iq.device)
                if total:
                    ws_bytes = lib.msa_index_kl_grad_tc_workspace_size(total, groups, ids.shape[2])
                    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=iq.device)
                    total_blocks = (csr.row_ptr.numel() - 1) // groups
                    call("msa_index_kl_grad_tc", ptr(iq), ptr(ik), DTYPE_CODE[iq.dtype], ptr(ids), ptr(cu),
                         ptr(csr.cu_block_lens), ptr(csr.row_ptr), ptr(csr.query_indices), ptr(csr.slot_indices),
                         cu.numel() - 1, total, groups, ids.shape[2], total_blocks, float(index_scale), ptr(pt),
                         ptr(diq), ptr(dik_acc), ptr(ws), ws_bytes, stream_of(iq))
            elif need_k:
                dik_acc = torch.zeros((total, 1, index_dim), dtype=diq.dtype, device=iq.device)
                ws_bytes = lib.msa_index_kl_dik_workspace_size(total, groups, index_dim, 0 if tc else 1)
                ws = torch.empty(ws_bytes, dtype=torch.uint8, device=iq.device)
                if total:
                    total_blocks = (csr.row_ptr.numel() - 1) // groups
                    call("msa_index_kl_dik", ptr(iq), DTYPE_CODE[iq.dtype], ptr(cu), ptr(csr.cu_block_lens),
                         ptr(csr.row_ptr), ptr(csr.query_indices), ptr(csr.slot_indices), cu.numel() - 1, total,
                         groups, index_dim, ids.shape[2], block_size, total_blocks, ptr(pt), 0 if tc else 1,
                         ptr(dik_acc), ptr(ws), ws_bytes, stream_of(iq))
        g = grad_loss.to(diq.dtype)
        d_iq = (diq * g).to(iq.dtype) if need_q else None
        d_ik = (dik_acc * g).to(ik.dtype) if need_k else None
        return d_iq, d_ik, None, None, None, None, None, None, None, None, None, None


def m3_index_kl_loss(
    index_q: torch.Tensor,
    index_k: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    indices: torch.Tensor,
    cu_seqlens: torch.Tensor,
    max_seqlen: int,
    *,
    block_size: int = 128,
    index_scale: float = 1.0,
    scale: float | None = None,
    lse: torch.Tensor | None = None,
    prepared=None,
) -> torch.Tensor:
    """KL(teacher || student) of the indexer on the selected tokens, a float32 scalar.

    ``index_q[T,G,Di]``, ``index_k[T,1,Di]`` (the student, differentiable), ``q[T,Hq,D]``,
    ``k[T,G,D]`` (the teacher, used detached), ``indices[T,G,K]`` (this step's top-k
    selection), ``cu_seqlens`` and ``max_seqlen`` as for ``m3_sparse_attention``.
    ``index_scale`` scales the student logits (``m3_index_score``'s ``scale``);
    ``scale`` the teacher's (default ``D ** -0.5``, the attention's). ``lse``: the
    attention's ``[T, Hq]`` LSE on the same inputs, reused by the teacher.
    """
    if index_q.ndim != 3 or index_k.ndim != 3 or q.ndim != 3 or k.ndim != 3:
        raise ValueError("expected index_q[T,G,Di], index_k[T,1,Di], q[T,Hq,D] and k[T,G,D]")
    total, groups, index_dim = index_q.shape
    if index_k.shape != (total, 1, index_dim) or index_dim < 1 or groups < 1:
        raise ValueError("expected index_q[T,G,Di] and index_k[T,1,Di] with G, Di > 0")
    if q.shape[0] != total or k.shape[0] != total or k.shape[1] != groups or q.shape[2] != k.shape[2]:
        raise ValueError("q[T,Hq,D] and k[T,G,D] must match the index tensors' T and G")
    if q.shape[1] % groups or q.shape[2] <= 0:
        raise ValueError("Hq must be a positive multiple of G")
    for x in (index_q, q):
        if x.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise TypeError("inputs must have BF16, FP16, or FP32 dtype")
    if index_k.dtype != index_q.dtype or k.dtype != q.dtype:
        raise TypeError("index_q/index_k and q/k must share their dtypes")
    if indices.ndim != 3 or indices.shape[:2] != (total, groups) or indices.dtype != torch.int32:
        raise ValueError("indices must be int32 [T,G,K]")
    if cu_seqlens.ndim != 1 or cu_seqlens.numel() < 2 or cu_seqlens.dtype != torch.int32:
        raise ValueError("cu_seqlens must be int32 [num_sequences + 1]")
    if any(x.device != index_q.device for x in (index_k, q, k, indices, cu_seqlens)):
        raise ValueError("All inputs must reside on the same device.")
    if not isinstance(block_size, int) or block_size <= 0:
        raise ValueError("block_size must be a positive integer.")
    if not isinstance(max_seqlen, int) or max_seqlen <= 0:
        raise ValueError("max_seqlen must be a positive integer.")
    if index_dim > 256:
        raise ValueError("index_dim must be at most 256")
    lengths = sequence_lengths(cu_seqlens, total, prepared)
    if max(lengths) > max_seqlen:
        raise ValueError("max_seqlen is smaller than an actual sequence.")
    teacher_scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    if not (math.isfinite(teacher_scale) and math.isfinite(index_scale)):
        raise ValueError("scale must be finite.")
    if lse is not None and (lse.shape != (total, q.shape[1]) or lse.dtype != torch.float32
                            or lse.device != q.device):
        raise ValueError("lse must be the attention's float32 [T, Hq] LSE")
    _lib.require_cuda(index_q)
    bounds = [0]
    for n in lengths:
        bounds.append(bounds[-1] + n)
    need_grad = torch.is_grad_enabled() and (index_q.requires_grad or index_k.requires_grad)
    return _IndexKL.apply(index_q, index_k, q, k, indices, cu_seqlens, block_size, float(index_scale),
                          teacher_scale, lse, bounds, need_grad)
