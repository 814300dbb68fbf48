"""Private block-to-query CSR metadata (drop-in for ``msa_triton.triton.k2q``).

``build_k2q_csr`` keeps the reference's validation, capacity checks and
output contract (triton/k2q.py:20-128) and builds the CSR with integer CUDA
kernels: per-tile histogram, exclusive scans, stable scatter.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import call, ptr, stream_of
from .layout import block_prefix
from .prepared import host_bounds

_INT32_MAX = 2**31 - 1


@dataclass(frozen=True)
class K2QCSR:
    """Reverse sparse edges, with every tensor on the indices device.

    ``row_ptr`` has ``total_blocks * G + 1`` int32 elements. Row
    ``global_block * G + group`` lists global packed query token ids in
    ``query_indices`` and their selection slots in ``slot_indices``, ordered by
    query then slot. Both edge arrays have capacity ``T * G * K``; entries past
    ``row_ptr[-1]`` are ``-1``. ``cu_block_lens`` is the int32 prefix sum of
    each sequence's block count. Duplicate selected blocks keep separate edges.
    """

    row_ptr: torch.Tensor
    query_indices: torch.Tensor
    slot_indices: torch.Tensor
    cu_block_lens: torch.Tensor


@torch.no_grad()
def build_k2q_csr(indices: torch.Tensor, cu_seqlens: torch.Tensor, *, block_size: int, prepared=None) -> K2QCSR:
    """Invert ``indices[T,G,K]`` into deterministic block/group CSR rows
    (``prepared``: boundaries from ``prepare_batch``, no device read)."""
    if indices.ndim != 3 or indices.dtype != torch.int32:
        raise ValueError("indices must be an int32 tensor with shape [T,G,K]")
    total, groups, slots = indices.shape
    if groups <= 0:
        raise ValueError("indices must have at least one group")
    if not isinstance(block_size, int) or isinstance(block_size, bool) or block_size <= 0:
        raise ValueError("block_size must be a positive integer")
    if cu_seqlens.ndim != 1 or cu_seqlens.dtype != torch.int32 or cu_seqlens.numel() < 2:
        raise ValueError("cu_seqlens must be a rank-1 int32 tensor with at least two entries")
    if cu_seqlens.device != indices.device:
        raise ValueError("cu_seqlens and indices must be on the same device")
    capacity = total * groups * slots
    if capacity > _INT32_MAX:
        raise OverflowError("T * G * K exceeds int32 edge capacity")
    bounds = host_bounds(cu_seqlens, prepared)
    lengths = [end - start for start, end in zip(bounds[:-1], bounds[1:])]
    if bounds[0] != 0 or bounds[-1] != total or any(length < 0 for length in lengths):
        raise ValueError("cu_seqlens must span T with nondecreasing boundaries starting at zero")
    block_bounds = block_prefix(lengths, block_size)
    num_rows = block_bounds[-1] * groups
    if num_rows >= _INT32_MAX:
        raise OverflowError("block/group row pointer length exceeds int32 indexing capacity")
    _lib.require_cuda(indices)
    device = indices.device
    row_ptr = torch.empty(num_rows + 1, dtype=torch.int32, device=device)
    query_indices = torch.empty(capacity, dtype=torch.int32, device=device)
    slot_indices = torch.empty(capacity, dtype=torch.int32, device=device)
    ids = indices.contiguous()
    cu = cu_seqlens.contiguous()
    host_cu = (ctypes.c_int32 * len(bounds))(*bounds)
    nseq = len(bounds) - 1
    lib = _lib.load()
    # computed on the device: a host-to-device copy here could queue behind bulk transfers
    cu_block_lens = torch.empty(len(block_bounds), dtype=torch.int32, device=device)
    with torch.cuda.device(device):
        call("msa_block_prefix", ptr(cu), nseq, block_size, ptr(cu_block_lens), stream_of(ids))
    ws_bytes = lib.msa_k2q_workspace_size(host_cu, nseq, groups, block_size)
    workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        call("msa_k2q_build", ptr(ids), ptr(cu), host_cu, ptr(cu_block_lens), nseq, total, groups, slots, block_size,
             ptr(row_ptr), ptr(query_indices), ptr(slot_indices), ptr(workspace), ws_bytes, stream_of(ids))
    return K2QCSR(row_ptr, query_indices, slot_indices, cu_block_lens)
