"""msa_k2q_build_noalloc (the allocation-free k2q CSR entry point, scratch in a
fixed device array) against msa_k2q_build on the same inputs, two calls in a
row: the fixed scratch is reused and no state carries over between calls.
The file name sorts last so the test also runs after every other GPU test."""

import ctypes

import pytest
import torch

from msa_triton_b200 import _lib
from msa_triton_b200.k2q import build_k2q_csr
from msa_triton_b200.layout import block_prefix
from msa_triton_b200.workloads import random_selection
from tests.helpers import cu_of

pytestmark = pytest.mark.gpu


def noalloc_build(ids, cu, lengths, block_size):
    total, groups, slots = ids.shape
    bounds = cu.cpu().tolist()
    host_cu = (ctypes.c_int32 * len(bounds))(*bounds)
    cbl = torch.tensor(block_prefix(lengths, block_size), dtype=torch.int32, device=ids.device)
    row_ptr = torch.full((int(cbl[-1]) * groups + 1,), 7, dtype=torch.int32, device=ids.device)
    query = torch.full((total * groups * slots,), 7, dtype=torch.int32, device=ids.device)
    slot = torch.full_like(query, 7)
    _lib.call("msa_k2q_build_noalloc", _lib.ptr(ids), _lib.ptr(cu), host_cu, _lib.ptr(cbl), len(bounds) - 1, total,
              groups, slots, block_size, _lib.ptr(row_ptr), _lib.ptr(query), _lib.ptr(slot), _lib.stream_of(ids))
    return row_ptr, query, slot


@pytest.mark.parametrize("lengths,groups,topk", [([1024, 1024], 4, 4), ([700, 0, 333, 129], 3, 5), ([4096], 8, 16)])
def test_noalloc_matches_workspace_build_twice(lengths, groups, topk, cuda_device):
    cu = cu_of(lengths, cuda_device)
    calls = []
    for seed in (0, 1):  # different selections: the second call must not see the first one's scratch
        ids = random_selection(lengths, groups, 128, topk, seed=seed).to(cuda_device)
        ids[::7, :, -1] = ids[::7, :, 0]  # some duplicate picks
        want = build_k2q_csr(ids, cu, block_size=128)
        got = noalloc_build(ids, cu, lengths, 128)
        torch.cuda.synchronize()
        assert torch.equal(got[0], want.row_ptr)
        assert torch.equal(got[1], want.query_indices)
        assert torch.equal(got[2], want.slot_indices)
        calls.append(got)
    assert not torch.equal(calls[0][1], calls[1][1])


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_device):
    lengths = [131072]  # histogram of 1024 tiles x 8 groups x 1024 blocks: 32 MiB > the 4 MiB buffer
    cu = cu_of(lengths, cuda_device)
    ids = torch.full((lengths[0], 8, 1), -1, dtype=torch.int32, device=cuda_device)
    with pytest.raises(_lib.MsaError, match="scratch"):
        noalloc_build(ids, cu, lengths, 128)
