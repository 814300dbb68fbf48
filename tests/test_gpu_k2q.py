"""k2q CSR parity on the GPU (restates the reference's test_k2q.py): bit-exact
against a pure-Python inversion, the reference's golden outputs and the oracle,
with random/invalid ids, duplicates, hot rows, empty sequences, non-contiguous
input, and benchmark-size properties (row sums, ordering, multiset)."""

from collections import Counter

import numpy as np
import pytest
import torch

from msa_triton_b200.k2q import build_k2q_csr
from oracle import msa_oracle as O
from tests.helpers import cu_of, random_distinct_selection

pytestmark = pytest.mark.gpu


def _invert_python(indices, lengths, block_size):
    tokens, groups, slots = indices.shape
    values = indices.tolist()
    prefix = [0]
    for length in lengths:
        prefix.append(prefix[-1] + (length + block_size - 1) // block_size)
    rows = [[] for _ in range(prefix[-1] * groups)]
    edges = []
    start = 0
    for seq, length in enumerate(lengths):
        nblocks = (length + block_size - 1) // block_size
        for local in range(length):
            query = start + local
            for g in range(groups):
                for s in range(slots):
                    b = values[query][g][s]
                    if b < 0 or b >= nblocks or b * block_size > local:
                        continue
                    row = (prefix[seq] + b) * groups + g
                    rows[row].append((query, s))
                    edges.append((row, query, s))
        start += length
    ptr, qs, ss = [0], [], []
    for row in rows:
        for query, s in sorted(row):
            qs.append(query)
            ss.append(s)
        ptr.append(len(qs))
    pad = tokens * groups * slots - len(qs)
    return ptr, qs + [-1] * pad, ss + [-1] * pad, prefix, edges


def _check(ids_cpu, lengths, block_size, device):
    ids = ids_cpu.to(device)
    original = ids.clone()
    result = build_k2q_csr(ids, cu_of(lengths, device), block_size=block_size)
    ptr, qs, ss, prefix, edges = _invert_python(ids_cpu, lengths, block_size)
    for actual, expected in ((result.row_ptr, ptr), (result.query_indices, qs), (result.slot_indices, ss),
                             (result.cu_block_lens, prefix)):
        assert actual.dtype == torch.int32 and actual.device == ids.device and not actual.requires_grad
        torch.testing.assert_close(actual.cpu(), torch.tensor(expected, dtype=torch.int32), rtol=0, atol=0)
    torch.testing.assert_close(ids, original, rtol=0, atol=0)
    got = []
    p, q, s = result.row_ptr.cpu().tolist(), result.query_indices.cpu().tolist(), result.slot_indices.cpu().tolist()
    for row, (lo, hi) in enumerate(zip(p[:-1], p[1:])):
        got += [(row, q[e], s[e]) for e in range(lo, hi)]
    assert Counter(got) == Counter(edges)
    return result


@pytest.mark.parametrize("lengths,groups,slots,block_size", [
    ([1], 1, 4, 128), ([3, 5], 3, 5, 2), ([0, 3, 0, 2, 0], 2, 4, 2), ([127, 128, 129], 4, 5, 128),
    ([0, 0], 3, 5, 128), ([4, 2], 3, 0, 2), ([300, 41], 2, 40, 3),
])
def test_k2q_python_inversion(lengths, groups, slots, block_size, cuda_device):
    max_blocks = (max(lengths) + block_size - 1) // block_size
    ids = torch.randint(-2, max_blocks + 4, (sum(lengths), groups, slots),
                        generator=torch.Generator().manual_seed(951), dtype=torch.int32)
    _check(ids, lengths, block_size, cuda_device)


def test_k2q_golden_vectors_from_reference(golden, cuda_device):
    g = golden.stage("k2q")
    for c in golden.cases("k2q"):
        n = c["name"]
        ids = torch.from_numpy(g[f"{n}/indices"]).to(cuda_device)
        r = build_k2q_csr(ids, torch.from_numpy(g[f"{n}/cu"]).to(cuda_device), block_size=c["block_size"])
        for key in ("row_ptr", "query_indices", "slot_indices", "cu_block_lens"):
            np.testing.assert_array_equal(getattr(r, key).cpu().numpy(), g[f"{n}/{key}"], err_msg=f"{n}/{key}")


def test_k2q_duplicate_slots_and_sequence_local_blocks(cuda_device):
    ids = torch.tensor([[[0, 0, 1], [1, 0, -1]], [[0, -1, 8], [0, 0, 1]], [[1, 0, 1], [0, 1, -2]],
                        [[0, 0, 1], [0, -1, 9]], [[0, 0, -1], [0, 0, -1]]], dtype=torch.int32)
    r = _check(ids, [3, 2], 2, cuda_device)
    assert r.cu_block_lens.cpu().tolist() == [0, 2, 3]
    ptr = r.row_ptr.cpu().tolist()
    assert set(r.query_indices[ptr[4]:ptr[5]].cpu().tolist()) == {3, 4}


def test_k2q_all_invalid(cuda_device):
    ids = torch.full((7, 2, 4), 99, dtype=torch.int32)
    ids[:, :, 0] = -1
    r = _check(ids, [3, 4], 2, cuda_device)
    assert r.row_ptr.count_nonzero().item() == 0
    assert (r.query_indices == -1).all().item()


def test_k2q_noncontiguous_input(cuda_device):
    base = torch.tensor([[[0, 1, 2, -1], [0, -1, 9, 0]]] * 5, dtype=torch.int32)
    _check(base.transpose(1, 2), [2, 3], 2, cuda_device)


def test_k2q_many_blocks_exceed_one_cursor_pass(cuda_device):
    """More blocks per sequence than one shared-memory cursor pass holds."""
    lengths, groups, slots, b = [5000, 300], 2, 6, 1
    ids = random_distinct_selection(lengths, groups, b, slots, seed=4)
    _check(ids, lengths, b, cuda_device)


@pytest.mark.parametrize("cfg", [4, 3])
def test_k2q_benchmark_size_against_oracle(cfg, cuda_device):
    from msa_triton_b200.workloads import CONFIGS
    w = CONFIGS[cfg]
    ids = random_distinct_selection(w.lengths, w.groups, w.block_size, w.topk_blocks, seed=cfg)
    cu = w.cu_seqlens()
    r = build_k2q_csr(ids.to(cuda_device), cu.to(cuda_device), block_size=w.block_size)
    want = O.k2q_csr(ids.numpy(), cu.numpy(), block_size=w.block_size)
    for arr, key in zip(want, ("row_ptr", "query_indices", "slot_indices", "cu_block_lens")):
        np.testing.assert_array_equal(getattr(r, key).cpu().numpy(), arr, err_msg=key)
