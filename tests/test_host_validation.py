"""Argument validation of the public ops: same exception types and messages as
the reference (triton/index_score.py:325-355, topk.py:12-29, k2q.py:54-81,
sparse_attention.py:452-483, layout.py:18-30). Validation runs on the host
before any device work, so these run on the CPU."""

import pytest
import torch

from msa_triton_b200 import m3_index_score, m3_sparse_attention, m3_topk
from msa_triton_b200.k2q import build_k2q_csr
from tests.helpers import cu_of


def test_score_rejects_invalid_metadata():
    q = torch.ones(3, 2, 4)
    k = torch.ones(3, 1, 4)
    with pytest.raises(ValueError, match="nondecreasing"):
        m3_index_score(q, k, torch.tensor([0, 2, 1, 3], dtype=torch.int32), 3)
    with pytest.raises(ValueError, match="max_seqlen"):
        m3_index_score(q, k, torch.tensor([0, 3], dtype=torch.int32), 2)
    with pytest.raises(ValueError, match="scale must be finite"):
        m3_index_score(q, k, torch.tensor([0, 3], dtype=torch.int32), 3, scale=float("nan"))
    with pytest.raises(TypeError):
        m3_index_score(q.int(), k.int(), torch.tensor([0, 3], dtype=torch.int32), 3)


def test_cpu_tensors_fail_loudly_instead_of_falling_back():
    q = torch.ones(3, 2, 4)
    k = torch.ones(3, 1, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        m3_index_score(q, k, torch.tensor([0, 3], dtype=torch.int32), 3)
    with pytest.raises(RuntimeError, match="CUDA"):
        m3_topk(torch.zeros(3, 2, 2), torch.tensor([0, 3], dtype=torch.int32), block_size=2, topk_blocks=1)


def test_topk_rejects_bad_arguments():
    s = torch.zeros(3, 2, 2)
    cu = torch.tensor([0, 3], dtype=torch.int32)
    with pytest.raises(ValueError, match="FP32"):
        m3_topk(s.double(), cu)
    with pytest.raises(ValueError, match="local_blocks"):
        m3_topk(s, cu, block_size=2, topk_blocks=1, local_blocks=2)
    with pytest.raises(ValueError, match="enough block slots"):
        m3_topk(s, cu, block_size=1, topk_blocks=1)
    with pytest.raises(ValueError, match="nondecreasing"):
        m3_topk(s, torch.tensor([0, 2, 1, 3], dtype=torch.int32), block_size=2)


def test_k2q_rejects_invalid_metadata_and_capacity_overflow():
    ids = torch.zeros(3, 2, 4, dtype=torch.int32)
    with pytest.raises(ValueError, match="nondecreasing"):
        build_k2q_csr(ids, torch.tensor([0, 2, 1, 3], dtype=torch.int32), block_size=2)
    with pytest.raises(ValueError, match="span T"):
        build_k2q_csr(ids, torch.tensor([0, 2], dtype=torch.int32), block_size=2)
    with pytest.raises(ValueError, match="block_size"):
        build_k2q_csr(ids, torch.tensor([0, 3], dtype=torch.int32), block_size=0)
    # A stride-zero view exercises the check without allocating billions of edges.
    oversized = torch.tensor(0, dtype=torch.int32).expand(1, 2, 2**30)
    with pytest.raises(OverflowError, match="edge capacity"):
        build_k2q_csr(oversized, torch.tensor([0, 1], dtype=torch.int32), block_size=1)


def _attn_args():
    q = torch.randn(2, 1, 4)
    k = torch.randn(2, 1, 4)
    v = torch.randn(2, 1, 4)
    ids = torch.zeros(2, 1, 1, dtype=torch.int32)
    return q, k, v, ids, cu_of([2])


@pytest.mark.parametrize("scale", [float("nan"), float("inf"), -float("inf")])
def test_attention_rejects_nonfinite_scale(scale):
    q, k, v, ids, cu = _attn_args()
    with pytest.raises(ValueError, match="scale must be finite"):
        m3_sparse_attention(q, k, v, ids, cu, 2, block_size=2, scale=scale)


def test_attention_rejects_invalid_sequence_metadata():
    q, k, v, ids, cu = _attn_args()
    with pytest.raises(ValueError, match="positive integer"):
        m3_sparse_attention(q, k, v, ids, cu, 0, block_size=2)
    with pytest.raises(ValueError, match="smaller"):
        m3_sparse_attention(q, k, v, ids, cu, 1, block_size=2)
    cu[-1] = 1
    with pytest.raises(ValueError, match="end at total_tokens"):
        m3_sparse_attention(q, k, v, ids, cu, 2, block_size=2)


def test_attention_rejects_bad_shapes_and_dtypes():
    q, k, v, ids, cu = _attn_args()
    with pytest.raises(ValueError, match="multiple of G"):
        m3_sparse_attention(torch.randn(2, 3, 4), torch.randn(2, 2, 4), torch.randn(2, 2, 4),
                            torch.zeros(2, 2, 1, dtype=torch.int32), cu, 2, block_size=2)
    with pytest.raises(TypeError):
        m3_sparse_attention(q.double(), k.double(), v.double(), ids, cu, 2, block_size=2)
    with pytest.raises(ValueError, match="int32"):
        m3_sparse_attention(q, k, v, ids.long(), cu, 2, block_size=2)


def test_prepare_batch_validates_and_checks_its_tensor():
    from msa_triton_b200 import prepare_batch

    cu = torch.tensor([0, 3, 3, 7], dtype=torch.int32)
    p = prepare_batch(cu)
    assert p.bounds == (0, 3, 3, 7) and p.lengths == [3, 0, 4] and p.total_tokens == 7 and p.max_seqlen == 4
    assert prepare_batch(cu, bounds=[0, 3, 3, 7]).bounds == p.bounds  # host copy handed over, nothing read
    with pytest.raises(ValueError, match="nondecreasing"):
        prepare_batch(torch.tensor([0, 2, 1], dtype=torch.int32))
    with pytest.raises(ValueError, match="one entry per"):
        prepare_batch(cu, bounds=[0, 7])
    with pytest.raises(ValueError, match="int32"):
        prepare_batch(cu.long())
    other = torch.tensor([0, 3, 3, 7], dtype=torch.int32)
    scores = torch.zeros(7, 1, 4)
    with pytest.raises(ValueError, match="different cu_seqlens"):
        m3_topk(scores, other, block_size=2, topk_blocks=1, prepared=p)
    with pytest.raises(ValueError, match="end at T"):  # the prepared bounds are validated like read ones
        m3_topk(torch.zeros(6, 1, 4), cu, block_size=2, topk_blocks=1, prepared=p)
