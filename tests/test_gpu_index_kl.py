"""Index KL loss on the GPU against the float64 oracle (oracle/msa_oracle.py:
index_kl_loss, itself checked against autograd in tests/test_oracle_kl.py).

Tolerances: the precise family (float64 kernels) at the reference suite's gate
(1e-4) on float32 inputs; the tensor-core family's teacher probabilities come
from float32 accumulations of exact bf16 products with an exact LSE (no bf16
rounding of P), so its loss is held to 1e-4 relative and its gradients to the
rounding of their bf16 outputs (rtol 1e-2, atol 1e-3 of the largest value)."""

import numpy as np
import pytest
import torch

from msa_triton_b200 import _dispatch, m3_index_kl_loss, m3_sparse_attention, prepare_batch
from msa_triton_b200.workloads import random_selection
from oracle import msa_oracle as O
from tests.helpers import GATE, cu_of, np64

pytestmark = pytest.mark.gpu


def unit_rms(x):
    return x / x.square().mean(-1, keepdim=True).sqrt()


def inputs(lengths, groups, ratio, dim, index_dim, block, topk, dtype, seed):
    gen = torch.Generator().manual_seed(seed)
    total = sum(lengths)
    iq = unit_rms(torch.randn(total, groups, index_dim, generator=gen)).to(dtype)
    ik = unit_rms(torch.randn(total, 1, index_dim, generator=gen)).to(dtype)
    q = unit_rms(torch.randn(total, groups * ratio, dim, generator=gen)).to(dtype)
    k = unit_rms(torch.randn(total, groups, dim, generator=gen)).to(dtype)
    ids = random_selection(lengths, groups, block, topk, seed=seed)
    return iq, ik, q, k, ids, cu_of(lengths)


def run(iq, ik, q, k, ids, cu, block, index_scale, dev, lse=None):
    a = iq.to(dev).requires_grad_()
    b = ik.to(dev).requires_grad_()
    loss = m3_index_kl_loss(a, b, q.to(dev), k.to(dev), ids.to(dev), cu.to(dev), int((cu[1:] - cu[:-1]).max()),
                            block_size=block, index_scale=index_scale, lse=lse)
    loss.backward()
    torch.cuda.synchronize()
    return float(loss), a.grad, b.grad


@pytest.mark.parametrize("lengths,groups,ratio,dim,index_dim,block,topk,index_scale", [
    ([37, 0, 90], 2, 3, 8, 5, 8, 4, 0.7), ([1, 16, 5], 1, 4, 4, 3, 4, 2, 1.0), ([200], 4, 2, 16, 64, 16, 3, -0.5),
])
def test_precise_family_matches_fp64(lengths, groups, ratio, dim, index_dim, block, topk, index_scale, cuda_device):
    iq, ik, q, k, ids, cu = inputs(lengths, groups, ratio, dim, index_dim, block, topk, torch.float32, 5)
    ids[0] = -1
    assert not _dispatch.attention_uses_tc(q, k, block)
    loss, diq, dik = run(iq, ik, q, k, ids, cu, block, index_scale, cuda_device)
    ref, rdiq, rdik = O.index_kl_loss(np64(iq), np64(ik), np64(q), np64(k), ids.numpy(), cu.numpy(), block_size=block,
                                      index_scale=index_scale)
    assert abs(loss - ref) <= 1e-6 * max(1.0, abs(ref))
    torch.testing.assert_close(diq.cpu(), torch.from_numpy(rdiq).float(), **GATE)
    torch.testing.assert_close(dik.cpu(), torch.from_numpy(rdik).float(), **GATE)


def close_bf16(got, ref, name):
    got = got.detach().double().cpu().numpy()
    scale = float(np.abs(ref).max()) or 1.0
    np.testing.assert_allclose(got, ref, rtol=1e-2, atol=1e-3 * scale, err_msg=name)


@pytest.mark.parametrize("lengths,groups,ratio,topk,dtype", [([700, 300], 2, 8, 4, torch.bfloat16),
                                                             ([1100], 1, 16, 3, torch.bfloat16),
                                                             ([129, 1, 640], 4, 4, 5, torch.bfloat16),
                                                             ([900, 200], 2, 8, 4, torch.float16)])
def test_tensor_core_family_matches_fp64(lengths, groups, ratio, topk, dtype, cuda_device):
    """float16 too: the logit gradients g (|g| <= |index_scale| / (T G), far below float16's
    normal range) enter the gradient MMAs scaled by a power of two."""
    iq, ik, q, k, ids, cu = inputs(lengths, groups, ratio, 128, 64, 128, topk, dtype, 7)
    ids[3] = -1
    ids[20, 0, 1] = ids[20, 0, 0]  # a repeated block id selects its block once
    assert _dispatch.attention_uses_tc(q, k, 128)
    loss, diq, dik = run(iq, ik, q, k, ids, cu, 128, 1.0, cuda_device)
    ref, rdiq, rdik = O.index_kl_loss(np64(iq), np64(ik), np64(q), np64(k), ids.numpy(), cu.numpy(), block_size=128)
    assert abs(loss - ref) <= 1e-4 * abs(ref), (loss, ref)
    close_bf16(diq, rdiq, "diq")
    close_bf16(dik, rdik, "dik")


def test_tensor_core_family_reuses_attention_lse(cuda_device):
    iq, ik, q, k, ids, cu = inputs([900, 200], 2, 8, 128, 64, 128, 4, torch.bfloat16, 9)
    dev = cuda_device
    _, lse = m3_sparse_attention(q.to(dev), k.to(dev), k.to(dev), ids.to(dev), cu.to(dev), 900, return_lse=True)
    a = run(iq, ik, q, k, ids, cu, 128, 1.0, dev, lse=lse)
    b = run(iq, ik, q, k, ids, cu, 128, 1.0, dev)
    assert abs(a[0] - b[0]) <= 1e-5 * abs(b[0])
    torch.testing.assert_close(a[1], b[1], atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(a[2], b[2], atol=1e-2, rtol=1e-2)


def test_no_grad_loss_equals_training_loss_and_grads_are_deterministic(cuda_device):
    iq, ik, q, k, ids, cu = inputs([600], 2, 8, 128, 64, 128, 3, torch.bfloat16, 13)
    dev = cuda_device
    prep = prepare_batch(cu.to(dev))
    with torch.no_grad():
        inference = float(m3_index_kl_loss(iq.to(dev), ik.to(dev), q.to(dev), k.to(dev), ids.to(dev), prep.cu_seqlens,
                                           600, prepared=prep))
    first = run(iq, ik, q, k, ids, cu, 128, 1.0, dev)
    second = run(iq, ik, q, k, ids, cu, 128, 1.0, dev)
    assert inference == pytest.approx(first[0], rel=1e-6)
    # the student pass and the key-owned dIK walk use no atomics: given the same teacher
    # probabilities the gradients repeat exactly; the teacher's LSE comes from the attention
    # forward, whose float32 sums may differ in the last bits between runs
    torch.testing.assert_close(first[1], second[1], atol=1e-2, rtol=1e-2)
    torch.testing.assert_close(first[2], second[2], atol=1e-2, rtol=1e-2)


def test_empty_batch_and_validation(cuda_device):
    dev = cuda_device
    z = lambda *s: torch.zeros(*s, dtype=torch.bfloat16, device=dev, requires_grad=True)
    loss = m3_index_kl_loss(z(0, 2, 64), z(0, 1, 64), z(0, 16, 128), z(0, 2, 128),
                            torch.zeros(0, 2, 4, dtype=torch.int32, device=dev), cu_of([0], dev), 1)
    assert float(loss) == 0.0
    with pytest.raises(ValueError, match="indices"):
        m3_index_kl_loss(z(4, 2, 64), z(4, 1, 64), z(4, 16, 128), z(4, 2, 128),
                         torch.zeros(4, 2, 4, dtype=torch.int64, device=dev), cu_of([4], dev), 4)
