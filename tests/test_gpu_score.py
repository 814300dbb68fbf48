"""Index score parity on the GPU (restates the reference's test_triton_score.py
strategy): forward and backward against the float64 oracle at the reference's
gate, golden vectors produced by the reference, exact ties, low-bit winners,
group independence, and no_grad bit-identity."""

import numpy as np
import pytest
import torch

from msa_triton_b200 import _dispatch, m3_index_score, m3_topk
from oracle import msa_oracle as O
from tests.helpers import GATE, assert_close_with_neginf, cu_of, np64

pytestmark = pytest.mark.gpu

DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def _run(q, k, cu, max_seqlen, block_size, scale, upstream, device):
    qd = q.to(device).clone().requires_grad_()
    kd = k.to(device).clone().requires_grad_()
    s = m3_index_score(qd, kd, cu.to(device), max_seqlen, block_size=block_size, scale=scale)
    s.backward(upstream.to(device))
    return s, qd.grad, kd.grad


@pytest.mark.parametrize("lengths,groups,dim,block_size,scale", [
    ([1], 1, 1, 4, 1.0), ([0, 0], 2, 7, 4, 1.0), ([0, 3, 0, 2, 0], 2, 7, 4, 1.0), ([3, 7], 2, 7, 4, 1.0),
    ([7, 11], 4, 16, 8, 0.5), ([9], 2, 64, 4, 1.0), ([5], 4, 128, 128, 1.0), ([300, 77], 3, 64, 16, -0.5),
])
def test_score_forward_backward_fp64(lengths, groups, dim, block_size, scale, cuda_device):
    gen = torch.Generator().manual_seed(731)
    q = torch.randn(sum(lengths), groups, dim, generator=gen).to(torch.bfloat16)
    k = torch.randn(sum(lengths), 1, dim, generator=gen).to(torch.bfloat16)
    cu = cu_of(lengths)
    max_seqlen = max(lengths) + block_size  # includes entirely invalid output blocks
    expected = O.index_score(np64(q), np64(k), cu.numpy(), max_seqlen, block_size=block_size, scale=scale)
    upstream = torch.randn(expected.shape, generator=gen).to(torch.bfloat16).float()
    s, dq, dk = _run(q, k, cu, max_seqlen, block_size, scale, upstream, cuda_device)
    assert s.dtype == torch.float32 and s.shape == expected.shape
    assert_close_with_neginf(s, torch.from_numpy(expected))
    edq, edk = O.index_score_backward(np64(q), np64(k), cu.numpy(), max_seqlen, upstream.double().numpy(),
                                      block_size=block_size, scale=scale)
    torch.testing.assert_close(dq.cpu(), torch.from_numpy(edq).to(dq.dtype), **GATE)
    torch.testing.assert_close(dk.cpu(), torch.from_numpy(edk).to(dk.dtype), **GATE)


def test_score_golden_vectors_from_reference(golden, cuda_device):
    """Every score case the reference's FP64 oracle produced (random, ties, low-bit winners, dtypes)."""
    g = golden.stage("score")
    for c in golden.cases("score"):
        n = c["name"]
        dtype = DT[c["dtype"]]
        q = torch.from_numpy(g[f"{n}/iq"]).to(dtype)
        k = torch.from_numpy(g[f"{n}/ik"]).to(dtype)
        cu = torch.from_numpy(g[f"{n}/cu"])
        up = torch.from_numpy(g[f"{n}/dscores"]).float()
        s, dq, dk = _run(q, k, cu, c["max_seqlen"], c["block_size"], c["scale"], up, cuda_device)
        assert_close_with_neginf(s, torch.from_numpy(g[f"{n}/scores"]))
        torch.testing.assert_close(dq.cpu(), torch.from_numpy(g[f"{n}/diq"]).to(dtype), **GATE, msg=n)
        torch.testing.assert_close(dk.cpu(), torch.from_numpy(g[f"{n}/dik"]).to(dtype), **GATE, msg=n)


@pytest.mark.parametrize("lengths", [[127], [128], [129], [1, 129, 257]])
def test_score_causal_block_and_packing_boundaries(lengths, cuda_device):
    gen = torch.Generator().manual_seed(97)
    q = torch.randn(sum(lengths), 2, 4, generator=gen).to(torch.bfloat16)
    k = torch.randn(sum(lengths), 1, 4, generator=gen).to(torch.bfloat16)
    cu = cu_of(lengths)
    actual = m3_index_score(q.to(cuda_device), k.to(cuda_device), cu.to(cuda_device), max(lengths), block_size=128)
    expected = O.index_score(np64(q), np64(k), cu.numpy(), max(lengths), block_size=128)
    assert_close_with_neginf(actual, torch.from_numpy(expected))


def test_score_groups_remain_independent(cuda_device):
    q = torch.tensor([[[1., 0.], [0., 1.]]] * 4, dtype=torch.bfloat16, device=cuda_device)
    k = torch.tensor([[[9., 1.]], [[1., 8.]], [[0., 0.]], [[0., 0.]]], dtype=torch.bfloat16, device=cuda_device)
    scores = m3_index_score(q, k, cu_of([4], cuda_device), 4, block_size=1)
    assert scores.shape == (4, 2, 4)
    assert scores[-1, 0].argmax().item() == 0
    assert scores[-1, 1].argmax().item() == 1


def test_no_grad_with_trainable_inputs_preserves_score_values(cuda_device):
    q = torch.tensor([[[1.0, 2**-12, 1.0]]] * 2, dtype=torch.bfloat16, device=cuda_device, requires_grad=True)
    k = torch.tensor([[[1.0, 2**-12, -1.0]], [[0.0, 0.0, 0.0]]], dtype=torch.bfloat16, device=cuda_device,
                     requires_grad=True)
    cu = cu_of([2], cuda_device)
    trainable = m3_index_score(q, k, cu, 4, block_size=2)
    with torch.no_grad():
        inference = m3_index_score(q, k, cu, 4, block_size=2)
    assert trainable.requires_grad and not inference.requires_grad
    torch.testing.assert_close(trainable, inference, atol=0, rtol=0)


def test_score_empty_batch_has_shaped_gradients(cuda_device):
    q = torch.zeros(0, 2, 8, device=cuda_device, requires_grad=True)
    k = torch.zeros(0, 1, 8, device=cuda_device, requires_grad=True)
    s = m3_index_score(q, k, cu_of([0, 0], cuda_device), 4, block_size=2)
    assert s.shape == (0, 2, 2)
    s.sum().backward()
    assert q.grad.shape == q.shape and k.grad.shape == k.shape


def test_score_does_not_mutate_inputs(cuda_device):
    gen = torch.Generator().manual_seed(5)
    q = torch.randn(40, 2, 16, generator=gen).bfloat16().to(cuda_device)
    k = torch.randn(40, 1, 16, generator=gen).bfloat16().to(cuda_device)
    q0, k0 = q.clone(), k.clone()
    m3_index_score(q, k, cu_of([40], cuda_device), 40, block_size=8)
    assert torch.equal(q, q0) and torch.equal(k, k0)


def unit_rms(x):
    return x / x.square().mean(-1, keepdim=True).sqrt()


@pytest.mark.parametrize("lengths,groups,dim,dtype,scale", [
    ([1000, 3000], 8, 64, "bf16", 1.0), ([129, 16, 1, 700], 4, 128, "f16", -0.5), ([2048], 2, 64, "bf16", 0.125),
    ([300, 0, 77], 16, 64, "bf16", 1.0), ([257], 1, 128, "bf16", 2.0),
])
def test_tensor_core_score_matches_fp64(lengths, groups, dim, dtype, scale, cuda_device):
    """tcgen05 score kernel: -inf pattern exact, values within the float32 accumulation bound of
    Di exact products (Di * 2^-24 * max|iq| * max|ik| * |scale|, plus one float32 ulp of the score);
    top-k of these scores matches the oracle's top-k of the same scores exactly."""
    gen = torch.Generator().manual_seed(sum(lengths) + groups)
    q = unit_rms(torch.randn(sum(lengths), groups, dim, generator=gen)).to(DT[dtype])
    k = unit_rms(torch.randn(sum(lengths), 1, dim, generator=gen)).to(DT[dtype])
    cu = cu_of(lengths)
    assert _dispatch.score_uses_tc(q, 128)
    with torch.no_grad():
        s = m3_index_score(q.to(cuda_device), k.to(cuda_device), cu.to(cuda_device), max(lengths), scale=scale)
    ref = O.index_score(np64(q), np64(k), cu.numpy(), max(lengths), block_size=128, scale=scale)
    got = s.cpu().double().numpy()
    assert np.array_equal(np.isneginf(got), np.isneginf(ref)) and not np.isnan(got).any()
    fin = np.isfinite(ref)
    qn = np.linalg.norm(np64(q), axis=-1).max()
    kn = np.linalg.norm(np64(k), axis=-1).max()
    bound = dim * 2.0 ** -24 * qn * kn * abs(scale) + 2.0 ** -23 * np.abs(ref[fin])
    assert (np.abs(got[fin] - ref[fin]) <= bound).all(), float(np.abs(got[fin] - ref[fin]).max())
    ids = m3_topk(s, cu.to(cuda_device), block_size=128, topk_blocks=8, local_blocks=1)
    np.testing.assert_array_equal(ids.cpu().numpy(), O.topk(s.cpu().numpy(), cu.numpy(), block_size=128,
                                                             topk_blocks=8, local_blocks=1))


def test_tensor_core_score_same_bits_with_and_without_grad(cuda_device):
    gen = torch.Generator().manual_seed(5)
    q = unit_rms(torch.randn(600, 4, 64, generator=gen)).bfloat16().to(cuda_device)
    k = unit_rms(torch.randn(600, 1, 64, generator=gen)).bfloat16().to(cuda_device)
    cu = cu_of([600], cuda_device)
    with torch.no_grad():
        a = m3_index_score(q, k, cu, 600)
    b = m3_index_score(q.clone().requires_grad_(), k.clone().requires_grad_(), cu, 600)
    assert torch.equal(a, b.detach())
