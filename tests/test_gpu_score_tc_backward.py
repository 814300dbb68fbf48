"""Tensor-core index score with gradients: the forward records the float64
winner state (float32 winners where an error margin separates them from every
other key, float64 recomputation elsewhere) and the backward transposes it
without atomics. Gradients against the float64 oracle at the reference's gate
(atol = rtol = 1e-4), with exact ties (gradient split equally) and against the
float64 kernel family on the same inputs."""

import numpy as np
import pytest
import torch

from msa_triton_b200 import _dispatch, m3_index_score
from oracle import msa_oracle as O
from tests.helpers import GATE, assert_close_with_neginf, cu_of, np64

pytestmark = pytest.mark.gpu

DT = {"bf16": torch.bfloat16, "f16": torch.float16}


def unit_rms(x):
    return x / x.square().mean(-1, keepdim=True).sqrt()


def grads(q, k, cu, max_seqlen, scale, upstream, device, precise=False):
    qd = q.to(device).clone().requires_grad_()
    kd = k.to(device).clone().requires_grad_()
    if precise:
        with _dispatch.precise_only():
            s = m3_index_score(qd, kd, cu.to(device), max_seqlen, scale=scale)
            s.backward(upstream.to(device))
    else:
        s = m3_index_score(qd, kd, cu.to(device), max_seqlen, scale=scale)
        s.backward(upstream.to(device))
    torch.cuda.synchronize()
    return s.detach(), qd.grad, kd.grad


@pytest.mark.parametrize("lengths,groups,dim,dtype,scale", [
    ([1000, 1500], 8, 64, "bf16", 1.0), ([129, 16, 1, 700], 4, 128, "f16", -0.5), ([2048], 1, 64, "bf16", 0.125),
    ([300, 0, 77], 16, 64, "bf16", 1.0),
])
def test_tc_score_backward_matches_fp64(lengths, groups, dim, dtype, scale, cuda_device):
    gen = torch.Generator().manual_seed(sum(lengths) * 3 + groups)
    q = unit_rms(torch.randn(sum(lengths), groups, dim, generator=gen)).to(DT[dtype])
    k = unit_rms(torch.randn(sum(lengths), 1, dim, generator=gen)).to(DT[dtype])
    cu = cu_of(lengths)
    assert _dispatch.score_uses_tc(q, 128)
    nb = (max(lengths) + 127) // 128
    upstream = torch.randn(sum(lengths), groups, nb, generator=gen)
    s, dq, dk = grads(q, k, cu, max(lengths), scale, upstream, cuda_device)
    with torch.no_grad():
        s_plain = m3_index_score(q.to(cuda_device), k.to(cuda_device), cu.to(cuda_device), max(lengths), scale=scale)
    assert torch.equal(s, s_plain)  # the state adds nothing to the public scores
    edq, edk = O.index_score_backward(np64(q), np64(k), cu.numpy(), max(lengths), upstream.double().numpy(),
                                      block_size=128, scale=scale)
    torch.testing.assert_close(dq.cpu(), torch.from_numpy(edq).to(dq.dtype), **GATE)
    torch.testing.assert_close(dk.cpu(), torch.from_numpy(edk).to(dk.dtype), **GATE)


def test_tc_score_backward_exact_ties(cuda_device):
    """Five distinct key rows repeated: every block ties between the copies of its
    best key, so every winner goes through the float64 fixup and splits the gradient."""
    gen = torch.Generator().manual_seed(77)
    lengths, groups, dim = [600, 260], 2, 64
    total = sum(lengths)
    q = unit_rms(torch.randn(total, groups, dim, generator=gen)).bfloat16()
    base = unit_rms(torch.randn(5, 1, dim, generator=gen)).bfloat16()
    k = base[torch.arange(total) % 5]
    cu = cu_of(lengths)
    nb = (max(lengths) + 127) // 128
    upstream = torch.randn(total, groups, nb, generator=gen)
    s, dq, dk = grads(q, k, cu, max(lengths), 1.0, upstream, cuda_device)
    exp = O.index_score(np64(q), np64(k), cu.numpy(), max(lengths), block_size=128, scale=1.0)
    assert_close_with_neginf(s, torch.from_numpy(exp), atol=1e-3, rtol=1e-3)
    edq, edk = O.index_score_backward(np64(q), np64(k), cu.numpy(), max(lengths), upstream.double().numpy(),
                                      block_size=128, scale=1.0)
    torch.testing.assert_close(dq.cpu(), torch.from_numpy(edq).to(dq.dtype), **GATE)
    torch.testing.assert_close(dk.cpu(), torch.from_numpy(edk).to(dk.dtype), **GATE)


def test_tc_score_backward_agrees_with_float64_kernels(cuda_device):
    gen = torch.Generator().manual_seed(9)
    lengths, groups, dim = [777, 1300], 8, 64
    q = unit_rms(torch.randn(sum(lengths), groups, dim, generator=gen)).bfloat16()
    k = unit_rms(torch.randn(sum(lengths), 1, dim, generator=gen)).bfloat16()
    cu = cu_of(lengths)
    upstream = torch.randn(sum(lengths), groups, (max(lengths) + 127) // 128, generator=gen)
    _, dq, dk = grads(q, k, cu, max(lengths), 1.0, upstream, cuda_device)
    _, pdq, pdk = grads(q, k, cu, max(lengths), 1.0, upstream, cuda_device, precise=True)
    torch.testing.assert_close(dq, pdq, **GATE)
    torch.testing.assert_close(dk, pdk, **GATE)
