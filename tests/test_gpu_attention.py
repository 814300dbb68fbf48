"""Sparse attention parity on the GPU (restates the reference's
test_triton_attention.py): forward/backward against the float64 oracle at the
reference's gate on the precise path, golden vectors from the reference's FP64
oracle, empty/future-only/non-contiguous inputs, the BF16 rounding regression,
key-owned vs atomic backward, block-order invariance, all seven needs_grad
combinations (CSR built iff K or V needs a gradient), dtypes and GQA 16."""

import importlib

import numpy as np
import pytest
import torch

from msa_triton_b200 import m3_sparse_attention
from msa_triton_b200.sparse_attention import _SparseAttentionAtomicReference
from oracle import msa_oracle as O
from tests.helpers import GATE, assert_close_with_neginf, attention_inputs, cu_of, np64

pytestmark = pytest.mark.gpu


def oracle(tensors, ids, cu, grad, block_size, scale=None):
    q, k, v = (np64(x) for x in tensors)
    out, lse = O.sparse_attention(q, k, v, ids.cpu().numpy(), cu.cpu().numpy(), block_size=block_size, scale=scale)
    grads = None
    if grad is not None:
        grads = O.sparse_attention_backward(q, k, v, ids.cpu().numpy(), cu.cpu().numpy(), np64(grad),
                                            block_size=block_size, scale=scale)
    return torch.from_numpy(out), torch.from_numpy(lse), grads


def check_grads(tensors, grads, needs=(True, True, True)):
    for t, ref, need in zip(tensors, grads, needs):
        if need:
            torch.testing.assert_close(t.grad.cpu(), torch.from_numpy(ref).to(t.dtype), **GATE)
        else:
            assert t.grad is None


@pytest.mark.parametrize("lengths,groups,ratio,dim,block_size,topk,scale", [
    ([1], 1, 1, 5, 128, 1, None), ([7, 3], 2, 2, 8, 3, 3, None), ([17, 5], 3, 1, 16, 8, 2, 0.2),
    ([129, 1], 1, 2, 8, 128, 3, None), ([127, 128, 257], 1, 1, 8, 128, 3, None), ([5, 1, 9], 2, 4, 32, 4, 4, None),
    ([5, 3], 2, 2, 128, 4, 2, None), ([0, 3, 0, 2, 0], 2, 2, 8, 2, 2, None),
])
def test_forward_backward_against_fp64(lengths, groups, ratio, dim, block_size, topk, scale, cuda_device):
    tensors, ids, cu = attention_inputs(lengths, groups, ratio, dim, block_size, topk, cuda_device)
    grad = torch.randn(tensors[0].shape, generator=torch.Generator().manual_seed(5678)).bfloat16()
    exp_out, exp_lse, grads = oracle(tensors, ids, cu, grad, block_size, scale)
    out, lse = m3_sparse_attention(*tensors, ids, cu, max(lengths), block_size=block_size, scale=scale,
                                   return_lse=True)
    assert out.dtype == torch.bfloat16 and lse.dtype == torch.float32 and not lse.requires_grad
    torch.testing.assert_close(out.detach().cpu(), exp_out.bfloat16(), **GATE)
    assert_close_with_neginf(lse, exp_lse)
    out.backward(grad.to(cuda_device))
    check_grads(tensors, grads)


def test_golden_vectors_from_reference(golden, cuda_device):
    g = golden.stage("attention")
    for c in golden.cases("attention"):
        n = c["name"]
        tensors = tuple(torch.from_numpy(g[f"{n}/{x}"]).bfloat16().to(cuda_device).requires_grad_() for x in "qkv")
        ids = torch.from_numpy(g[f"{n}/indices"]).to(cuda_device)
        cu = torch.from_numpy(g[f"{n}/cu"]).to(cuda_device)
        from msa_triton_b200 import _dispatch
        with _dispatch.precise_only():
            out, lse = m3_sparse_attention(*tensors, ids, cu, max(c["lengths"]), block_size=c["block_size"],
                                           scale=c["scale"], return_lse=True)
            out.backward(torch.from_numpy(g[f"{n}/grad_out"]).bfloat16().to(cuda_device))
        torch.testing.assert_close(out.detach().cpu(), torch.from_numpy(g[f"{n}/out"]).bfloat16(), **GATE, msg=lambda m: f"{n}: {m}")
        assert_close_with_neginf(lse, torch.from_numpy(g[f"{n}/lse"]))
        for t, key in zip(tensors, ("dq", "dk", "dv")):
            torch.testing.assert_close(t.grad.cpu(), torch.from_numpy(g[f"{n}/{key}"]).bfloat16(), **GATE,
                                       msg=lambda m, n=n, key=key: f"{n}/{key}: {m}")


@pytest.mark.parametrize("topk", [0, 3])
def test_empty_selection_has_zero_output_and_gradients(topk, cuda_device):
    tensors, ids, cu = attention_inputs([3, 2], 2, 2, 7, 2, topk, cuda_device)
    ids.fill_(-1)
    out, lse = m3_sparse_attention(*tensors, ids, cu, 3, block_size=2, return_lse=True)
    assert torch.count_nonzero(out) == 0 and torch.isneginf(lse).all()
    out.sum().backward()
    for t in tensors:
        assert t.grad is not None and torch.count_nonzero(t.grad) == 0


def test_noncontiguous_inputs_and_masked_queries(cuda_device):
    tensors, ids, cu = attention_inputs([5, 2], 2, 2, 5, 3, 2, cuda_device)
    tensors = tuple(x.detach().transpose(1, 2).contiguous().transpose(1, 2).requires_grad_() for x in tensors)
    ids[1] = -1
    grad = torch.randn(tensors[0].shape, generator=torch.Generator().manual_seed(73)).bfloat16()
    exp_out, exp_lse, grads = oracle(tensors, ids, cu, grad, 3)
    out, lse = m3_sparse_attention(*tensors, ids, cu, 5, block_size=3, return_lse=True)
    torch.testing.assert_close(out.detach().cpu(), exp_out.bfloat16(), **GATE)
    assert_close_with_neginf(lse, exp_lse)
    out.backward(grad.to(cuda_device))
    check_grads(tensors, grads)
    assert torch.count_nonzero(tensors[0].grad[1]) == 0


def test_default_return_is_output_tensor(cuda_device):
    tensors, ids, cu = attention_inputs([2], 1, 1, 4, 2, 1, cuda_device)
    out = m3_sparse_attention(*tensors, ids, cu, 2, block_size=2)
    assert isinstance(out, torch.Tensor) and out.shape == tensors[0].shape


def test_future_only_selected_blocks_are_safely_masked(cuda_device):
    tensors, ids, cu = attention_inputs([5, 2], 1, 2, 8, 3, 1, cuda_device)
    ids.fill_(1)
    grad = torch.ones(tensors[0].shape, dtype=torch.bfloat16)
    exp_out, exp_lse, grads = oracle(tensors, ids, cu, grad, 3)
    out, lse = m3_sparse_attention(*tensors, ids, cu, 5, block_size=3, return_lse=True)
    torch.testing.assert_close(out.detach().cpu(), exp_out.bfloat16(), **GATE)
    assert_close_with_neginf(lse, exp_lse)
    out.sum().backward()
    check_grads(tensors, grads)


def test_empty_packed_input(cuda_device):
    tensors, ids, cu = attention_inputs([0, 0], 1, 2, 8, 4, 1, cuda_device)
    out, lse = m3_sparse_attention(*tensors, ids, cu, 4, block_size=4, return_lse=True)
    assert out.shape == (0, 2, 8) and lse.shape == (0, 2)
    out.sum().backward()
    for t in tensors:
        assert t.grad is not None and t.grad.shape == t.shape


def test_long_key_accumulation_bf16_rounding_regression(cuda_device):
    """Inputs near a BF16 rounding boundary (numpy rng 1234, as the reference's regression)."""
    rng = np.random.default_rng(1234)
    tensors = tuple(torch.from_numpy(rng.standard_normal((512, 1, 8))).float().bfloat16()[255:]
                    .to(cuda_device).detach().requires_grad_() for _ in range(3))
    grad = torch.from_numpy(rng.standard_normal((512, 1, 8))).float().bfloat16()[255:]
    ids = torch.full((257, 1, 3), -1, dtype=torch.int32)
    for token in range(257):
        cur = token // 128
        chosen = [cur] + [b for b in range(cur) if b % 2 == 0]
        ids[token, 0, :len(chosen)] = torch.tensor(chosen, dtype=torch.int32)
    cu = cu_of([257], cuda_device)
    ids = ids.to(cuda_device)
    exp_out, _, grads = oracle(tensors, ids, cu, grad, 128)
    out = m3_sparse_attention(*tensors, ids, cu, 257)
    torch.testing.assert_close(out.detach().cpu(), exp_out.bfloat16(), **GATE)
    out.backward(grad.to(cuda_device))
    check_grads(tensors, grads)


def test_kv_owner_matches_query_owner_and_fp64_with_hotspots(cuda_device):
    lengths, groups, ratio, dim, block = [41, 5], 2, 4, 16, 8
    tensors, _, cu = attention_inputs(lengths, groups, ratio, dim, block, 2, cuda_device)
    sel = torch.full((sum(lengths), groups, 2), -1, dtype=torch.int32)
    start = 0
    for length in lengths:
        for p in range(length):
            sel[start + p, 0, 0] = 0            # one highly shared block
            sel[start + p, 1, 0] = p // block   # only the current block
        start += length
    ids = sel.to(cuda_device)
    prev_inputs = tuple(x.detach().clone().requires_grad_() for x in tensors)
    grad = torch.randn(tensors[0].shape, generator=torch.Generator().manual_seed(819)).bfloat16()
    exp_out, _, grads = oracle(tensors, ids, cu, grad, block)
    out = m3_sparse_attention(*tensors, ids, cu, max(lengths), block_size=block)
    prev, _ = _SparseAttentionAtomicReference.apply(*prev_inputs, ids, cu, block, dim ** -0.5)
    torch.testing.assert_close(out, prev, atol=0, rtol=0)
    torch.testing.assert_close(out.detach().cpu(), exp_out.bfloat16(), **GATE)
    out.backward(grad.to(cuda_device))
    prev.backward(grad.to(cuda_device))
    check_grads(tensors, grads)
    for cur, pr in zip(tensors, prev_inputs):
        torch.testing.assert_close(cur.grad, pr.grad, **GATE)


def test_selected_block_order_preserves_output_and_gradients(cuda_device):
    tensors, ids, cu = attention_inputs([9, 3], 2, 2, 7, 3, 3, cuda_device)
    host = ids.cpu()
    reordered = torch.full(ids.shape, -1, dtype=torch.int32)
    for t in range(ids.shape[0]):
        for g in range(ids.shape[1]):
            row = host[t, g]
            row = row[row >= 0].flip(0)
            reordered[t, g, :row.numel()] = row
    grad = torch.randn(tensors[0].shape, generator=torch.Generator().manual_seed(127)).bfloat16()
    exp_out, _, grads = oracle(tensors, ids, cu, grad, 3)
    for sel in (ids, reordered.to(cuda_device)):
        cur = tuple(x.detach().clone().requires_grad_() for x in tensors)
        out = m3_sparse_attention(*cur, sel, cu, 9, block_size=3)
        torch.testing.assert_close(out.detach().cpu(), exp_out.bfloat16(), **GATE)
        out.backward(grad.to(cuda_device))
        check_grads(cur, grads)


@pytest.mark.parametrize("needs", [(True, False, False), (False, True, False), (False, False, True),
                                   (True, True, False), (True, False, True), (False, True, True), (True, True, True)])
def test_independent_input_gradients_and_q_only_skips_csr(needs, cuda_device, monkeypatch):
    tensors, ids, cu = attention_inputs([0, 5, 0, 3, 0], 2, 2, 8, 3, 2, cuda_device)
    tensors = tuple(x.detach().requires_grad_(n) for x, n in zip(tensors, needs))
    saved = tuple(x.detach().clone() for x in tensors)
    ids[2] = -1
    k2q_module = importlib.import_module("msa_triton_b200.k2q")
    original = k2q_module.build_k2q_csr
    calls = []

    def checked_build(*args, **kwargs):
        assert needs[1] or needs[2], "Q-only backward must not build CSR"
        calls.append(True)
        return original(*args, **kwargs)

    monkeypatch.setattr(k2q_module, "build_k2q_csr", checked_build)
    grad = torch.randn(tensors[0].shape, generator=torch.Generator().manual_seed(190)).bfloat16()
    exp_out, _, grads = oracle(tensors, ids, cu, grad, 3)
    out = m3_sparse_attention(*tensors, ids, cu, 5, block_size=3)
    torch.testing.assert_close(out.detach().cpu(), exp_out.bfloat16(), **GATE)
    out.backward(grad.to(cuda_device))
    assert len(calls) == int(needs[1] or needs[2])
    for t, s in zip(tensors, saved):
        torch.testing.assert_close(t.detach(), s, atol=0, rtol=0)
    check_grads(tensors, grads, needs)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_dtype_and_gqa16_forward_backward_against_fp64(dtype, cuda_device):
    tensors, ids, cu = attention_inputs([5, 3], 1, 16, 8, 3, 2, cuda_device)
    gen = torch.Generator().manual_seed(320)
    tensors = tuple(torch.randn(x.shape, generator=gen).to(dtype=dtype, device=cuda_device).requires_grad_()
                    for x in tensors)
    grad = torch.randn(tensors[0].shape, generator=gen).to(dtype)
    exp_out, exp_lse, grads = oracle(tensors, ids, cu, grad, 3)
    out, lse = m3_sparse_attention(*tensors, ids, cu, 5, block_size=3, return_lse=True)
    torch.testing.assert_close(out.detach().cpu(), exp_out.to(dtype), **GATE)
    assert_close_with_neginf(lse, exp_lse)
    out.backward(grad.to(cuda_device))
    check_grads(tensors, grads)


@pytest.mark.parametrize("needs", [(False, True, False), (False, False, True)])
def test_private_atomic_reference_independent_kv_gradients(needs, cuda_device):
    tensors, ids, cu = attention_inputs([3, 2], 1, 2, 8, 2, 2, cuda_device)
    tensors = tuple(x.detach().requires_grad_(n) for x, n in zip(tensors, needs))
    grad = torch.randn(tensors[0].shape, generator=torch.Generator().manual_seed(801)).bfloat16()
    _, _, grads = oracle(tensors, ids, cu, grad, 2)
    out, _ = _SparseAttentionAtomicReference.apply(*tensors, ids, cu, 2, 8 ** -0.5)
    out.backward(grad.to(cuda_device))
    check_grads(tensors, grads, needs)


def test_duplicate_block_ids_select_once(cuda_device):
    """A repeated id counts once, as in the float64 oracle's mask semantics."""
    tensors, ids, cu = attention_inputs([12], 1, 2, 8, 4, 3, cuda_device)
    ids[:, :, 1] = ids[:, :, 0]
    grad = torch.randn(tensors[0].shape, generator=torch.Generator().manual_seed(3)).bfloat16()
    exp_out, _, grads = oracle(tensors, ids, cu, grad, 4)
    out = m3_sparse_attention(*tensors, ids, cu, 12, block_size=4)
    torch.testing.assert_close(out.detach().cpu(), exp_out.bfloat16(), **GATE)
    out.backward(grad.to(cuda_device))
    check_grads(tensors, grads)
