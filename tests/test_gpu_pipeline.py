"""Three-stage composition on the GPU (restates the reference's
test_pipeline.py): score -> top-k -> attention against the float64 oracle, and
a projection -> MSA -> projection module whose parameter gradients match a
float64 torch autograd reference with the same frozen selection."""

import numpy as np
import pytest
import torch

from msa_triton_b200 import m3_index_score, m3_sparse_attention, m3_topk
from oracle import msa_oracle as O
from tests.helpers import GATE, cu_of, np64

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("lengths,groups,ratio,dim", [([1, 3], 1, 1, 8), ([7, 5], 2, 2, 16), ([17, 9], 4, 1, 8)])
def test_composed_pipeline_fp64(lengths, groups, ratio, dim, cuda_device):
    gen = torch.Generator().manual_seed(51)
    total, block, topk = sum(lengths), 4, 2
    cu = cu_of(lengths, cuda_device)
    iq = torch.randn(total, groups, dim, generator=gen).bfloat16().to(cuda_device)
    ik = torch.randn(total, 1, dim, generator=gen).bfloat16().to(cuda_device)
    q, k, v = [torch.randn(total, h, dim, generator=gen).bfloat16().to(cuda_device).requires_grad_()
               for h in (groups * ratio, groups, groups)]
    score = m3_index_score(iq, ik, cu, max(lengths), block_size=block)
    ref_score = O.index_score(np64(iq), np64(ik), cu.cpu().numpy(), max(lengths), block_size=block)
    torch.testing.assert_close(score.cpu(), torch.from_numpy(ref_score).float(), **GATE)
    ids = m3_topk(score, cu, block_size=block, topk_blocks=topk)
    np.testing.assert_array_equal(ids.cpu().numpy(), O.topk(score.cpu().numpy(), cu.cpu().numpy(), block_size=block,
                                                            topk_blocks=topk, local_blocks=1))
    out = m3_sparse_attention(q, k, v, ids, cu, max(lengths), block_size=block)
    ref_out, _ = O.sparse_attention(np64(q), np64(k), np64(v), ids.cpu().numpy(), cu.cpu().numpy(), block_size=block)
    torch.testing.assert_close(out.detach().cpu(), torch.from_numpy(ref_out).bfloat16(), **GATE)
    grad = torch.randn(out.shape, generator=gen).bfloat16()
    out.backward(grad.to(cuda_device))
    refs = O.sparse_attention_backward(np64(q), np64(k), np64(v), ids.cpu().numpy(), cu.cpu().numpy(), np64(grad),
                                       block_size=block)
    for t, r in zip((q, k, v), refs):
        torch.testing.assert_close(t.grad.cpu(), torch.from_numpy(r).bfloat16(), **GATE)


def _dense_reference_attention(q, k, v, ids, lengths, block):
    """float64 torch autograd attention with an explicit mask (small sizes only)."""
    total, hq, dim = q.shape
    groups = k.shape[1]
    ratio = hq // groups
    out = torch.zeros_like(q)
    start = 0
    for n in lengths:
        for g in range(groups):
            pos = torch.arange(n)
            sel = ((pos[None, :, None] // block) == ids[start:start + n, g].cpu().long()[:, None, :]).any(-1)
            allowed = sel & (pos[None, :] <= pos[:, None])
            hs = slice(g * ratio, (g + 1) * ratio)
            logits = torch.einsum("trd,kd->trk", q[start:start + n, hs], k[start:start + n, g]) * dim ** -0.5
            logits = logits.masked_fill(~allowed[:, None, :], -float("inf"))
            probs = torch.softmax(logits, dim=-1).nan_to_num(0.0)
            out = out.index_add(0, torch.arange(start, start + n),
                                torch.nn.functional.pad(torch.einsum("trk,kd->trd", probs, v[start:start + n, g]),
                                                        (0, 0, g * ratio, hq - (g + 1) * ratio)))
        start += n
    return out


def test_small_module_parameter_gradients(cuda_device):
    torch.manual_seed(54)
    total, hidden, groups, ratio, dim = 8, 12, 2, 2, 4
    base = [torch.randn(total, hidden), torch.randn(hidden, groups * ratio * dim) * 0.2,
            torch.randn(hidden, groups * dim) * 0.2, torch.randn(hidden, groups * dim) * 0.2,
            torch.randn(groups * ratio * dim, hidden) * 0.2]
    lengths = [5, 3]
    cu = cu_of(lengths, cuda_device)
    wiq = torch.randn(hidden, groups * dim, device=cuda_device, requires_grad=True)
    wik = torch.randn(hidden, dim, device=cuda_device, requires_grad=True)
    x, wq, wk, wv, wo = [a.to(cuda_device).clone().requires_grad_() for a in base]
    with torch.no_grad():
        iq = (x @ wiq).reshape(total, groups, dim)
        ik = (x @ wik).reshape(total, 1, dim)
        ids = m3_topk(m3_index_score(iq, ik, cu, 5, block_size=2), cu, block_size=2, topk_blocks=2)
    q = (x @ wq).reshape(total, groups * ratio, dim)
    k, v = [(x @ w).reshape(total, groups, dim) for w in (wk, wv)]
    out = m3_sparse_attention(q, k, v, ids, cu, 5, block_size=2)
    (out.reshape(total, -1) @ wo).square().mean().backward()
    rx, rq, rk, rv, ro = [a.double().requires_grad_() for a in base]
    qq = (rx @ rq).reshape(total, groups * ratio, dim)
    kk, vv = [(rx @ w).reshape(total, groups, dim) for w in (rk, rv)]
    ref = _dense_reference_attention(qq, kk, vv, ids, lengths, 2)
    (ref.reshape(total, -1) @ ro).square().mean().backward()
    for mine, r in zip((x, wq, wk, wv, wo), (rx, rq, rk, rv, ro)):
        torch.testing.assert_close(mine.grad.cpu().double(), r.grad, atol=1e-4, rtol=1e-4)
    assert wiq.grad is None and wik.grad is None
