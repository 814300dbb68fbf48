"""The index KL loss oracle (oracle/msa_oracle.py:index_kl_loss) against an
independent dense autograd computation of the same definition
(docs/msa_training_flow.md:92-138 of the reference: KL(teacher || student) on
the selected causal tokens, teacher = group mean of the main attention's
per-head softmax, mean over (token, group) pairs). The reference has no
implementation to pin against, so the hand-derived gradients are checked
against torch autograd here."""

import numpy as np
import pytest
import torch

from msa_triton_b200.workloads import random_selection
from oracle import msa_oracle as O


def dense_kl(iq, ik, q, k, ids, cu, block, index_scale, scale):
    total, groups = q.shape[0], k.shape[1]
    ratio = q.shape[1] // groups
    bounds = [int(x) for x in cu]
    loss = torch.zeros((), dtype=torch.float64)
    for a, b in zip(bounds[:-1], bounds[1:]):
        n = b - a
        if n == 0:
            continue
        pos = torch.arange(n)
        for g in range(groups):
            sel = ((pos[None, :] // block)[:, :, None] == ids[a:b, g][:, None, :].long()).any(-1)
            sel &= pos[None, :] <= pos[:, None]
            has = sel.any(-1)
            tl = torch.einsum("trd,kd->trk", q[a:b, g * ratio:(g + 1) * ratio], k[a:b, g]) * scale
            tl = tl.masked_fill(~sel[:, None, :], -float("inf"))
            tp = torch.softmax(torch.where(has[:, None, None], tl, torch.zeros_like(tl)), -1).mean(1)
            s = (iq[a:b, g] @ ik[a:b, 0].T) * index_scale
            s = s.masked_fill(~sel, -float("inf"))
            logps = torch.log_softmax(torch.where(has[:, None], s, torch.zeros_like(s)), -1)
            term = torch.where(sel & (tp > 0), tp * (torch.log(tp.clamp_min(1e-300)) - logps), torch.zeros_like(tp))
            loss = loss + term[has].sum()
    return loss / (total * groups)


@pytest.mark.parametrize("lengths,groups,ratio,dim,index_dim,block,topk,index_scale,scale", [
    ([37, 0, 90], 2, 3, 8, 5, 8, 4, 0.7, 0.3),
    ([1, 16, 5], 1, 4, 4, 3, 4, 2, 1.0, None),
    ([64], 4, 1, 16, 8, 16, 3, -0.5, 0.25),
])
def test_kl_oracle_matches_autograd(lengths, groups, ratio, dim, index_dim, block, topk, index_scale, scale):
    gen = torch.Generator().manual_seed(sum(lengths) + groups)
    total = sum(lengths)
    iq = torch.randn(total, groups, index_dim, generator=gen, dtype=torch.float64, requires_grad=True)
    ik = torch.randn(total, 1, index_dim, generator=gen, dtype=torch.float64, requires_grad=True)
    q = torch.randn(total, groups * ratio, dim, generator=gen, dtype=torch.float64)
    k = torch.randn(total, groups, dim, generator=gen, dtype=torch.float64)
    ids = random_selection(lengths, groups, block, topk, seed=5)
    ids[0] = -1  # a pair with no key contributes 0
    if total > 10:
        ids[10, 0, 1] = ids[10, 0, 0]  # a duplicated id selects its block once
    cu = np.cumsum([0] + lengths).astype(np.int32)
    loss, diq, dik = O.index_kl_loss(iq.detach().numpy(), ik.detach().numpy(), q.numpy(), k.numpy(), ids.numpy(), cu,
                                     block_size=block, index_scale=index_scale, scale=scale)
    ref = dense_kl(iq, ik, q, k, ids, cu, block, index_scale, dim ** -0.5 if scale is None else scale)
    ref.backward()
    assert abs(loss - float(ref.detach())) < 1e-12
    np.testing.assert_allclose(diq, iq.grad.numpy(), atol=1e-13)
    np.testing.assert_allclose(dik, ik.grad.numpy(), atol=1e-13)
    assert loss >= 0.0
