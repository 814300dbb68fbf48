"""``prepared=prepare_batch(cu_seqlens)``: the three ops and the k2q build give
the same results as without it and read nothing from the device (the host
copy of the boundaries is taken from the prepared batch)."""

import pytest
import torch

from msa_triton_b200 import _lib, m3_index_score, m3_sparse_attention, m3_topk, prepare_batch
from msa_triton_b200.k2q import build_k2q_csr
from msa_triton_b200.workloads import random_selection
from tests.helpers import cu_of

pytestmark = pytest.mark.gpu


def test_prepared_batch_matches_and_reads_nothing(cuda_device, monkeypatch):
    lengths = [700, 300, 129]
    total, groups, ratio, dim, block, topk = sum(lengths), 2, 8, 128, 128, 3
    gen = torch.Generator().manual_seed(21)
    dev = lambda x: x.to(cuda_device)
    cu = cu_of(lengths, cuda_device)
    iq = dev(torch.randn(total, groups, 64, generator=gen).bfloat16())
    ik = dev(torch.randn(total, 1, 64, generator=gen).bfloat16())
    q, k, v, go = (dev(torch.randn(total, h, dim, generator=gen).bfloat16()) for h in (groups * ratio, groups, groups,
                                                                                      groups * ratio))
    ids = dev(random_selection(lengths, groups, block, topk, seed=4))

    def run(prepared):
        s = m3_index_score(iq, ik, cu, max(lengths), prepared=prepared)
        sel = m3_topk(s, cu, topk_blocks=topk, prepared=prepared)
        csr = build_k2q_csr(ids, cu, block_size=block, prepared=prepared)
        qq, kk, vv = (x.clone().requires_grad_() for x in (q, k, v))
        out = m3_sparse_attention(qq, kk, vv, ids, cu, max(lengths), prepared=prepared)
        out.backward(go)
        torch.cuda.synchronize()
        return [s, sel, csr.row_ptr, csr.query_indices, csr.slot_indices, csr.cu_block_lens, qq.grad, kk.grad, vv.grad]

    want = run(None)
    prepared = prepare_batch(cu)

    def no_read(_t):
        raise AssertionError("device read with a prepared batch")

    monkeypatch.setattr(_lib, "host_ints", no_read)
    got = run(prepared)
    assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])
    for a, b in zip(got[2:6], want[2:6]):
        assert torch.equal(a, b)
    for a, b in zip(got[6:], want[6:]):  # dQ sums in a different order run to run
        torch.testing.assert_close(a, b, atol=2e-2, rtol=2e-2)
