"""Decode over a paged KV cache on the GPU: each request's newest token against
its cached keys, pages scattered through a block table, compared with the float64
oracle on the request's contiguous sequence (the prefill semantics at the last
position) and with this library's prefill operators on the same data.

Tolerance: the decode kernels compute in float32 from the exact inputs, so the
bf16/f16 outputs are within one rounding step of the float64 values (rtol 2^-7,
atol 1e-3 of the largest value); LSE and scores within 1e-4 (scores: the
float32 accumulation bound of the index score tests); top-k bit-exact on the
same scores."""

import numpy as np
import pytest
import torch

from msa_triton_b200 import m3_index_score_decode, m3_sparse_attention, m3_sparse_decode, m3_topk_decode
from oracle import msa_oracle as O

pytestmark = pytest.mark.gpu


def unit_rms(x):
    return x / x.square().mean(-1, keepdim=True).sqrt()


def paged(seq_lists, page_size, gen):
    """Scatter each list of per-request [L, H, D] tensors into its own page pool, all with one
    random page order (a few pages stay unused); returns the pools and the block table."""
    lens = [s.shape[0] for s in seq_lists[0]]
    pages_per = [(n + page_size - 1) // page_size for n in lens]
    total_pages = sum(pages_per) + 3
    perm = torch.randperm(total_pages, generator=gen)
    table = torch.zeros(len(lens), max(pages_per), dtype=torch.int32)
    pools = [torch.zeros(total_pages, page_size, *seqs[0].shape[1:], dtype=seqs[0].dtype) for seqs in seq_lists]
    nxt = 0
    for b, n in enumerate(lens):
        for i in range(pages_per[b]):
            p = int(perm[nxt])
            nxt += 1
            table[b, i] = p
            for pool, seqs in zip(pools, seq_lists):
                chunk = seqs[b][i * page_size:(i + 1) * page_size]
                pool[p, :chunk.shape[0]] = chunk
    return pools, table


@pytest.mark.parametrize("lens,groups,ratio,dim,idim,block,page,topk,dtype", [
    ([1, 130, 700, 2049, 300], 2, 8, 128, 64, 128, 128, 4, torch.bfloat16),
    ([5, 64, 333], 2, 4, 128, 64, 128, 16, 6, torch.bfloat16),
    ([3, 40, 17], 3, 3, 24, 8, 16, 4, 3, torch.float32),
])
def test_decode_matches_fp64_and_prefill(lens, groups, ratio, dim, idim, block, page, topk, dtype, cuda_device):
    gen = torch.Generator().manual_seed(sum(lens))
    hq = groups * ratio
    ks = [unit_rms(torch.randn(n, groups, dim, generator=gen)).to(dtype) for n in lens]
    vs = [unit_rms(torch.randn(n, groups, dim, generator=gen)).to(dtype) for n in lens]
    iks = [unit_rms(torch.randn(n, 1, idim, generator=gen)).to(dtype) for n in lens]
    q = unit_rms(torch.randn(len(lens), hq, dim, generator=gen)).to(dtype)
    iq = unit_rms(torch.randn(len(lens), groups, idim, generator=gen)).to(dtype)
    (k_cache, v_cache, ik_cache), table = paged([ks, vs, iks], page, gen)
    seq_lens = torch.tensor(lens, dtype=torch.int32)
    max_seqlen = max(lens)
    dev = cuda_device

    scores = m3_index_score_decode(iq.to(dev), ik_cache.to(dev), table.to(dev), seq_lens.to(dev), max_seqlen,
                                   block_size=block)
    ids = m3_topk_decode(scores, seq_lens.to(dev), block_size=block, topk_blocks=topk, local_blocks=1)
    out, lse = m3_sparse_decode(q.to(dev), k_cache.to(dev), v_cache.to(dev), table.to(dev), seq_lens.to(dev), ids,
                                block_size=block, return_lse=True)
    got_scores, got_ids = scores.cpu().double().numpy(), ids.cpu().numpy()
    expected_ids = O.topk_at_positions(scores.cpu().numpy(), np.array(lens) - 1, block_size=block, topk_blocks=topk,
                                       local_blocks=1)
    np.testing.assert_array_equal(got_ids, expected_ids)
    for b, n in enumerate(lens):
        cu = np.array([0, n], dtype=np.int32)
        iq_full = np.zeros((n, groups, idim))
        iq_full[n - 1] = iq[b].double().numpy()
        ref_s = O.index_score_rows(iq_full, iks[b].double().numpy(), cu, max_seqlen, [n - 1], block_size=block)[0]
        assert np.array_equal(np.isneginf(got_scores[b]), np.isneginf(ref_s))
        fin = np.isfinite(ref_s)
        np.testing.assert_allclose(got_scores[b][fin], ref_s[fin], rtol=1e-5, atol=1e-4)
        q_full = np.zeros((n, hq, dim))
        q_full[n - 1] = q[b].double().numpy()
        ids_full = np.full((n, groups, topk), -1, dtype=np.int32)
        ids_full[n - 1] = got_ids[b]
        ref = O.sparse_attention_sampled(q_full, ks[b].double().numpy(), vs[b].double().numpy(), ids_full, cu,
                                         block_size=block, query_tokens=[n - 1])
        a = out[b].cpu().double().numpy()
        scale = float(np.abs(ref["out"][0]).max()) or 1.0
        np.testing.assert_allclose(a, ref["out"][0], rtol=2 ** -7, atol=1e-3 * scale)
        np.testing.assert_allclose(lse[b].cpu().numpy(), ref["lse"][0], rtol=1e-5, atol=1e-4)
        # this library's prefill path on the contiguous sequence, last row
        qp = torch.zeros(n, hq, dim, dtype=dtype)
        qp[n - 1] = q[b]
        pre = m3_sparse_attention(qp.to(dev), ks[b].to(dev), vs[b].to(dev), torch.from_numpy(ids_full).to(dev),
                                  torch.tensor(cu).to(dev), n, block_size=block)
        torch.testing.assert_close(out[b], pre[n - 1], rtol=2 ** -7, atol=2e-2 * scale)


def test_decode_repeated_and_empty_selections(cuda_device):
    gen = torch.Generator().manual_seed(3)
    lens, groups, ratio, dim, block, page, topk = [300, 129], 2, 8, 128, 128, 64, 4
    ks = [unit_rms(torch.randn(n, groups, dim, generator=gen)).bfloat16() for n in lens]
    (k_cache,), table = paged([ks], page, gen)
    q = unit_rms(torch.randn(2, groups * ratio, dim, generator=gen)).bfloat16()
    seq_lens = torch.tensor(lens, dtype=torch.int32)
    ids = torch.tensor([[[2, 2, 0, -1], [5, -1, -1, -1]], [[1, 0, 1, 3], [-1, -1, -1, -1]]], dtype=torch.int32)
    dev = cuda_device
    out, lse = m3_sparse_decode(q.to(dev), k_cache.to(dev), k_cache.to(dev), table.to(dev), seq_lens.to(dev),
                                ids.to(dev), block_size=block, return_lse=True)
    # request 0 group 1 selects only a future block; request 1 group 1 nothing: zero output, -inf lse
    assert torch.count_nonzero(out[0, 8:]) == 0 and torch.isneginf(lse[0, 8:]).all()
    assert torch.count_nonzero(out[1, 8:]) == 0 and torch.isneginf(lse[1, 8:]).all()
    for b, n in enumerate(lens):
        cu = np.array([0, n], dtype=np.int32)
        q_full = np.zeros((n, groups * ratio, dim))
        q_full[n - 1] = q[b].double().numpy()
        ids_full = np.full((n, groups, topk), -1, dtype=np.int32)
        ids_full[n - 1] = ids[b].numpy()
        ref = O.sparse_attention_sampled(q_full, ks[b].double().numpy(), ks[b].double().numpy(), ids_full, cu,
                                         block_size=block, query_tokens=[n - 1])
        np.testing.assert_allclose(out[b].cpu().double().numpy(), ref["out"][0], rtol=2 ** -7, atol=1e-3)
