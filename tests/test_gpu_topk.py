"""Top-k parity on the GPU (restates the reference's test_topk.py): an
independent ranking oracle, the golden outputs of the reference's two top-k
implementations (equivalent up to tie choice; bit-exact in canonical order when
no ties), and the float64 oracle bit-exactly at benchmark-like sizes."""

import numpy as np
import pytest
import torch

from msa_triton_b200 import m3_topk
from oracle import msa_oracle as O
from tests.helpers import cu_of

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("lengths,block,k,local", [
    ([1, 7, 3], 2, 3, 1), ([127, 128, 129], 128, 16, 1), ([17, 0, 9], 4, 2, 0), ([8, 5], 2, 3, 3), ([2], 1, 0, 0),
])
def test_topk_matches_independent_ranking(lengths, block, k, local, cuda_device):
    cu = cu_of(lengths, cuda_device)
    groups, blocks = 3, (max(lengths) + block - 1) // block
    scores_cpu = torch.randn(sum(lengths), groups, blocks, generator=torch.Generator().manual_seed(82))
    scores = scores_cpu.to(cuda_device)
    saved = scores.clone()
    selected = m3_topk(scores, cu, block_size=block, topk_blocks=k, local_blocks=local)
    assert selected.dtype == torch.int32 and selected.shape == (sum(lengths), groups, k)
    torch.testing.assert_close(scores, saved, atol=0, rtol=0)
    selected = selected.cpu()
    start = 0
    for length in lengths:
        for position in range(length):
            current = position // block
            forced = set(range(max(0, current - local + 1), current + 1)) if local else set()
            for group in range(groups):
                candidates = [b for b in range(current + 1) if b not in forced]
                candidates.sort(key=lambda b: -float(scores_cpu[start + position, group, b]))
                expected = forced | set(candidates[:k - len(forced)])
                actual = selected[start + position, group].tolist()
                kept = [b for b in actual if b != -1]
                assert len(kept) == len(set(kept))
                assert set(kept) == expected
                assert actual == kept + [-1] * (k - len(kept))
        start += length


def test_equal_scores_local_and_no_gradient(cuda_device):
    scores = torch.zeros(7, 2, 4, requires_grad=True, device=cuda_device)
    out = m3_topk(scores, cu_of([7], cuda_device), block_size=2, topk_blocks=2, local_blocks=1)
    assert not out.requires_grad
    out = out.cpu()
    for token in range(7):
        for group in range(2):
            valid = out[token, group][out[token, group] >= 0].tolist()
            assert token // 2 in valid
            assert len(valid) == min(2, token // 2 + 1)
            assert len(set(valid)) == len(valid)
            assert all(0 <= b <= token // 2 for b in valid)


def test_topk_golden_vectors_from_reference(golden, cuda_device):
    g = golden.stage("topk")
    for c in golden.cases("topk"):
        n = c["name"]
        kw = dict(block_size=c["block_size"], topk_blocks=c["topk_blocks"], local_blocks=c["local_blocks"])
        scores = torch.from_numpy(g[f"{n}/scores"])
        cu = torch.from_numpy(g[f"{n}/cu"])
        mine = m3_topk(scores.to(cuda_device), cu.to(cuda_device), **kw).cpu().numpy()
        np.testing.assert_array_equal(mine, O.topk(scores.numpy(), cu.numpy(), **kw), err_msg=n)
        for impl in ("eager", "native"):
            assert O.topk_equivalent(mine, g[f"{n}/{impl}"], scores.numpy(), cu.numpy(), block_size=c["block_size"],
                                     local_blocks=c["local_blocks"]), f"{n}/{impl}"


@pytest.mark.parametrize("lengths,groups,block,k,local", [
    ([8192], 8, 128, 16, 1), ([3000, 5000, 700], 4, 64, 32, 2), ([131072 // 8], 2, 16, 32, 2),
])
def test_topk_bit_exact_against_oracle_at_size(lengths, groups, block, k, local, cuda_device):
    nb = (max(lengths) + block - 1) // block
    scores = torch.randn(sum(lengths), groups, nb, generator=torch.Generator().manual_seed(3))
    cu = cu_of(lengths)
    mine = m3_topk(scores.to(cuda_device), cu.to(cuda_device), block_size=block, topk_blocks=k, local_blocks=local)
    np.testing.assert_array_equal(mine.cpu().numpy(),
                                  O.topk(scores.numpy(), cu.numpy(), block_size=block, topk_blocks=k,
                                         local_blocks=local))


@pytest.mark.parametrize("k,local", [(7, 2), (16, 2), (32, 2), (48, 2), (49, 2), (64, 2), (16, 12), (16, 16), (40, 40)])
@pytest.mark.parametrize("values", ["randn_inf", "rounded", "three_levels", "wide", "signed_zero"])
def test_topk_threshold_and_round_paths(k, local, values, cuda_device):
    """Each K class (up to 16, up to 48, above 48) on rows of up to 2048 blocks.
    Rounded and three-level scores put long runs of equal values at the K-th
    rank, which the threshold search cannot split: those rows take the round
    path, and both paths must agree with the oracle bit for bit. With
    ``local`` close to or equal to K the answer lies among the forced keys.
    Scores over 60 decades ("wide") give candidates whose rank words span more
    than a 32-bit sort key can hold next to the block id (the 64-bit sort);
    "signed_zero" mixes -0.0 and +0.0, which rank equal."""
    lengths, groups, block = [4096, 2000, 137], 2, 2
    nb = (max(lengths) + block - 1) // block
    gen = torch.Generator().manual_seed(11 + k)
    scores = torch.randn(sum(lengths), groups, nb, generator=gen)
    if values == "randn_inf":
        u = torch.rand(scores.shape, generator=gen)
        scores[u < 0.02] = float("-inf")
        scores[u > 0.99] = float("inf")
    elif values == "rounded":
        scores = (scores * 2).round()
    elif values == "wide":
        scores = scores * torch.pow(10.0, torch.randint(-30, 31, scores.shape, generator=gen).float())
    elif values == "signed_zero":
        u = torch.rand(scores.shape, generator=gen)
        scores[u < 0.3] = 0.0
        scores[u > 0.7] = -0.0
    else:
        scores = torch.randint(0, 3, scores.shape, generator=gen).float()
    cu = cu_of(lengths)
    mine = m3_topk(scores.to(cuda_device), cu.to(cuda_device), block_size=block, topk_blocks=k, local_blocks=local)
    np.testing.assert_array_equal(mine.cpu().numpy(),
                                  O.topk(scores.numpy(), cu.numpy(), block_size=block, topk_blocks=k,
                                         local_blocks=local))
