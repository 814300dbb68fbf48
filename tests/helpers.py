"""Shared helpers for the parity tests (inputs, conversions, tolerances)."""

from __future__ import annotations

import numpy as np
import torch

GATE = dict(atol=1e-4, rtol=1e-4)  # the reference suite's gate vs float64 (test_triton_attention.py:91)


def cu_of(lengths, device=None):
    bounds = [0]
    for n in lengths:
        bounds.append(bounds[-1] + n)
    return torch.tensor(bounds, dtype=torch.int32, device=device)


def np64(t):
    return t.detach().cpu().double().numpy()


def reference_selection(lengths, groups, block_size, topk):
    """The distinct, causal selection pattern used by the reference's attention tests."""
    total = sum(lengths)
    ids = torch.full((total, groups, topk), -1, dtype=torch.int32)
    start = 0
    for length in lengths:
        for offset in range(length):
            for g in range(groups):
                cur = offset // block_size
                cand = [cur] + [b for b in range(cur) if (b + g) % 2 == 0]
                chosen = cand[:topk]
                if chosen:
                    ids[start + offset, g, :len(chosen)] = torch.tensor(chosen, dtype=torch.int32)
        start += length
    return ids


def attention_inputs(lengths, groups, ratio, dim, block_size, topk, device, dtype=torch.bfloat16, seed=1234):
    gen = torch.Generator().manual_seed(seed)
    total = sum(lengths)
    q = torch.randn(total, groups * ratio, dim, generator=gen).to(dtype)
    k = torch.randn(total, groups, dim, generator=gen).to(dtype)
    v = torch.randn(total, groups, dim, generator=gen).to(dtype)
    ids = reference_selection(lengths, groups, block_size, topk)
    tensors = tuple(x.to(device).requires_grad_() for x in (q, k, v))
    return tensors, ids.to(device), cu_of(lengths, device)


def assert_close_with_neginf(actual, expected, **tol):
    actual = actual.detach().cpu()
    expected = expected.detach().cpu().to(actual.dtype)
    assert torch.equal(torch.isneginf(actual), torch.isneginf(expected))
    assert not torch.isnan(actual).any()
    fin = torch.isfinite(expected)
    torch.testing.assert_close(actual[fin], expected[fin], **(tol or GATE))


from msa_triton_b200.workloads import random_selection as random_distinct_selection  # noqa: E402,F401
