"""Shared helpers for the parity tests (inputs, conversions, tolerances)."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

GATE = dict(atol=1e-4, rtol=1e-4)  # the reference suite's gate vs float64 (test_triton_attention.py:91)

# native bf16 eager error vs float64 on configuration 1, measured by running the reference
EAGER = json.loads((Path(__file__).parent / "golden" / "manifest.json").read_text())["eager_error_cfg1"]


def _err(actual, expected):
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    fin = np.isfinite(e)
    assert np.array_equal(np.isneginf(a), np.isneginf(e)) and not np.isnan(a).any()
    d = np.abs(a[fin] - e[fin])
    return float(d.max()), float(np.linalg.norm(d) / max(np.linalg.norm(e[fin]), 1e-30))


def eager_gate(name, actual, expected, eager):
    """The tensor-core path's stated tolerance on any inputs: max-abs and relative Frobenius
    error against float64 no worse than twice the reference's native bf16 eager numerics on
    the same inputs (oracle.sparse_attention_eager)."""
    a_mx, a_rf = _err(actual, expected)
    e_mx, e_rf = _err(eager, expected)
    assert a_mx <= 2 * e_mx, f"{name}: max_abs {a_mx} > 2x eager {e_mx}"
    assert a_rf <= 2 * e_rf, f"{name}: rel_fro {a_rf} > 2x eager {e_rf}"
    return a_mx, e_mx


def scaled_check(name, actual, expected):
    """The tensor-core path's gate at any size or input scale: relative Frobenius error at
    most twice the eager one, and max-abs error at most twice eager's relative to the RMS of
    the values compared (``max_abs / ref_rms`` of the eager measurement); ``lse`` keeps the
    absolute bound. -inf pattern exact, no NaN."""
    a = np.asarray(actual, dtype=np.float64)
    e = np.asarray(expected, dtype=np.float64)
    assert a.shape == e.shape, name
    fin = np.isfinite(e)
    assert np.array_equal(np.isneginf(a), np.isneginf(e)), f"{name}: -inf pattern differs"
    assert not np.isnan(a).any(), f"{name}: NaN"
    d = np.abs(a[fin] - e[fin])
    rel_fro = float(np.linalg.norm(d) / max(np.linalg.norm(e[fin]), 1e-30))
    ref = EAGER[name]
    assert rel_fro <= 2 * ref["rel_fro"], f"{name}: rel_fro {rel_fro} > 2x eager {ref['rel_fro']}"
    if name == "lse":
        limit = 2 * ref["max_abs"]
    else:
        limit = 2 * ref["max_abs"] / ref["ref_rms"] * float(np.sqrt(np.mean(e[fin] ** 2)))
    assert float(d.max()) <= limit, f"{name}: max_abs {float(d.max())} > {limit}"
    return float(d.max()), rel_fro


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
