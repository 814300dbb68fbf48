"""The oracle's sampled helpers (used by the at-scale GPU tests, where the full
restatement would not finish) agree with the full float64 restatement on small
cases: packed sequences with an empty one, exact ties, partial last blocks,
duplicated and invalid selections."""

import numpy as np
import pytest

from oracle import msa_oracle as O

LENGTHS = [300, 0, 517]
CU = np.array([0, 300, 300, 817], dtype=np.int32)
TOKENS = [0, 5, 7, 127, 128, 299, 300, 301, 700, 816]


def _bf16_grid(rng, shape):
    """float64 values on the bf16 grid (what the library's inputs hold)."""
    x = rng.standard_normal(shape).astype(np.float32)
    return (x.view(np.uint32) & np.uint32(0xFFFF0000)).view(np.float32).astype(np.float64)


def _selection(rng, total, groups, topk, cu):
    _, start, pos = O.token_positions(cu)
    ids = np.full((total, groups, topk), -1, dtype=np.int32)
    for t in range(total):
        cur = int(pos[t]) // 128
        for g in range(groups):
            picks = rng.integers(-1, cur + 2, size=topk)  # -1, valid, future
            picks[0] = cur
            if topk > 2:
                picks[2] = picks[1]  # a duplicate
            ids[t, g] = picks
    return ids


@pytest.mark.parametrize("scale", [1.0, -0.5])
def test_index_score_rows_and_backward_sampled(scale):
    rng = np.random.default_rng(11)
    total, groups, dim = sum(LENGTHS), 3, 16
    iq = _bf16_grid(rng, (total, groups, dim))
    ik = _bf16_grid(rng, (total, 1, dim))
    ik[7] = ik[5]  # an exact tie inside block 0 of the first sequence
    nb = (max(LENGTHS) + 127) // 128
    ds = rng.standard_normal((total, groups, nb))
    full = O.index_score(iq, ik, CU, max(LENGTHS), block_size=128, scale=scale)
    rows = O.index_score_rows(iq, ik, CU, max(LENGTHS), TOKENS, block_size=128, scale=scale)
    np.testing.assert_array_equal(rows, full[TOKENS])
    dq, dk = O.index_score_backward(iq, ik, CU, max(LENGTHS), ds, block_size=128, scale=scale)
    blocks = [(0, 0), (0, 2), (2, 0), (2, 3), (2, 4), (1, 0)]
    sdq, sdk = O.index_score_backward_sampled(iq, ik, CU, ds, tokens=TOKENS, key_blocks=blocks, block_size=128,
                                              scale=scale, chunk=100)
    np.testing.assert_allclose(sdq, dq[TOKENS], rtol=1e-12, atol=1e-12)
    bounds = CU.tolist()
    for r, (s, b) in enumerate(blocks):
        k0 = bounds[s] + b * 128
        n = max(0, min(128, bounds[s + 1] - k0))
        np.testing.assert_allclose(sdk[r, :n], dk[k0:k0 + n, 0], rtol=1e-12, atol=1e-12)
        assert not sdk[r, n:].any()


def test_sparse_attention_sampled_matches_full():
    rng = np.random.default_rng(12)
    total, hq, groups, dim, topk = sum(LENGTHS), 4, 2, 8, 4
    q = _bf16_grid(rng, (total, hq, dim))
    k = _bf16_grid(rng, (total, groups, dim))
    v = _bf16_grid(rng, (total, groups, dim))
    dout = _bf16_grid(rng, (total, hq, dim))
    ids = _selection(rng, total, groups, topk, CU)
    out, lse = O.sparse_attention(q, k, v, ids, CU, block_size=128)
    dq, dk, dv = O.sparse_attention_backward(q, k, v, ids, CU, dout, block_size=128)
    key_rows = [(0, 0, 0), (0, 2, 1), (2, 1, 0), (2, 4, 1)]
    ref = O.sparse_attention_sampled(q, k, v, ids, CU, dout, block_size=128, query_tokens=TOKENS,
                                     key_rows=key_rows)
    np.testing.assert_allclose(ref["out"], out[TOKENS], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(ref["lse"], lse[TOKENS], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(ref["dq"], dq[TOKENS], rtol=1e-12, atol=1e-12)
    bounds = CU.tolist()
    for r, (s, b, g) in enumerate(key_rows):
        k0 = bounds[s] + b * 128
        n = min(128, bounds[s + 1] - k0)
        np.testing.assert_allclose(ref["dk"][r, :n], dk[k0:k0 + n, g], rtol=1e-11, atol=1e-12)
        np.testing.assert_allclose(ref["dv"][r, :n], dv[k0:k0 + n, g], rtol=1e-11, atol=1e-12)


def test_index_kl_pairs_matches_full():
    rng = np.random.default_rng(13)
    total, hq, groups, dim, idim, topk = sum(LENGTHS), 4, 2, 8, 8, 4
    q = _bf16_grid(rng, (total, hq, dim))
    k = _bf16_grid(rng, (total, groups, dim))
    iq = _bf16_grid(rng, (total, groups, idim))
    ik = _bf16_grid(rng, (total, 1, idim))
    ids = _selection(rng, total, groups, topk, CU)
    loss, diq, dik = O.index_kl_loss(iq, ik, q, k, ids, CU, block_size=128, index_scale=0.7)
    pairs = [(t, g) for t in range(total) for g in range(groups)]
    kls, rows, kb = O.index_kl_pairs(iq, ik, q, k, ids, CU, pairs, block_size=128, index_scale=0.7,
                                     key_block=(300 + 128, 128))
    np.testing.assert_allclose(kls.sum() / (total * groups), loss, rtol=1e-12)
    np.testing.assert_allclose(rows.reshape(total, groups, idim), diq, rtol=1e-10, atol=1e-14)
    np.testing.assert_allclose(kb, dik[428:556, 0], rtol=1e-10, atol=1e-14)
