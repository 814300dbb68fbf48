"""CPU oracle for the MiniMax-M3 three-stage sparse attention path.

TEST INFRASTRUCTURE ONLY. This module is the checker that the CUDA library is
compared against; it is never the thing measured or shipped. Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs
of ``bench.py`` may import it. The product path (``msa_triton_b200``) never
imports it and fails loudly when its CUDA library is missing.

It is a float64 numpy restatement of the reference algorithm
(yeyeyeping/msa_triton); each function cites the reference file:line it
follows. Parity of this restatement is pinned against golden vectors generated
by running the reference itself (``tests/golden/make_golden.py``) and checked
by ``tests/test_oracle_golden.py``.

Conventions (identical to the reference):
* TND layout: ``q[T, Hq, D]``, ``k/v[T, G, D]``, ``index_q[T, G, Di]``,
  ``index_k[T, 1, Di]``; packed sequences delimited by int32 ``cu_seqlens``.
* Blocks are numbered from the start of each packed sequence.
* Query heads ``g*(Hq/G) .. (g+1)*(Hq/G)-1`` share group ``g``'s selection.
"""

from __future__ import annotations

import math

import numpy as np


# ---------------------------------------------------------------------------
# metadata
# ---------------------------------------------------------------------------

def sequence_lengths(cu_seqlens, total_tokens: int) -> list[int]:
    """Validate packed boundaries; layout.py:18-30 (same messages)."""
    cu = np.asarray(cu_seqlens)
    if cu.ndim != 1 or cu.size < 2:
        raise ValueError("cu_seqlens must be a vector with at least two entries")
    bounds = [int(x) for x in cu.tolist()]
    if bounds[0] != 0 or bounds[-1] != total_tokens:
        raise ValueError("cu_seqlens must start at zero and end at total_tokens")
    lengths = [b - a for a, b in zip(bounds[:-1], bounds[1:])]
    if min(lengths) < 0:
        raise ValueError("cu_seqlens must be nondecreasing")
    return lengths


def token_positions(cu_seqlens):
    """Per packed token: (sequence id, sequence start, position in sequence)."""
    bounds = [int(x) for x in np.asarray(cu_seqlens).tolist()]
    total = bounds[-1]
    seq = np.zeros(total, dtype=np.int64)
    start = np.zeros(total, dtype=np.int64)
    for s, (a, b) in enumerate(zip(bounds[:-1], bounds[1:])):
        seq[a:b] = s
        start[a:b] = a
    pos = np.arange(total, dtype=np.int64) - start
    return seq, start, pos


# ---------------------------------------------------------------------------
# stage 1: index score (block max of causal index logits)
# ---------------------------------------------------------------------------

def index_score(index_q, index_k, cu_seqlens, max_seqlen, *, block_size=128, scale=1.0):
    """float64 ``S[t,g,b] = max_{j in block b, j<=t} scale * iq[t,g].ik[j]``.

    Follows tests/reference_fp64.py:16-45 (per-sequence, per-block causal max;
    future and out-of-sequence blocks are -inf) with the output width
    ``ceil(max_seqlen / block_size)`` of triton/index_score.py:243.
    """
    q = np.asarray(index_q, dtype=np.float64)
    k = np.asarray(index_k, dtype=np.float64)[:, 0, :]
    total, groups, _ = q.shape
    nb = (max_seqlen + block_size - 1) // block_size
    out = np.full((total, groups, nb), -np.inf, dtype=np.float64)
    bounds = [int(x) for x in np.asarray(cu_seqlens).tolist()]
    for a, b in zip(bounds[:-1], bounds[1:]):
        length = b - a
        if length == 0:
            continue
        # [L, G, L] logits of this sequence, chunked over queries.
        for q0 in range(0, length, 1024):
            q1 = min(length, q0 + 1024)
            logits = np.einsum("tgd,kd->tgk", q[a + q0:a + q1], k[a:b]) * scale
            pos = np.arange(q0, q1)[:, None]
            keys = np.arange(length)[None, :]
            logits = np.where((keys <= pos)[:, None, :], logits, -np.inf)
            for blk in range(nb):
                lo, hi = blk * block_size, min((blk + 1) * block_size, length)
                if lo >= hi:
                    continue
                out[a + q0:a + q1, :, blk] = logits[:, :, lo:hi].max(axis=-1)
    return out


def index_score_backward(index_q, index_k, cu_seqlens, max_seqlen, dscores, *,
                         block_size=128, scale=1.0):
    """Gradients of :func:`index_score` w.r.t. index_q and index_k (float64).

    torch.amax semantics, as required by triton/index_score.py:307-316 and
    implemented by its backward kernels (:139-232): the gradient of a block
    maximum is split equally among the keys attaining it; masked (future,
    out-of-sequence) positions receive nothing.
    """
    q = np.asarray(index_q, dtype=np.float64)
    k = np.asarray(index_k, dtype=np.float64)[:, 0, :]
    ds = np.asarray(dscores, dtype=np.float64)
    total, groups, _ = q.shape
    nb = (max_seqlen + block_size - 1) // block_size
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    bounds = [int(x) for x in np.asarray(cu_seqlens).tolist()]
    for a, b in zip(bounds[:-1], bounds[1:]):
        length = b - a
        for p in range(length):
            t = a + p
            for blk in range(nb):
                lo = blk * block_size
                hi = min(lo + block_size, length, p + 1)
                if lo >= hi:
                    continue
                logits = k[a + lo:a + hi] @ q[t].T * scale  # [n, G]
                best = logits.max(axis=0)
                for g in range(groups):
                    winners = np.nonzero(logits[:, g] == best[g])[0]
                    w = ds[t, g, blk] * scale / len(winners)
                    dq[t, g] += w * k[a + lo + winners].sum(axis=0)
                    dk[a + lo + winners] += w * q[t, g]
    return dq, dk[:, None, :]


# ---------------------------------------------------------------------------
# stage 2: top-k block selection
# ---------------------------------------------------------------------------

def topk(scores, cu_seqlens, *, block_size=128, topk_blocks=16, local_blocks=1):
    """int32 ``[T, G, K]`` block ids; triton/topk.py:11-47, eager/ops.py:94-129.

    Future blocks are masked to -inf; the ``local_blocks`` most recent causal
    blocks are forced to +inf; the top ``min(K, NB)`` by descending value are
    kept; -inf picks become -1 and the tail is padded with -1. The reference's
    order inside a run of equal values is whatever torch.topk returns; this
    oracle fixes it to ascending block id (tests compare the reference's
    output after applying the same canonical order within equal runs).
    """
    s = np.asarray(scores, dtype=np.float32)
    if s.shape[0] == 0 or topk_blocks == 0:
        return np.full((*s.shape[:2], topk_blocks), -1, dtype=np.int32)
    _, _, pos = token_positions(cu_seqlens)
    return topk_at_positions(s, pos, block_size=block_size, topk_blocks=topk_blocks, local_blocks=local_blocks)


def topk_at_positions(scores, positions, *, block_size=128, topk_blocks=16, local_blocks=1):
    """:func:`topk` for score rows whose in-sequence token positions are given directly
    (rows sampled from a large problem); same rule, triton/topk.py:33-46."""
    s = np.asarray(scores, dtype=np.float32)
    total, groups, nb = s.shape
    out = np.full((total, groups, topk_blocks), -1, dtype=np.int32)
    if total == 0 or topk_blocks == 0:
        return out
    pos = np.asarray(positions, dtype=np.int64)
    qb = pos // block_size
    blocks = np.arange(nb)
    valid = blocks[None, :] <= qb[:, None]
    ranked = np.where(valid[:, None, :], s, -np.inf)
    if local_blocks:
        local = valid & (blocks[None, :] > qb[:, None] - local_blocks)
        ranked = np.where(local[:, None, :], np.inf, ranked)
    count = min(topk_blocks, nb)
    # Stable sort on the negated value gives descending value, ascending id.
    order = np.argsort(-ranked, axis=-1, kind="stable")[..., :count]
    values = np.take_along_axis(ranked, order, axis=-1)
    out[..., :count] = np.where(values == -np.inf, -1, order).astype(np.int32)
    return out


def canonical_ties(indices, scores, cu_seqlens, *, block_size, local_blocks):
    """Reorder each row's ids so equal ranked values appear in ascending id.

    Applies to any valid top-k output (for example torch.topk's) the canonical
    tie order that :func:`topk` produces, so outputs can be compared exactly.
    """
    ids = np.array(indices, dtype=np.int64, copy=True)
    s = np.asarray(scores, dtype=np.float32)
    _, _, pos = token_positions(cu_seqlens)
    qb = pos // block_size
    total, groups, kk = ids.shape
    for t in range(total):
        for g in range(groups):
            row = ids[t, g]
            kept = [int(b) for b in row if b >= 0]
            def rank_value(b):
                if local_blocks and qb[t] - local_blocks < b <= qb[t]:
                    return math.inf
                return float(s[t, g, b])
            kept.sort(key=lambda b: (-rank_value(b), b))
            ids[t, g] = kept + [-1] * (kk - len(kept))
    return ids.astype(np.int32)


def topk_equivalent(a, b, scores, cu_seqlens, *, block_size, local_blocks):
    """True when two top-k outputs differ only in how exact ties were broken.

    The reference leaves the choice among equal candidates to torch.topk
    (docs/msa_training_flow.md section 2.2: equal scores may select different
    equivalent candidates). Rows must rank the same multiset of values in the
    same order; ids may differ only inside runs of equal values, and only in
    the last run (cut by K) may the chosen members of the run differ.
    """
    s = np.asarray(scores, dtype=np.float32)
    _, _, pos = token_positions(cu_seqlens)
    qb = pos // block_size
    a, b = np.asarray(a), np.asarray(b)
    if a.shape != b.shape:
        return False
    for t in range(a.shape[0]):
        for g in range(a.shape[1]):
            def ranked(row):
                vals = []
                for x in row:
                    if x < 0:
                        vals.append(None)
                    elif local_blocks and qb[t] - local_blocks < x <= qb[t]:
                        vals.append(math.inf)
                    else:
                        vals.append(float(s[t, g, x]))
                return vals
            va, vb = ranked(a[t, g]), ranked(b[t, g])
            if va != vb:
                return False
            kept = [v for v in va if v is not None]
            last = kept[-1] if kept else None
            for value in set(kept):
                ia = sorted(int(x) for x, v in zip(a[t, g], va) if v == value)
                ib = sorted(int(x) for x, v in zip(b[t, g], vb) if v == value)
                if value != last and ia != ib:
                    return False
    return True


# ---------------------------------------------------------------------------
# k2q: block -> query CSR transpose
# ---------------------------------------------------------------------------

INT32_MAX = 2 ** 31 - 1


def k2q_csr(indices, cu_seqlens, *, block_size):
    """(row_ptr, query_indices, slot_indices, cu_block_lens); triton/k2q.py:39-128.

    Row ``(cu_block_lens[seq] + b) * G + g`` lists the valid edges
    ``(query, slot)`` that selected sequence-local block ``b`` for group ``g``,
    ordered by query then slot (k2q.py:117-127). An edge is valid iff
    ``0 <= b < nblocks(seq)`` and ``b <= (t - seq_start) // block_size``
    (k2q.py:101-106). Edge arrays have capacity ``T*G*K`` with a -1 tail.
    """
    ids = np.asarray(indices, dtype=np.int64)
    total, groups, slots = ids.shape
    capacity = total * groups * slots
    if capacity > INT32_MAX:
        raise OverflowError("T * G * K exceeds int32 edge capacity")
    bounds = [int(x) for x in np.asarray(cu_seqlens).tolist()]
    lengths = [b - a for a, b in zip(bounds[:-1], bounds[1:])]
    nblocks = [(n + block_size - 1) // block_size for n in lengths]
    cu_block = np.concatenate([[0], np.cumsum(nblocks)]).astype(np.int64)
    num_rows = int(cu_block[-1]) * groups
    seq, start, pos = token_positions(cu_seqlens)
    cur = pos // block_size
    nbl = np.asarray(nblocks, dtype=np.int64)[seq] if total else np.zeros(0, np.int64)
    valid = (ids >= 0) & (ids < nbl[:, None, None]) & (ids <= cur[:, None, None])
    rows = (cu_block[seq][:, None, None] + ids) * groups + np.arange(groups)[None, :, None]
    flat_valid = valid.reshape(-1)
    flat_rows = rows.reshape(-1)[flat_valid]
    edges = np.nonzero(flat_valid)[0]
    order = np.argsort(flat_rows, kind="stable")  # edge ids are already (query, group, slot)
    edges = edges[order]
    counts = np.bincount(flat_rows, minlength=num_rows) if num_rows else np.zeros(0, np.int64)
    row_ptr = np.zeros(num_rows + 1, dtype=np.int32)
    row_ptr[1:] = np.cumsum(counts)
    query = np.full(capacity, -1, dtype=np.int32)
    slot = np.full(capacity, -1, dtype=np.int32)
    query[:edges.size] = edges // (groups * slots)
    slot[:edges.size] = edges % slots
    return row_ptr, query, slot, cu_block.astype(np.int32)


# ---------------------------------------------------------------------------
# stage 3: block-sparse GQA attention
# ---------------------------------------------------------------------------

def selected_keys(ids_row, seq_start, pos, block_size):
    """Packed key ids a query attends to: union of selected blocks, causal.

    tests/reference_fp64.py:74-75: a key is visible when its block is among the
    selected ids and it is not in the future. Duplicate ids select once.
    """
    blocks = sorted({int(b) for b in ids_row if 0 <= b <= pos // block_size})
    keys = [np.arange(seq_start + b * block_size, seq_start + min((b + 1) * block_size, pos + 1))
            for b in blocks]
    return np.concatenate(keys) if keys else np.zeros(0, dtype=np.int64)


def sparse_attention(q, k, v, indices, cu_seqlens, *, block_size=128, scale=None):
    """float64 (out[T,Hq,D], lse[T,Hq]); tests/reference_fp64.py:48-85.

    Softmax over the selected causal keys of the query's group; rows with no
    visible key give out=0 and lse=-inf (sparse_attention.py:78-84).
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    ids = np.asarray(indices)
    total, hq, dim = q.shape
    groups = k.shape[1]
    ratio = hq // groups
    scale = dim ** -0.5 if scale is None else float(scale)
    out = np.zeros_like(q)
    lse = np.full((total, hq), -np.inf)
    _, start, pos = token_positions(cu_seqlens)
    for t in range(total):
        for g in range(groups):
            keys = selected_keys(ids[t, g], start[t], pos[t], block_size)
            if keys.size == 0:
                continue
            heads = slice(g * ratio, (g + 1) * ratio)
            logits = q[t, heads] @ k[keys, g].T * scale          # [R, n]
            m = logits.max(axis=1, keepdims=True)
            p = np.exp(logits - m)
            l = p.sum(axis=1, keepdims=True)
            out[t, heads] = (p / l) @ v[keys, g]
            lse[t, heads] = (m + np.log(l))[:, 0]
    return out, lse


def sparse_attention_backward(q, k, v, indices, cu_seqlens, dout, *, block_size=128, scale=None):
    """float64 (dq, dk, dv) of ``sum(out * dout)``; the analytic softmax backward.

    Same function the reference differentiates (reference_fp64.py:48-85 under
    autograd; Triton kernels sparse_attention.py:87-295 compute it as
    dS = P * (dP - sum(P*dP)) * scale, dQ = dS K, dK = dS^T Q, dV = P^T dO).
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    do = np.asarray(dout, dtype=np.float64)
    ids = np.asarray(indices)
    total, hq, dim = q.shape
    groups = k.shape[1]
    ratio = hq // groups
    scale = dim ** -0.5 if scale is None else float(scale)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    _, start, pos = token_positions(cu_seqlens)
    for t in range(total):
        for g in range(groups):
            keys = selected_keys(ids[t, g], start[t], pos[t], block_size)
            if keys.size == 0:
                continue
            heads = slice(g * ratio, (g + 1) * ratio)
            kk, vv = k[keys, g], v[keys, g]
            logits = q[t, heads] @ kk.T * scale
            p = np.exp(logits - logits.max(axis=1, keepdims=True))
            p /= p.sum(axis=1, keepdims=True)
            dp = do[t, heads] @ vv.T
            ds = p * (dp - (p * dp).sum(axis=1, keepdims=True)) * scale
            dq[t, heads] = ds @ kk
            np.add.at(dk[:, g], keys, ds.T @ q[t, heads])
            np.add.at(dv[:, g], keys, p.T @ do[t, heads])
    return dq, dk, dv


# ---------------------------------------------------------------------------
# algorithmic work counters (used by bench/tests to state roofline figures)
# ---------------------------------------------------------------------------

def selected_key_count(cu_seqlens, *, block_size, topk_blocks):
    """Sum over tokens of n_sel for distinct valid selections (value independent).

    A token at position p sees (p mod B)+1 keys of its own block plus B keys
    from each of min(K, p//B + 1) - 1 earlier blocks.
    """
    bounds = [int(x) for x in np.asarray(cu_seqlens).tolist()]
    total = 0
    for a, b in zip(bounds[:-1], bounds[1:]):
        p = np.arange(b - a, dtype=np.int64)
        total += int(((p % block_size) + 1 + block_size * (np.minimum(topk_blocks, p // block_size + 1) - 1)).sum())
    return total


# ---------------------------------------------------------------------------
# sampled evaluation for large problems
# ---------------------------------------------------------------------------
#
# The functions above loop over every token, which is exact but far too slow
# for the benchmark shapes (32K-131K tokens x 64 heads). These compute the same
# float64 quantities at sampled positions only: whole score rows of chosen
# query tokens, and the attention outputs / gradients of chosen query tokens
# and chosen (key block, group) rows. They are the same mathematics (they
# reduce to :func:`index_score`, :func:`sparse_attention` and
# :func:`sparse_attention_backward` on small cases, which the CPU tests check),
# organised by key block so that each block's keys meet the selecting queries
# in one matrix product.

def index_score_rows(index_q, index_k, cu_seqlens, max_seqlen, tokens, *, block_size=128, scale=1.0):
    """float64 rows ``S[t, :, :]`` of :func:`index_score` for the packed tokens ``tokens``.

    Same definition as tests/reference_fp64.py:16-45: per (group, block) the
    causal maximum of ``scale * iq[t,g] . ik[j]`` over the block's keys up to
    the token, -inf for future and out-of-sequence blocks.
    """
    nb = (max_seqlen + block_size - 1) // block_size
    k = np.asarray(index_k)[:, 0, :]
    _, start, pos = token_positions(cu_seqlens)
    out = np.full((len(tokens), np.asarray(index_q).shape[1], nb), -np.inf)
    for i, t in enumerate(tokens):
        a, p = int(start[t]), int(pos[t])
        logits = (np.asarray(index_q[t], dtype=np.float64) @ k[a:a + p + 1].astype(np.float64).T) * scale  # [G, p+1]
        for blk in range(p // block_size + 1):
            out[i, :, blk] = logits[:, blk * block_size:min((blk + 1) * block_size, p + 1)].max(axis=1)
    return out


def index_score_backward_sampled(index_q, index_k, cu_seqlens, dscores, *, tokens, key_blocks,
                                 block_size=128, scale=1.0, chunk=2048):
    """Sampled rows of :func:`index_score_backward` (float64): ``dq[t]`` for the packed
    tokens ``tokens`` ([len(tokens), G, Di]) and the ``index_k`` gradient of whole key
    blocks ``key_blocks`` = [(sequence, block)] ([len(key_blocks), block_size, Di], rows
    past the sequence zero), each summed over every (token, group) whose causal block
    maximum the key attains (ties split equally; triton/index_score.py:139-232).
    """
    q = np.asarray(index_q, dtype=np.float64)
    k = np.asarray(index_k, dtype=np.float64)[:, 0, :]
    ds = np.asarray(dscores, dtype=np.float64)
    groups, dim = q.shape[1], q.shape[2]
    _, start, pos = token_positions(cu_seqlens)
    bounds = [int(x) for x in np.asarray(cu_seqlens).tolist()]
    dq = np.zeros((len(tokens), groups, dim))
    for i, t in enumerate(tokens):
        a, p = int(start[t]), int(pos[t])
        nblk = p // block_size + 1
        logits = np.full((nblk * block_size, groups), -np.inf)
        logits[:p + 1] = (k[a:a + p + 1] @ q[t].T) * scale
        blocks = logits.reshape(nblk, block_size, groups)
        win = blocks == blocks.max(axis=1, keepdims=True)
        wt = win * (ds[t, :, :nblk].T * scale / win.sum(axis=1))[:, None, :]  # [nblk, block, G]
        dq[i] = wt.reshape(-1, groups)[:p + 1].T @ k[a:a + p + 1]
    dk = np.zeros((len(key_blocks), block_size, dim))
    for r, (s, b) in enumerate(key_blocks):
        a, length = bounds[s], bounds[s + 1] - bounds[s]
        lo = b * block_size
        n = min(block_size, length - lo)
        if n <= 0:
            continue
        kb = k[a + lo:a + lo + n]
        for c0 in range(lo, length, chunk):  # the sequence's tokens at positions >= lo
            c1 = min(length, c0 + chunk)
            qc = q[a + c0:a + c1].reshape(-1, dim)  # [(t, g), Di]
            logits = ((qc @ kb.T) * scale).reshape(c1 - c0, groups, n)
            future = (lo + np.arange(n))[None, :] > np.arange(c0, c1)[:, None]  # key past the token
            logits[np.broadcast_to(future[:, None, :], logits.shape)] = -np.inf
            win = logits == logits.max(axis=2, keepdims=True)
            wt = win * (ds[a + c0:a + c1, :, b] * scale / win.sum(axis=2))[:, :, None]
            dk[r, :n] += wt.reshape(-1, n).T @ qc
    return dq, dk


def _pairs_edges(ids, seq, start, pos, pairs_t, pairs_g, block_size):
    """Distinct valid (pair, block) edges of the given (token, group) pairs."""
    picks = np.asarray(ids)[pairs_t, pairs_g].astype(np.int64)  # [N, K]
    cur = (pos[pairs_t] // block_size)[:, None]
    ok = (picks >= 0) & (picks <= cur)
    # duplicated ids select their block once (tests/reference_fp64.py:74: membership test)
    srt = np.sort(np.where(ok, picks, -1), axis=1)
    ok = (srt >= 0) & np.concatenate([np.ones((srt.shape[0], 1), bool), srt[:, 1:] != srt[:, :-1]], axis=1)
    pair_of, col = np.nonzero(ok)
    return pair_of, srt[pair_of, col]


def sparse_attention_sampled(q, k, v, indices, cu_seqlens, dout=None, *, block_size=128, scale=None,
                             query_tokens=(), key_rows=()):
    """float64 attention values at sampled positions (tests/reference_fp64.py:48-85 and its autograd).

    Returns a dict with, for the packed tokens ``query_tokens``: ``out`` [n, Hq, D],
    ``lse`` [n, Hq] and, when ``dout`` is given, ``dq`` [n, Hq, D]; for each
    ``(seq, block, group)`` of ``key_rows`` (sequence-local block id): ``dk`` and
    ``dv`` [n_rows, block_size, D] for the block's key tokens (rows past the end of
    the sequence are zero). dK/dV of a block sum over every query that selected it,
    so every such query's softmax statistics are computed first.
    """
    ids = np.asarray(indices)
    total, hq, dim = q.shape
    groups = k.shape[1]
    ratio = hq // groups
    scale = dim ** -0.5 if scale is None else float(scale)
    seq, start, pos = token_positions(cu_seqlens)
    bounds = [int(x) for x in np.asarray(cu_seqlens).tolist()]
    # the (token, group) pairs whose rows are needed
    pair_set = {(int(t), g) for t in query_tokens for g in range(groups)}
    row_members = []
    for s_, b, g in key_rows:
        a, e = bounds[s_], bounds[s_ + 1]
        toks = np.arange(a + b * block_size, e)
        hit = (ids[toks, g, :] == b).any(axis=1)
        members = toks[hit]
        row_members.append(members)
        pair_set.update((int(t), g) for t in members)
    pairs = sorted(pair_set)
    pt = np.array([p[0] for p in pairs], dtype=np.int64)
    pg = np.array([p[1] for p in pairs], dtype=np.int64)
    pair_index = {p: i for i, p in enumerate(pairs)}
    pair_of, blk = _pairs_edges(ids, seq, start, pos, pt, pg, block_size)
    n = len(pairs)
    m = np.full((n, ratio), -np.inf)
    l = np.zeros((n, ratio))
    o = np.zeros((n, ratio, dim))

    def block_groups(edge_mask):
        """Edges grouped by (group, absolute first key of the block)."""
        e = np.nonzero(edge_mask)[0]
        key0 = start[pt[pair_of[e]]] + blk[e] * block_size
        order = np.lexsort((key0, pg[pair_of[e]]))
        e, key0 = e[order], key0[order]
        gg = pg[pair_of[e]]
        cuts = np.nonzero((np.diff(key0) != 0) | (np.diff(gg) != 0))[0] + 1
        for part in np.split(np.arange(e.size), cuts):
            if part.size:
                yield e[part], int(gg[part[0]]), int(key0[part[0]])

    def block_logits(es, g, key0):
        tt = pt[pair_of[es]]
        seq_end = np.array([bounds[int(seq[t]) + 1] for t in tt[:1]])[0]
        nk = min(block_size, seq_end - key0)
        kk = np.asarray(k[key0:key0 + nk, g], dtype=np.float64)
        vv = np.asarray(v[key0:key0 + nk, g], dtype=np.float64)
        qq = np.asarray(q[tt, g * ratio:(g + 1) * ratio], dtype=np.float64)  # [E, R, D]
        s = (qq @ kk.T) * scale  # [E, R, nk]
        visible = (key0 + np.arange(nk))[None, :] <= tt[:, None]  # causal (diagonal block)
        s = np.where(visible[:, None, :], s, -np.inf)
        return tt, qq, kk, vv, s

    # pass 1: online softmax statistics and outputs of every needed pair (float64)
    for es, g, key0 in block_groups(np.ones(pair_of.size, bool)):
        tt, qq, kk, vv, s = block_logits(es, g, key0)
        pi = pair_of[es]
        m_new = np.maximum(m[pi], s.max(axis=2))
        alpha = np.where(np.isfinite(m[pi]), np.exp(m[pi] - m_new), 0.0)
        p = np.exp(s - m_new[:, :, None])
        l[pi] = l[pi] * alpha + p.sum(axis=2)
        o[pi] = o[pi] * alpha[:, :, None] + p @ vv
        m[pi] = m_new
    has = l > 0
    lse = np.where(has, m + np.log(np.where(has, l, 1.0)), -np.inf)
    out = np.where(has[:, :, None], o / np.where(has, l, 1.0)[:, :, None], 0.0)

    result = {}
    qsel = [pair_index[(int(t), g)] for t in query_tokens for g in range(groups)]
    shape_q = (len(query_tokens), groups, ratio)
    result["out"] = out[qsel].reshape(*shape_q, dim).reshape(len(query_tokens), hq, dim)
    result["lse"] = lse[qsel].reshape(len(query_tokens), hq)
    if dout is None:
        return result

    # pass 2: dS = P (dP - delta) scale; dq for the sampled queries, dK/dV for the sampled rows
    go = np.asarray(dout)
    delta = np.einsum("nrd,nrd->nr", np.asarray(go[pt.reshape(-1, 1), pg.reshape(-1, 1) * ratio + np.arange(ratio)],
                                                 dtype=np.float64), out)
    want_q = np.zeros(n, bool)
    want_q[qsel] = True
    row_of = {}
    for r, (s_, b, g) in enumerate(key_rows):
        row_of[(g, bounds[s_] + b * block_size)] = r
    dq = np.zeros((n, ratio, dim))
    dk = np.zeros((len(key_rows), block_size, dim))
    dv = np.zeros((len(key_rows), block_size, dim))
    key0_all = start[pt[pair_of]] + blk * block_size
    in_row = np.array([(int(pg[i]), int(k0)) in row_of for i, k0 in zip(pair_of, key0_all)], dtype=bool)
    for es, g, key0 in block_groups(want_q[pair_of] | in_row):
        tt, qq, kk, vv, s = block_logits(es, g, key0)
        pi = pair_of[es]
        p = np.where(has[pi][:, :, None], np.exp(s - np.where(has[pi], lse[pi], 0.0)[:, :, None]), 0.0)
        dd = np.asarray(go[tt[:, None], g * ratio + np.arange(ratio)], dtype=np.float64)  # [E, R, D]
        dp = dd @ vv.T
        ds = p * (dp - delta[pi][:, :, None]) * scale
        sel = want_q[pi]
        if sel.any():
            np.add.at(dq, pi[sel], ds[sel] @ kk)
        r = row_of.get((g, key0))
        if r is not None:
            nk = kk.shape[0]
            dk[r, :nk] += np.einsum("erj,erd->jd", ds, qq)
            dv[r, :nk] += np.einsum("erj,erd->jd", p, dd)
    result["dq"] = dq[qsel].reshape(len(query_tokens), hq, dim)
    result["dk"] = dk
    result["dv"] = dv
    result["key_row_queries"] = [int(x.size) for x in row_members]
    return result


# ---------------------------------------------------------------------------
# index KL loss (indexer training, sparse stage)
# ---------------------------------------------------------------------------

def index_kl_loss(index_q, index_k, q, k, indices, cu_seqlens, *, block_size=128, index_scale=1.0, scale=None):
    """float64 ``(loss, d_index_q, d_index_k)`` of the indexer's KL objective.

    The reference specifies this loss but does not implement it
    (docs/msa_training_flow.md:92-138, docs/implementation_plan.md:66-69): on the
    selected causal tokens J(t, g) of each (query token, group) -- the same key set
    the sparse attention uses, without the top-k's +inf local boost --

    * student ``p_s = softmax_J(index_scale * iq[t,g] . ik[j])`` (token logits of
      the index projections, not the block scores);
    * teacher ``p_T = mean over the group's heads h of softmax_J(scale * q[t,h] . k[j,g])``
      (the main attention's probabilities, detached);
    * ``loss = sum_{t,g} KL(p_T || p_s) / (T * G)`` -- the mean over the packed
      batch's real (token, group) pairs; a pair that selects no key contributes 0.

    Gradients reach index_q / index_k only: ``dL/ds_j = (p_s(j) - p_T(j)) / (T G)``.
    Parity is unpinned by reference outputs (the reference has no implementation);
    tests check this restatement against an independent autograd computation.
    """
    iq = np.asarray(index_q, dtype=np.float64)
    ik = np.asarray(index_k, dtype=np.float64)[:, 0, :]
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    ids = np.asarray(indices)
    total, hq, dim = q.shape
    groups = k.shape[1]
    ratio = hq // groups
    scale = dim ** -0.5 if scale is None else float(scale)
    _, start, pos = token_positions(cu_seqlens)
    n = max(total * groups, 1)
    loss = 0.0
    diq = np.zeros_like(iq)
    dik = np.zeros_like(ik)
    for t in range(total):
        for g in range(groups):
            keys = selected_keys(ids[t, g], start[t], pos[t], block_size)
            if keys.size == 0:
                continue
            tl = q[t, g * ratio:(g + 1) * ratio] @ k[keys, g].T * scale  # [R, n]
            tp = np.exp(tl - tl.max(axis=1, keepdims=True))
            tp /= tp.sum(axis=1, keepdims=True)
            pt = tp.mean(axis=0)
            s = ik[keys] @ iq[t, g] * index_scale
            m = s.max()
            lse_s = m + np.log(np.exp(s - m).sum())
            logp_s = s - lse_s
            pos_t = pt > 0
            loss += float((pt[pos_t] * (np.log(pt[pos_t]) - logp_s[pos_t])).sum())
            ds = (np.exp(logp_s) - pt) / n * index_scale
            diq[t, g] = ds @ ik[keys]
            np.add.at(dik, keys, ds[:, None] * iq[t, g][None, :])
    return loss / n, diq, dik[:, None, :]


def index_kl_pairs(index_q, index_k, q, k, indices, cu_seqlens, pairs, *, block_size=128, index_scale=1.0,
                   scale=None, key_block=None):
    """float64 terms of ``index_kl_loss`` for the listed (token, group) pairs only (same
    formulas, N = T * G of the whole batch): their KL values, their d_index_q rows, and,
    when ``key_block = (first_key, n_keys)`` is given, the d_index_k rows of those keys
    summed over the listed pairs (exact for the block when the list holds every pair
    that selects it). Lets tests check sampled pairs of a batch too large for the full
    restatement."""
    iq = np.asarray(index_q)
    ik = np.asarray(index_k)[:, 0, :].astype(np.float64)
    ids = np.asarray(indices)
    total, groups = ids.shape[0], ids.shape[1]
    hq, dim = q.shape[1], q.shape[2]
    ratio = hq // groups
    scale = dim ** -0.5 if scale is None else float(scale)
    _, start, pos = token_positions(cu_seqlens)
    n = max(total * groups, 1)
    kls, diq = [], []
    dik = None
    if key_block is not None:
        k0, nk = key_block
        dik = np.zeros((nk, ik.shape[1]))
    for t, g in pairs:
        keys = selected_keys(ids[t, g], start[t], pos[t], block_size)
        if keys.size == 0:
            kls.append(0.0)
            diq.append(np.zeros(ik.shape[1]))
            continue
        qt = np.asarray(q[t, g * ratio:(g + 1) * ratio], dtype=np.float64)
        kt = np.asarray(k[keys, g], dtype=np.float64)
        tl = qt @ kt.T * scale
        tp = np.exp(tl - tl.max(axis=1, keepdims=True))
        tp /= tp.sum(axis=1, keepdims=True)
        pt = tp.mean(axis=0)
        iqt = np.asarray(iq[t, g], dtype=np.float64)
        sl = ik[keys] @ iqt * index_scale
        m = sl.max()
        logp_s = sl - (m + np.log(np.exp(sl - m).sum()))
        pos_t = pt > 0
        kls.append(float((pt[pos_t] * (np.log(pt[pos_t]) - logp_s[pos_t])).sum()))
        ds = (np.exp(logp_s) - pt) / n * index_scale
        diq.append(ds @ ik[keys])
        if dik is not None:
            inside = (keys >= k0) & (keys < k0 + nk)
            np.add.at(dik, keys[inside] - k0, ds[inside, None] * iqt[None, :])
    return np.array(kls), np.array(diq), dik


# ---------------------------------------------------------------------------
# native-dtype eager numerics (the tolerance yardstick of the tensor-core path)
# ---------------------------------------------------------------------------

def sparse_attention_eager(q, k, v, indices, cu_seqlens, max_seqlen, dout=None, *, block_size=128, scale=None):
    """The reference's native-dtype eager attention numerics, with gradients.

    Restates eager/ops.py:130-215 (with the padding adapters of layout.py:27-74):
    sequences right-padded to ``[B, S, H, D]``; ``Q K^T`` in the input dtype,
    times ``scale``; the block/causal/padding keep-mask applied with -inf; softmax
    in float32 cast back to the input dtype; ``P V`` in the input dtype; LSE from
    the float32 logits. Gradients come from torch autograd through the same graph.
    It runs on the CPU in torch (numpy has no bfloat16) and serves only as the
    yardstick of the fast path's stated tolerance ("no worse than twice native
    eager on the same inputs"). Returns float64 numpy ``(out, lse)`` or, with
    ``dout``, ``(out, lse, dq, dk, dv)``.
    """
    import torch

    q = torch.as_tensor(q).detach().cpu()
    k = torch.as_tensor(k).detach().cpu()
    v = torch.as_tensor(v).detach().cpu()
    ids = torch.as_tensor(np.asarray(indices)).to(torch.int64)
    bounds = [int(x) for x in np.asarray(cu_seqlens).tolist()]
    lengths = [b - a for a, b in zip(bounds[:-1], bounds[1:])]
    hq, groups = q.shape[1], k.shape[1]
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    leaves = [x.clone().requires_grad_(dout is not None) for x in (q, k, v)]

    def pad(x, fill):
        rows = [torch.cat([x[a:b], x.new_full((max_seqlen - (b - a), *x.shape[1:]), fill)])
                for a, b in zip(bounds[:-1], bounds[1:])]
        return torch.stack(rows)

    qb, kb, vb = (pad(x, 0) for x in leaves)
    idb = pad(ids, -1)
    valid = torch.arange(max_seqlen)[None, :] < torch.tensor(lengths)[:, None]
    nblk = (max_seqlen + block_size - 1) // block_size
    sel = idb.transpose(1, 2)
    sel = sel.masked_fill((sel < 0) | (sel >= nblk), nblk)
    keep_b = torch.zeros((len(lengths), groups, max_seqlen, nblk + 1), dtype=torch.bool)
    keep_b.scatter_(-1, sel, True)
    keep = keep_b[..., :nblk].repeat_interleave(block_size, dim=-1)[..., :max_seqlen]
    keep = keep.repeat_interleave(hq // groups, dim=1)
    pos = torch.arange(max_seqlen)
    keep = keep & (pos[None, :] <= pos[:, None])[None, None] & valid[:, None, None, :] & valid[:, None, :, None]
    qh = qb.transpose(1, 2)
    kh = kb.transpose(1, 2).repeat_interleave(hq // groups, dim=1)
    vh = vb.transpose(1, 2).repeat_interleave(hq // groups, dim=1)
    w = torch.matmul(qh, kh.transpose(-1, -2)) * scale
    w = w.masked_fill(~keep, float("-inf"))
    has = keep.any(-1, keepdim=True)
    safe = torch.where(has, w, torch.zeros_like(w))
    probs = torch.softmax(safe, dim=-1, dtype=torch.float32).to(q.dtype).masked_fill(~has, 0)
    out = torch.matmul(probs, vh).transpose(1, 2)
    lse = torch.logsumexp(safe.float(), dim=-1).masked_fill(~has.squeeze(-1), float("-inf")).transpose(1, 2)
    out_p = torch.cat([out[i, :n] for i, n in enumerate(lengths)])
    lse_p = torch.cat([lse[i, :n] for i, n in enumerate(lengths)])
    res = [out_p.detach().double().numpy(), lse_p.detach().double().numpy()]
    if dout is None:
        return tuple(res)
    out_p.backward(torch.as_tensor(dout).to(q.dtype))
    return tuple(res + [x.grad.double().numpy() for x in leaves])
