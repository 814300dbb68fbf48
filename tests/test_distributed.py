"""Multi-process sharding logic on the CPU (gloo, world sizes 2 and 4): whole-sequence
sharding of packed batches (LPT) and context parallelism of one sequence
(all-gather of index_k / K / V, reduce-scatter of dK / dV). The per-rank compute
is the float64 oracle here (the CUDA kernels need a GPU); what is under test is
the partitioning and the collectives, checked against the single-process oracle."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from msa_triton_b200 import distributed as D
from msa_triton_b200.workloads import CONFIGS, random_selection
from oracle import msa_oracle as O
from tests.helpers import cu_of

def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def spawn(world, fn, *args):
    port = free_port()
    mp.spawn(_entry, args=(world, fn, port, args), nprocs=world, join=True)


def _entry(rank, world, fn, port, args):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fn(rank, *args)
    finally:
        dist.destroy_process_group()


def inputs(lengths, groups, ratio, dim, topk, seed):
    gen = torch.Generator().manual_seed(seed)
    total = sum(lengths)
    q = torch.randn(total, groups * ratio, dim, generator=gen, dtype=torch.float64)
    k = torch.randn(total, groups, dim, generator=gen, dtype=torch.float64)
    v = torch.randn(total, groups, dim, generator=gen, dtype=torch.float64)
    go = torch.randn(total, groups * ratio, dim, generator=gen, dtype=torch.float64)
    ids = random_selection(lengths, groups, 16, topk, seed=seed)
    return q, k, v, go, ids


# ------------------------------------------------------------------ LPT planning (no processes)
def test_lpt_plan_assigns_each_sequence_once_and_balances():
    w = CONFIGS[3]
    cost = [D.sequence_cost(n, q_heads=w.q_heads, groups=w.groups, dim=w.dim, index_dim=w.index_dim,
                            block_size=w.block_size, topk_blocks=w.topk_blocks) for n in w.lengths]
    for world in (1, 2, 4, 8):
        shards = D.plan_sequence_shards(cost, world)
        assert sorted(i for s in shards for i in s) == list(range(len(cost)))
        loads = [sum(cost[i] for i in s) for s in shards]
        assert max(loads) <= sum(cost) / world + max(cost)  # LPT bound
    assert D.plan_sequence_shards(cost, 4) == D.plan_sequence_shards(cost, 4)


def test_selected_keys_matches_workload_count():
    from msa_triton_b200.workloads import selected_key_count
    w = CONFIGS[3]
    assert sum(D.selected_keys(n, w.block_size, w.topk_blocks) for n in w.lengths) == selected_key_count(w)


def test_shard_tokens_cover_the_batch_once():
    lengths = [40, 0, 130, 7, 64, 1]
    cu = cu_of(lengths)
    seen = []
    for r in range(3):
        sh = D.shard_packed_batch(cu, 3, r, q_heads=4, groups=2, dim=8, index_dim=8, block_size=16, topk_blocks=2)
        assert sh.cu_seqlens[-1].item() == sh.token_index.numel()
        assert sh.max_seqlen == max([lengths[s] for s in sh.sequences], default=0)
        seen.append(sh.token_index)
    assert torch.equal(torch.sort(torch.cat(seen)).values, torch.arange(sum(lengths)))


def test_context_parallel_range_requires_even_split():
    assert D.context_parallel_range(1024, 4, 3) == (768, 1024)
    with pytest.raises(ValueError, match="divisible"):
        D.context_parallel_range(1000, 3, 0)


# ------------------------------------------------------------------ packed batch over 2 and 4 ranks
def _packed_rank(rank, lengths, groups, ratio, dim, topk):
    q, k, v, go, ids = inputs(lengths, groups, ratio, dim, topk, seed=3)
    cu = cu_of(lengths)
    world = dist.get_world_size()
    sh = D.shard_packed_batch(cu, world, rank, q_heads=groups * ratio, groups=groups, dim=dim, index_dim=dim,
                              block_size=16, topk_blocks=topk)
    lq, lk, lv, lids = (D.take_tokens(x, sh) for x in (q, k, v, ids))
    out, _ = O.sparse_attention(lq.numpy(), lk.numpy(), lv.numpy(), lids.numpy(), sh.cu_seqlens.numpy(),
                                block_size=16)
    parts = [None] * world
    dist.all_gather_object(parts, (sh.token_index.numpy(), out))
    if rank == 0:
        full, _ = O.sparse_attention(q.numpy(), k.numpy(), v.numpy(), ids.numpy(), cu.numpy(), block_size=16)
        got = np.zeros_like(full)
        for index, o in parts:
            got[index] = o
        np.testing.assert_allclose(got, full, rtol=0, atol=1e-12)


@pytest.mark.parametrize("world", [2, 4])
def test_packed_batch_sharding_matches_single_process(world):
    spawn(world, _packed_rank, [37, 80, 5, 64, 0, 21], 2, 2, 8, 3)


# ------------------------------------------------------------------ context parallelism over 2 and 4 ranks
def _oracle_prepare(ids_full, cu, block_size):
    return None


def _oracle_forward_local(q_full, k_full, v_full, ids_full, cu, block_size, scale, lo, hi, csr):
    # rows outside [lo, hi) are left uninitialised by the rank-local path: poison them
    out, _ = O.sparse_attention(q_full.double().numpy(), k_full.double().numpy(), v_full.double().numpy(),
                                ids_full.numpy(), cu.numpy(), block_size=block_size, scale=scale)
    out[:lo] = np.nan
    out[hi:] = np.nan
    return torch.from_numpy(out).to(q_full.dtype), (q_full, k_full, v_full, ids_full, cu, block_size, scale)


def _oracle_backward_local(state, grad_full, lo, hi):
    q, k, v, ids, cu, block_size, scale = state
    g = grad_full.double().clone()
    g[:lo] = 0  # never-written rows of the full-length gradient buffer; their queries select nothing
    g[hi:] = 0
    dq, dk, dv = O.sparse_attention_backward(q.double().nan_to_num().numpy(), k.double().numpy(), v.double().numpy(),
                                             ids.numpy(), cu.numpy(), g.numpy(), block_size=block_size, scale=scale)
    return torch.from_numpy(dq).to(q.dtype), torch.from_numpy(dk).float(), torch.from_numpy(dv).float()


def _cp_rank(rank, total, groups, ratio, dim, topk):
    D._cp_prepare = _oracle_prepare
    D._cp_forward_local = _oracle_forward_local
    D._cp_backward_local = _oracle_backward_local
    q, k, v, go, ids = inputs([total], groups, ratio, dim, topk, seed=11)
    lo, hi = D.context_parallel_range(total, dist.get_world_size(), rank)
    lq, lk, lv = (x[lo:hi].clone().requires_grad_() for x in (q, k, v))
    out = D.cp_sparse_attention(lq, lk, lv, ids[lo:hi].contiguous(), total, block_size=16)
    out.backward(go[lo:hi])
    cu = cu_of([total])
    ref_out, _ = O.sparse_attention(q.numpy(), k.numpy(), v.numpy(), ids.numpy(), cu.numpy(), block_size=16)
    rdq, rdk, rdv = O.sparse_attention_backward(q.numpy(), k.numpy(), v.numpy(), ids.numpy(), cu.numpy(), go.numpy(),
                                                block_size=16)
    np.testing.assert_allclose(out.detach().numpy(), ref_out[lo:hi], rtol=0, atol=1e-12)
    np.testing.assert_allclose(lq.grad.numpy(), rdq[lo:hi], rtol=0, atol=1e-12)
    # dK / dV: float32 partial sums reduce-scattered, then cast back
    np.testing.assert_allclose(lk.grad.numpy(), rdk[lo:hi], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(lv.grad.numpy(), rdv[lo:hi], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("world", [2, 4])
def test_context_parallel_attention_matches_single_process(world):
    spawn(world, _cp_rank, 128, 2, 2, 8, 3)


def _oracle_scores(iq_full, ik_full, total, lo, hi, block_size, scale):
    s = O.index_score(iq_full.double().numpy(), ik_full.double().numpy(), np.array([0, total]), total,
                      block_size=block_size, scale=scale)
    s[:lo] = np.nan  # rows the kernel does not compute
    s[hi:] = np.nan
    return torch.from_numpy(s).float()


def _oracle_topk(scores_local, lo, total, block_size, topk_blocks, local_blocks):
    s = scores_local.numpy().copy()
    assert not np.isnan(s).any()  # only the rank's (computed) rows are ranked
    return torch.from_numpy(O.topk_at_positions(s, np.arange(lo, lo + s.shape[0]), block_size=block_size,
                                                topk_blocks=topk_blocks, local_blocks=local_blocks))


def _cp_select_rank(rank, total, groups, dim, topk):
    D._cp_scores = _oracle_scores
    D._cp_topk = _oracle_topk
    gen = torch.Generator().manual_seed(5)
    iq = torch.randn(total, groups, dim, generator=gen).bfloat16().float()
    ik = torch.randn(total, 1, dim, generator=gen).bfloat16().float()
    lo, hi = D.context_parallel_range(total, dist.get_world_size(), rank)
    ids = D.cp_select_blocks(iq[lo:hi].contiguous(), ik[lo:hi].contiguous(), total, block_size=16, topk_blocks=topk)
    full = O.index_score(iq.double().numpy(), ik.double().numpy(), np.array([0, total]), total, block_size=16)
    want = O.topk(full.astype(np.float32), np.array([0, total]), block_size=16, topk_blocks=topk, local_blocks=1)
    np.testing.assert_array_equal(ids.numpy(), want[lo:hi])


@pytest.mark.parametrize("world,total", [(2, 96), (4, 128)])
def test_context_parallel_block_selection_matches_single_process(world, total):
    spawn(world, _cp_select_rank, total, 2, 8, 3)
