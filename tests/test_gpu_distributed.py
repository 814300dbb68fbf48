"""Context parallelism and packed-batch sharding on GPUs (NCCL). With one GPU the
context-parallel path runs as a single rank (the query-range score kernel, the
full-length attention buffers and the float32 dK/dV partials are all on the
path); with two or more GPUs, two ranks split one sequence and each rank
compares its slice with the single-GPU result of the whole sequence."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from msa_triton_b200 import distributed as D
from msa_triton_b200 import m3_index_score, m3_sparse_attention, m3_topk
from tests.helpers import cu_of

pytestmark = pytest.mark.gpu


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def unit_rms(x):
    return x / x.square().mean(-1, keepdim=True).sqrt()


def make(total, groups, ratio, seed=7):
    gen = torch.Generator().manual_seed(seed)
    iq = unit_rms(torch.randn(total, groups, 64, generator=gen)).bfloat16()
    ik = unit_rms(torch.randn(total, 1, 64, generator=gen)).bfloat16()
    q = unit_rms(torch.randn(total, groups * ratio, 128, generator=gen)).bfloat16()
    k = unit_rms(torch.randn(total, groups, 128, generator=gen)).bfloat16()
    v = unit_rms(torch.randn(total, groups, 128, generator=gen)).bfloat16()
    go = unit_rms(torch.randn(total, groups * ratio, 128, generator=gen)).bfloat16()
    return iq, ik, q, k, v, go


def direct(dev, total, iq, ik, q, k, v, go, topk):
    cu = cu_of([total], dev)
    with torch.no_grad():
        ids = m3_topk(m3_index_score(iq.to(dev), ik.to(dev), cu, total), cu, topk_blocks=topk)
    qkv = [x.to(dev).requires_grad_() for x in (q, k, v)]
    out = m3_sparse_attention(*qkv, ids, cu, total)
    out.backward(go.to(dev))
    return ids, out.detach(), [x.grad for x in qkv]


def cp_run(dev, rank, world, total, iq, ik, q, k, v, go, topk):
    lo, hi = D.context_parallel_range(total, world, rank)
    ids = D.cp_select_blocks(iq[lo:hi].to(dev), ik[lo:hi].to(dev), total, topk_blocks=topk)
    qkv = [x[lo:hi].to(dev).requires_grad_() for x in (q, k, v)]
    out = D.cp_sparse_attention(*qkv, ids, total)
    out.backward(go[lo:hi].to(dev))
    return ids, out.detach(), [x.grad for x in qkv]


def close(name, got, want):
    """Within two bf16 rounding steps of the single-GPU value (rtol 2^-6) plus 1e-2: the
    context-parallel dK/dV are float32 partial sums added across ranks and rounded once,
    the single-GPU ones one float32 sum rounded once, and dQ / out accumulate their float32
    sums in another order; |dK| reaches several units at these sizes, where one bf16 step
    is 2^-6 .. 2^-5."""
    got, want = got.float(), want.float()
    assert torch.isfinite(got).all(), name
    err = (got - want).abs()
    bound = 2 ** -6 * want.abs() + 1e-2
    worst = int((err - bound).argmax())
    assert bool((err <= bound).all()), (f"{name}: max err {err.max().item():.4g} at |want| "
                                        f"{want.flatten()[worst].abs().item():.4g} (bound "
                                        f"{bound.flatten()[worst].item():.4g}), max |want| {want.abs().max().item():.4g}")


def compare(rank, world, total, cp, ref):
    lo, hi = D.context_parallel_range(total, world, rank)
    assert torch.equal(cp[0], ref[0][lo:hi])  # identical selections
    close("out", cp[1], ref[1][lo:hi])
    for name, got, want in zip(("dq", "dk", "dv"), cp[2], ref[2]):
        close(name, got, want[lo:hi])


@pytest.mark.parametrize("world", [2, 4, 8])
def test_context_parallel_ranks_emulated_on_one_gpu(world, cuda_device):
    """Every rank of a `world`-rank context-parallel run, one after another on one GPU:
    the rank's selection (query-range score + top-k on the gathered index_k), its local
    forward and backward on full-length buffers (query-range entry points, rows of other
    ranks left unwritten), and the float32 dK/dV partials summed over ranks as the
    reduce-scatter would, against the single-GPU run of the whole sequence."""
    total, groups, ratio, topk = 4096, 2, 8, 8
    iq, ik, q, k, v, go = (x.to(cuda_device) for x in make(total, groups, ratio))
    ref = direct(cuda_device, total, iq, ik, q, k, v, go, topk)
    cu = cu_of([total], cuda_device)
    scale = 128 ** -0.5
    dk_sum = torch.zeros(k.shape, dtype=torch.float32, device=cuda_device)
    dv_sum = torch.zeros_like(dk_sum)
    for rank in range(world):
        lo, hi = D.context_parallel_range(total, world, rank)
        iq_full = torch.full_like(iq, float("nan"))  # rows of other ranks must never be read
        iq_full[lo:hi] = iq[lo:hi]
        scores = D._cp_scores(iq_full, ik, total, lo, hi, 128, 1.0)
        ids = D._cp_topk(scores[lo:hi], lo, total, 128, topk, 1)
        assert torch.equal(ids, ref[0][lo:hi]), rank
        ids_full = torch.full((total, groups, topk), -1, dtype=torch.int32, device=cuda_device)
        ids_full[lo:hi] = ids
        q_full = torch.full_like(q, float("nan"))
        q_full[lo:hi] = q[lo:hi]
        csr = D._cp_prepare(ids_full, cu, 128)
        out_full, state = D._cp_forward_local(q_full, k, v, ids_full, cu, 128, scale, lo, hi, csr)
        close(f"out rank {rank}", out_full[lo:hi], ref[1][lo:hi])
        grad_full = torch.full_like(go, float("nan"))
        grad_full[lo:hi] = go[lo:hi]
        dq_full, dk, dv = D._cp_backward_local(state, grad_full, lo, hi)
        close(f"dq rank {rank}", dq_full[lo:hi], ref[2][0][lo:hi])
        assert torch.isfinite(dk).all() and torch.isfinite(dv).all(), rank
        dk_sum += dk
        dv_sum += dv
    close("dk", dk_sum.to(k.dtype), ref[2][1])
    close("dv", dv_sum.to(v.dtype), ref[2][2])


def test_context_parallel_single_rank_matches_direct(cuda_device):
    total, groups, ratio, topk = 2048, 2, 8, 6
    data = make(total, groups, ratio)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(free_port())
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=cuda_device)
    try:
        cp = cp_run(cuda_device, 0, 1, total, *data, topk)
    finally:
        dist.destroy_process_group()
    compare(0, 1, total, cp, direct(cuda_device, total, *data, topk))


def _two_rank(rank, port, total, groups, ratio, topk):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=2, device_id=dev)
    try:
        data = make(total, groups, ratio)
        cp = cp_run(dev, rank, 2, total, *data, topk)
    finally:
        dist.destroy_process_group()
    compare(rank, 2, total, cp, direct(dev, total, *data, topk))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_context_parallel_two_ranks_match_single_gpu():
    mp.spawn(_two_rank, args=(free_port(), 4096, 2, 8, 8), nprocs=2, join=True)


def test_packed_shard_runs_unchanged_ops(cuda_device):
    lengths = [700, 129, 1500, 64]
    cu = cu_of(lengths)
    _, _, q, k, v, go = make(sum(lengths), 2, 8, seed=3)
    from msa_triton_b200.workloads import random_selection
    ids = random_selection(lengths, 2, 128, 4, seed=3)
    qkv = [x.to(cuda_device).requires_grad_() for x in (q, k, v)]
    full = m3_sparse_attention(*qkv, ids.to(cuda_device), cu.to(cuda_device), max(lengths))
    for r in range(2):
        sh = D.shard_packed_batch(cu, 2, r, q_heads=16, groups=2, dim=128, index_dim=64, topk_blocks=4)
        lq, lk, lv, lids = (D.take_tokens(x.to(cuda_device), sh) for x in (q, k, v, ids))
        out = m3_sparse_attention(lq, lk, lv, lids, sh.cu_seqlens.to(cuda_device), sh.max_seqlen)
        want = D.take_tokens(full.detach(), sh)
        assert (out.float() - want.float()).abs().max().item() < 2e-2
