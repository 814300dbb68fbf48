"""Seeded synthetic workloads for the benchmark configurations.

The reference publishes no dataset or benchmark suite for this path; these
generators reproduce the five configurations' shapes and value distributions:
every tensor is drawn N(0, 1) in float32 from one ``torch.Generator`` seeded 0
in the order index_q, index_k, q, k, v, grad_out; each head vector is divided
by its RMS over the last dimension (unit RMS, as after norm/RoPE) and cast to
the compute dtype. Generation happens on the CPU so values are identical on
every machine; callers move the tensors to the device.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    lengths: tuple[int, ...]
    q_heads: int
    groups: int
    dim: int
    index_dim: int
    block_size: int
    topk_blocks: int
    local_blocks: int
    backward: bool
    note: str = field(default="")

    @property
    def total_tokens(self) -> int:
        return sum(self.lengths)

    @property
    def max_seqlen(self) -> int:
        return max(self.lengths)

    def cu_seqlens(self) -> torch.Tensor:
        bounds = [0]
        for n in self.lengths:
            bounds.append(bounds[-1] + n)
        return torch.tensor(bounds, dtype=torch.int32)


def _config3_lengths() -> tuple[int, ...]:
    gen = torch.Generator().manual_seed(0)
    return tuple(int(x) * 128 for x in torch.randint(4, 65, (16,), generator=gen).tolist())


CONFIGS = {
    1: Workload("cfg1_varlen_2x1024", (1024, 1024), 16, 4, 128, 64, 128, 4, 1, True,
                "CPU-runnable small varlen case, fwd+bwd"),
    2: Workload("cfg2_prefill_8k", (8192,), 32, 8, 128, 64, 128, 16, 1, False,
                "single-sequence prefill, forward only"),
    3: Workload("cfg3_packed_16seq", _config3_lengths(), 32, 8, 128, 64, 128, 16, 1, True,
                "packed varlen training batch, sharded by whole sequences"),
    4: Workload("cfg4_32k_headline", (32768,), 64, 8, 128, 64, 128, 16, 1, True,
                "long-context headline, fwd+bwd"),
    5: Workload("cfg5_128k_cp", (131072,), 64, 8, 128, 64, 128, 32, 2, True,
                "context-parallel very long sequence"),
}


def _unit_rms(x: torch.Tensor) -> torch.Tensor:
    return x / x.square().mean(dim=-1, keepdim=True).sqrt()


def make_inputs(w: Workload, *, dtype=torch.bfloat16, seed: int = 0):
    """Return dict(index_q, index_k, q, k, v, grad_out, cu_seqlens) on the CPU."""
    gen = torch.Generator().manual_seed(seed)
    t = w.total_tokens

    def draw(heads, dim):
        return _unit_rms(torch.randn(t, heads, dim, generator=gen)).to(dtype)

    iq = draw(w.groups, w.index_dim)
    ik = draw(1, w.index_dim)
    q = draw(w.q_heads, w.dim)
    k = draw(w.groups, w.dim)
    v = draw(w.groups, w.dim)
    go = draw(w.q_heads, w.dim)
    return dict(index_q=iq, index_k=ik, q=q, k=k, v=v, grad_out=go, cu_seqlens=w.cu_seqlens())


def selected_key_count(w: Workload) -> int:
    """Sum over tokens of the keys a token attends to (distinct valid picks)."""
    total = 0
    for n in w.lengths:
        p = torch.arange(n, dtype=torch.int64)
        kb = torch.clamp(p // w.block_size + 1, max=w.topk_blocks)
        total += int(((p % w.block_size) + 1 + w.block_size * (kb - 1)).sum())
    return total


def attention_flops(w: Workload) -> dict:
    """Algorithmic FLOPs: fwd 4*D*n_sel*Hq, bwd 8*D*n_sel*Hq (no recompute)."""
    nsel = selected_key_count(w) * w.q_heads
    fwd = 4 * w.dim * nsel
    return {"fwd": fwd, "bwd": 2 * fwd, "fwd_bwd": 3 * fwd}


def index_score_flops(w: Workload) -> int:
    """2*Di*G per causal (query, key) pair."""
    pairs = sum(n * (n + 1) // 2 for n in w.lengths)
    return 2 * w.index_dim * w.groups * pairs


def random_selection(lengths, groups, block_size, topk, seed=0, local_blocks=1):
    """Distinct causal picks: the local blocks plus random earlier blocks, -1 padded.

    Random scores ranked with the selection rule of the top-k stage (future
    blocks excluded, local blocks forced), so rows look like real selections.
    """
    gen = torch.Generator().manual_seed(seed)
    total = sum(lengths)
    nb = (max(lengths) + block_size - 1) // block_size
    pos = torch.cat([torch.arange(n) for n in lengths]) if total else torch.zeros(0, dtype=torch.long)
    qb = (pos // block_size)[:, None, None]
    blocks = torch.arange(nb)[None, None, :]
    scores = torch.rand(total, groups, nb, generator=gen)
    scores = scores.masked_fill(blocks > qb, -float("inf"))
    scores = scores.masked_fill((blocks <= qb) & (blocks > qb - local_blocks), float("inf"))
    count = min(topk, nb)
    values, picked = torch.topk(scores, count, dim=-1)
    ids = torch.full((total, groups, topk), -1, dtype=torch.int32)
    ids[..., :count] = picked.masked_fill(values == -float("inf"), -1).to(torch.int32)
    return ids
