"""torch.library operators on the GPU: a projection -> index score -> top-k ->
sparse attention -> projection module under ``torch.compile(fullgraph=True)``
matches the same module run eagerly (restates the reference's
tests/test_pipeline.py:60-87 module with a compiled twin), for both kernel
families; and the registered ops pass ``torch.library.opcheck``."""

import pytest
import torch

from msa_triton_b200 import _lib, m3_index_score, m3_sparse_attention, m3_topk, prepare_batch
from tests.helpers import cu_of

pytestmark = pytest.mark.gpu


class Layer(torch.nn.Module):
    """x -> (index_q, index_k) -> scores -> top-k ids; x -> q, k, v -> sparse attention -> output."""

    def __init__(self, hidden, groups, ratio, dim, index_dim, block, topk, dtype):
        super().__init__()
        g = torch.Generator().manual_seed(7)

        def w(i, o, s):
            return torch.nn.Parameter((torch.randn(i, o, generator=g) * s).to(dtype))

        self.groups, self.ratio, self.dim, self.index_dim = groups, ratio, dim, index_dim
        self.block, self.topk = block, topk
        self.wq = w(hidden, groups * ratio * dim, hidden ** -0.5)
        self.wk = w(hidden, groups * dim, hidden ** -0.5)
        self.wv = w(hidden, groups * dim, hidden ** -0.5)
        self.wo = w(groups * ratio * dim, hidden, (groups * ratio * dim) ** -0.5)
        self.wiq = w(hidden, groups * index_dim, hidden ** -0.5)
        self.wik = w(hidden, index_dim, hidden ** -0.5)

    def forward(self, x, cu, prepared, max_seqlen):
        t = x.shape[0]
        iq = (x @ self.wiq).reshape(t, self.groups, self.index_dim)
        ik = (x @ self.wik).reshape(t, 1, self.index_dim)
        scores = m3_index_score(iq, ik, cu, max_seqlen, block_size=self.block, prepared=prepared)
        ids = m3_topk(scores.detach(), cu, block_size=self.block, topk_blocks=self.topk, local_blocks=1,
                      prepared=prepared)
        q = (x @ self.wq).reshape(t, self.groups * self.ratio, self.dim)
        k = (x @ self.wk).reshape(t, self.groups, self.dim)
        v = (x @ self.wv).reshape(t, self.groups, self.dim)
        out = m3_sparse_attention(q, k, v, ids, cu, max_seqlen, block_size=self.block, prepared=prepared)
        y = out.reshape(t, -1) @ self.wo
        # the indexer trains through its finite scores (future blocks are -inf)
        index_term = torch.where(torch.isfinite(scores), scores, torch.zeros_like(scores)).float().mean()
        return y, ids, index_term


def run(model, x, cu, prepared, max_seqlen, fn):
    model.zero_grad(set_to_none=True)
    xx = x.detach().clone().requires_grad_()
    y, ids, index_term = fn(xx, cu, prepared, max_seqlen)
    loss = y.float().square().mean() + 1e-3 * index_term
    loss.backward()
    torch.cuda.synchronize()
    return [y.detach().float(), ids] + [xx.grad.float()] + [p.grad.float() for p in model.parameters()]


@pytest.mark.parametrize("family", ["tensor-core", "precise"])
def test_compiled_layer_matches_eager(family, cuda_device):
    torch._dynamo.reset()
    if family == "tensor-core":  # bf16, head dim 128, block 128, 8 query heads per group
        lengths, hidden, groups, ratio, dim, index_dim, block, topk, dtype = [700, 333], 256, 2, 8, 128, 64, 128, 3, \
            torch.bfloat16
    else:  # float32, small dims: the float64 precise kernels
        lengths, hidden, groups, ratio, dim, index_dim, block, topk, dtype = [13, 30], 24, 2, 2, 8, 8, 4, 3, \
            torch.float32
    model = Layer(hidden, groups, ratio, dim, index_dim, block, topk, dtype).to(cuda_device)
    x = torch.randn(sum(lengths), hidden, generator=torch.Generator().manual_seed(3)).to(dtype).to(cuda_device)
    cu = cu_of(lengths, cuda_device)
    prepared = prepare_batch(cu)
    eager = run(model, x, cu, prepared, max(lengths), model)
    launches = _lib.kernel_launches()
    compiled = torch.compile(model, fullgraph=True)
    got = run(model, x, cu, prepared, max(lengths), compiled)
    assert _lib.kernel_launches() > launches  # the compiled graph launched this library's kernels
    assert torch.equal(got[1], eager[1])  # the same selection
    tol = dict(atol=2e-2, rtol=2e-2) if dtype == torch.bfloat16 else dict(atol=1e-5, rtol=1e-5)
    names = ["y", "ids", "x.grad"] + [n for n, _ in model.named_parameters()]
    for name, a, e in zip(names, got, eager):
        if name == "ids":
            continue
        scale = float(e.abs().max()) or 1.0
        torch.testing.assert_close(a / scale, e / scale, **tol, msg=name)


def test_registered_ops_pass_opcheck(cuda_device):
    """Schema, fake kernels and autograd registration checked by torch.library.opcheck."""
    gen = torch.Generator().manual_seed(11)
    lengths = [300, 129]
    cu = cu_of(lengths, cuda_device)
    bounds = [0, 300, 429]
    for dtype, dim, ratio, block in ((torch.bfloat16, 128, 8, 128), (torch.float32, 8, 2, 4)):
        q = torch.randn(429, 2 * ratio, dim, generator=gen).to(dtype).to(cuda_device).requires_grad_()
        k = torch.randn(429, 2, dim, generator=gen).to(dtype).to(cuda_device).requires_grad_()
        v = torch.randn(429, 2, dim, generator=gen).to(dtype).to(cuda_device).requires_grad_()
        iq = torch.randn(429, 2, 64, generator=gen).to(dtype).to(cuda_device).requires_grad_()
        ik = torch.randn(429, 1, 64, generator=gen).to(dtype).to(cuda_device).requires_grad_()
        torch.library.opcheck(torch.ops.msa_b200.index_score.default, (iq, ik, cu, 300, block, 1.0, True),
                              test_utils=("test_schema", "test_faketensor"))
        scores = m3_index_score(iq.detach(), ik.detach(), cu, 300, block_size=block)
        torch.library.opcheck(torch.ops.msa_b200.topk.default, (scores, cu, bounds, block, 3, 1),
                              test_utils=("test_schema", "test_faketensor"))
        ids = m3_topk(scores, cu, block_size=block, topk_blocks=3)
        torch.library.opcheck(torch.ops.msa_b200.sparse_attention.default,
                              (q, k, v, ids, cu, bounds, block, dim ** -0.5),
                              test_utils=("test_schema", "test_faketensor"))
