"""The torch.library operators' fake (meta) kernels on the CPU: output shapes and
dtypes from the arguments alone, for both kernel families, under
FakeTensorMode (no device, no CUDA library call)."""

import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import msa_triton_b200.library  # noqa: F401  (registers the msa_b200 operators)


def test_fake_kernels_give_output_shapes():
    ops = torch.ops.msa_b200
    with FakeTensorMode():
        cu = torch.empty(3, dtype=torch.int32, device="cuda")
        bounds = [0, 300, 429]
        iq = torch.empty(429, 8, 64, dtype=torch.bfloat16, device="cuda")
        ik = torch.empty(429, 1, 64, dtype=torch.bfloat16, device="cuda")
        s, mv, tie = ops.index_score(iq, ik, cu, 300, 128, 1.0, True)
        assert s.shape == (429, 8, 3) and s.dtype == torch.float32
        assert mv.shape == (429, 8, 3) and mv.dtype == torch.float64 and tie.dtype == torch.int32
        s2, mv2, _ = ops.index_score(iq, ik, cu, 300, 128, 1.0, False)
        assert s2.shape == (429, 8, 3) and mv2.numel() == 0
        dq, dk = ops.index_score_backward(iq, ik, cu, mv, tie, s, 128, 1.0, True, True, False)
        assert dq.shape == iq.shape and dk.numel() == 0
        ids = ops.topk(s, cu, bounds, 128, 16, 1)
        assert ids.shape == (429, 8, 16) and ids.dtype == torch.int32
        # tensor-core family: float32 LSE saved, the CSR of (3 + 2 blocks) x 8 groups + 1 rows
        q = torch.empty(429, 64, 128, dtype=torch.bfloat16, device="cuda")
        k = torch.empty(429, 8, 128, dtype=torch.bfloat16, device="cuda")
        out = ops.sparse_attention(q, k, k, ids, cu, bounds, 128, 128 ** -0.5)
        assert out[0].shape == q.shape and out[1].shape == (429, 64) and out[2].numel() == 0
        assert out[3].shape == (5 * 8 + 1,) and out[4].shape == (429 * 8 * 16,) and out[6].shape == (3,)
        grads = ops.sparse_attention_backward(q, k, k, ids, cu, bounds, 128, 0.1, *out, q, True, True, False, True)
        assert grads[0].shape == q.shape and grads[1].numel() == 0 and grads[2].shape == k.shape
        # precise family (float32): float64 LSE saved, no CSR from the forward
        q32 = torch.empty(429, 4, 8, dtype=torch.float32, device="cuda")
        k32 = torch.empty(429, 2, 8, dtype=torch.float32, device="cuda")
        ids2 = torch.empty(429, 2, 3, dtype=torch.int32, device="cuda")
        out = ops.sparse_attention(q32, k32, k32, ids2, cu, bounds, 4, 0.3)
        assert out[2].shape == (429, 4) and out[2].dtype == torch.float64 and out[3].numel() == 0
