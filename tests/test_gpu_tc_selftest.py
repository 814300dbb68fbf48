"""Pins the tcgen05 building blocks (TMA 128-byte-swizzle loads, K-major and
MN-major UMMA shared-memory descriptors, instruction descriptor, TMEM
allocation and loads) against torch.matmul before the kernels built on them
are trusted."""

import pytest
import torch

from msa_triton_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("k", [64, 128])
@pytest.mark.parametrize("layout", range(8))
def test_umma_tile_matches_torch(dtype, k, layout, cuda_device):
    """layout bit 0: B stored [K][N] (MN-major); bit 1: A stored [K][M]
    (MN-major); bit 2: 64-column tiles (N = 64 per instruction)."""
    gen = torch.Generator().manual_seed(k + layout)
    mt, nt = 2, 3
    nw = 64 if layout & 4 else 128
    m, n = 128 * mt, nw * nt
    a_logical = torch.randn(m, k, generator=gen).to(dtype)
    b_logical = torch.randn(k, n, generator=gen).to(dtype)
    a = a_logical.T.contiguous() if layout & 2 else a_logical
    b = b_logical if layout & 1 else b_logical.T.contiguous()
    want = (a_logical.float() @ b_logical.float()).to(cuda_device)
    a, b = a.to(cuda_device), b.to(cuda_device)
    c = torch.full((m, n), float("nan"), device=cuda_device)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    _lib.call("msa_selftest_umma", _lib.ptr(a), _lib.ptr(b), _lib.DTYPE_CODE[dtype], mt, nt, k, layout,
              _lib.ptr(c), _lib.ptr(err), _lib.stream_of(a))
    torch.cuda.synchronize()
    assert err.item() == 0
    torch.testing.assert_close(c, want, atol=1e-3, rtol=1e-3)
