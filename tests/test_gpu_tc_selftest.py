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
@pytest.mark.parametrize("b_mn_major", [0, 1])
def test_umma_tile_matches_torch(dtype, k, b_mn_major, cuda_device):
    gen = torch.Generator().manual_seed(k + b_mn_major)
    mt, nt = 2, 3
    a = torch.randn(128 * mt, k, generator=gen).to(dtype).to(cuda_device)
    if b_mn_major:
        b = torch.randn(k, 128 * nt, generator=gen).to(dtype).to(cuda_device)
        want = a.float() @ b.float()
    else:
        b = torch.randn(128 * nt, k, generator=gen).to(dtype).to(cuda_device)
        want = a.float() @ b.float().T
    c = torch.full((128 * mt, 128 * nt), float("nan"), device=cuda_device)
    err = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    _lib.call("msa_selftest_umma", _lib.ptr(a), _lib.ptr(b), _lib.DTYPE_CODE[dtype], mt, nt, k, b_mn_major,
              _lib.ptr(c), _lib.ptr(err), _lib.stream_of(a))
    torch.cuda.synchronize()
    assert err.item() == 0
    torch.testing.assert_close(c, want, atol=1e-3, rtol=1e-3)
