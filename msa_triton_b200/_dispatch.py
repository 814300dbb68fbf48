"""Internal kernel-family choice (no user-visible backend switch).

Shapes on the tensor-core path (bf16/f16, head dims and block size the tcgen05
kernels are specialised for) use it; everything else uses the float64 precise
kernels. ``precise_only()`` is an internal context manager the tests use to
compare the two families on the same inputs.
"""

from __future__ import annotations

import contextlib
import threading

import torch

_state = threading.local()


def _forced_precise() -> bool:
    return getattr(_state, "precise", False)


@contextlib.contextmanager
def precise_only():
    prev = _forced_precise()
    _state.precise = True
    try:
        yield
    finally:
        _state.precise = prev


# The last tensor-core forward workspace (with total tokens, query heads and CSR rows)
# and backward workspace, kept only under keep_fwd_workspace().
last_fwd_workspace = None
last_bwd_workspace = None


def keep_workspace() -> bool:
    """Tests keep the tensor-core forward's workspace to read its error word."""
    return getattr(_state, "keep_ws", False)


@contextlib.contextmanager
def keep_fwd_workspace():
    prev = keep_workspace()
    _state.keep_ws = True
    try:
        yield
    finally:
        _state.keep_ws = prev


TC_DTYPES = (torch.bfloat16, torch.float16)


def score_uses_tc(index_q: torch.Tensor, block_size: int) -> bool:
    from . import _lib
    return (not _forced_precise() and _lib.HAS_TC_SCORE and index_q.dtype in TC_DTYPES
            and index_q.shape[2] in (64, 128) and block_size == 128 and index_q.shape[1] in (1, 2, 4, 8, 16, 32, 64, 128))


def attention_uses_tc(q: torch.Tensor, k: torch.Tensor, block_size: int) -> bool:
    from . import _lib
    ratio = q.shape[1] // k.shape[1]
    return (not _forced_precise() and _lib.HAS_TC_ATTENTION and q.dtype in TC_DTYPES
            and q.shape[2] == 128 and block_size == 128 and ratio in (4, 8, 16) and q.shape[1] >= 8)
