"""ctypes binding of the C ABI declared in include/msa_b200.h.

The CUDA library is loaded from the package directory (``libmsa_b200.so``,
built by ``python -m msa_triton_b200.build``). There is no fallback: if the
library is missing or a launch fails, the calling op raises.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import c_double, c_float, c_int, c_int32, c_int64, c_size_t, c_void_p
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libmsa_b200.so"

DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

_P = c_void_p
_SIGNATURES = {
    "msa_version": ([], ctypes.c_char_p),
    "msa_last_error": ([], ctypes.c_char_p),
    "msa_kernel_launches": ([], ctypes.c_uint64),
    "msa_timing_enable": ([c_int], c_int),
    "msa_timing_read": ([ctypes.c_char_p, _P, _P], c_int),
    "msa_index_score_fwd": ([_P, _P, c_int, _P, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32, c_double,
                             _P, _P, _P, _P], c_int),
    "msa_index_score_bwd": ([_P, _P, c_int, _P, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32, c_double,
                             _P, _P, _P, _P, _P, _P], c_int),
    "msa_index_score_fwd_tc": ([_P, _P, c_int, _P, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32, c_float,
                                c_int64, c_int64, _P, _P], c_int),
    "msa_topk": ([_P, _P, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32, _P, _P], c_int),
    "msa_k2q_workspace_size": ([_P, c_int32, c_int32, c_int32], c_size_t),
    "msa_k2q_build": ([_P, _P, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32, _P, _P, _P, _P, c_size_t, _P],
                      c_int),
    "msa_k2q_build_noalloc": ([_P, _P, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32, _P, _P, _P, _P], c_int),
    "msa_attn_fwd": ([_P, _P, _P, c_int, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32,
                      c_double, _P, _P, _P, _P], c_int),
    "msa_attn_fwd_tc_workspace_size": ([c_int64, c_int32, c_int32, c_int32, c_int32], c_size_t),
    "msa_attn_fwd_tc": ([_P, _P, _P, c_int, _P, _P, _P, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32,
                         c_int32, c_double, c_int32, _P, _P, _P, c_size_t, _P], c_int),
    "msa_attn_fwd_tc_range": ([_P, _P, _P, c_int, _P, _P, _P, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32,
                               c_int32, c_int32, c_double, c_int32, c_int64, c_int64, _P, _P, _P, c_size_t, _P], c_int),
    "msa_attn_bwd_tc_range": ([_P, _P, _P, _P, _P, _P, c_int, _P, _P, _P, _P, c_int32, c_int64, c_int32, c_int32,
                               c_int32, c_int32, c_int32, c_double, c_int32, c_int64, c_int64, _P, _P, _P, c_int, _P,
                               c_size_t, _P], c_int),
    "msa_attn_fwd_tc_error": ([_P, c_int64, c_int32, c_int32, _P], c_int),
    "msa_attn_fwd_tc_rerun_counts": ([_P, c_int64, c_int32, c_int32, _P, _P], c_int),
    "msa_attn_bwd_tc_workspace_size": ([c_int64, c_int32, c_int32, c_int32, c_int32], c_size_t),
    "msa_attn_bwd_tc": ([_P, _P, _P, _P, _P, _P, c_int, _P, _P, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32,
                         c_int32, c_int32, c_double, c_int32, _P, _P, _P, c_int, _P, c_size_t, _P], c_int),
    "msa_attn_bwd_tc_error": ([_P, _P], c_int),
    "msa_attn_bwd_q": ([_P, _P, _P, _P, c_int, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32,
                        c_int32, c_double, _P, _P, _P, _P], c_int),
    "msa_attn_bwd_kv": ([_P, _P, _P, _P, c_int, _P, _P, _P, _P, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32,
                         c_int32, c_int32, c_double, _P, _P, _P, _P, _P], c_int),
    "msa_selftest_umma": ([_P, _P, c_int, c_int32, c_int32, c_int32, c_int32, _P, _P, _P], c_int),
    "msa_read_i32": ([_P, c_int64, _P, _P], c_int),
    "msa_index_score_state_workspace_size": ([c_int64, c_int32], c_size_t),
    "msa_index_score_fwd_tc_state": ([_P, _P, c_int, _P, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32,
                                      c_float, _P, _P, _P, _P, c_size_t, _P], c_int),
    "msa_index_score_bwd_tc_workspace_size": ([c_int64, c_int32, c_int32, c_int32, c_int32], c_size_t),
    "msa_index_score_bwd_tc": ([_P, _P, c_int, _P, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32, c_double,
                                _P, _P, _P, _P, _P, _P, c_size_t, _P], c_int),
    "msa_block_prefix": ([_P, c_int32, c_int32, _P, _P], c_int),
    "msa_decode_index_score": ([_P, _P, c_int, _P, _P, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32,
                                c_int32, c_double, _P, _P], c_int),
    "msa_topk_positions": ([_P, _P, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32, _P, _P], c_int),
    "msa_decode_attn_workspace_size": ([c_int32, c_int32, c_int32, c_int32], c_size_t),
    "msa_decode_attn": ([_P, _P, _P, c_int, _P, _P, _P, c_int32, c_int32, c_int32, c_int32, c_int32, c_int32,
                         c_int32, c_int32, c_double, _P, _P, _P, c_size_t, _P], c_int),
    "msa_index_kl_teacher_tc_workspace_size": ([c_int64, c_int32, c_int32, c_int32, c_int32], c_size_t),
    "msa_index_kl_teacher_tc": ([_P, _P, c_int, _P, _P, _P, _P, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32,
                                 c_int32, c_int32, c_double, c_int32, _P, _P, c_size_t, _P], c_int),
    "msa_index_kl_logits_tc": ([_P, _P, c_int, _P, _P, _P, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32,
                                c_double, _P, _P], c_int),
    "msa_index_kl_student_tc": ([_P, _P, _P, _P, c_int32, c_int64, c_int32, c_int32, c_double, c_int, _P, _P,
                                 c_size_t, _P], c_int),
    "msa_index_kl_grad_tc_workspace_size": ([c_int64, c_int32, c_int32], c_size_t),
    "msa_index_kl_grad_tc": ([_P, _P, c_int, _P, _P, _P, _P, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32,
                              c_double, _P, _P, _P, _P, c_size_t, _P], c_int),
    "msa_index_kl_teacher": ([_P, _P, c_int, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32, c_int32,
                              c_double, _P, _P], c_int),
    "msa_index_kl_student_workspace_size": ([c_int64, c_int32], c_size_t),
    "msa_index_kl_student": ([_P, _P, c_int, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32, c_double,
                              _P, c_int, c_int, _P, _P, _P, c_size_t, _P], c_int),
    "msa_index_kl_dik_workspace_size": ([c_int64, c_int32, c_int32, c_int], c_size_t),
    "msa_index_kl_dik": ([_P, c_int, _P, _P, _P, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32,
                          c_int32, _P, c_int, _P, _P, c_size_t, _P], c_int),
    "msa_attn_bwd_atomic": ([_P, _P, _P, _P, c_int, _P, _P, c_int32, c_int64, c_int32, c_int32, c_int32, c_int32,
                             c_int32, c_double, _P, _P, _P, _P, _P, _P, _P], c_int),
}

_lock = threading.Lock()
_lib = None


def load():
    """Load the CUDA library once and declare every exported signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"msa_triton_b200: CUDA library {LIB_PATH.name} is not built; "
                    "run `python -m msa_triton_b200.build` (nvcc, sm_100a)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (args, res) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _lib = lib
    return _lib


def kernel_launches() -> int:
    """Kernels launched by the library so far in this process."""
    return int(load().msa_kernel_launches())


def timing_enable(on: bool) -> None:
    """Record device times of the tensor-core attention kernels (see kernel_time)."""
    call("msa_timing_enable", 1 if on else 0)


def kernel_time(name: str) -> tuple[float, int]:
    """(total ms, launches) of `name` recorded since the last read; waits for them."""
    total = ctypes.c_double(0.0)
    n = ctypes.c_int64(0)
    call("msa_timing_read", name.encode(), ctypes.byref(total), ctypes.byref(n))
    return total.value, n.value


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


class MsaError(RuntimeError):
    """A launch or argument check inside the CUDA library failed."""


def call(name: str, *args) -> None:
    lib = load()
    status = getattr(lib, name)(*args)
    if status != 0:
        msg = lib.msa_last_error().decode(errors="replace")
        raise MsaError(f"{name} failed (status {status}): {msg}")


def ptr(t: torch.Tensor | None):
    return None if t is None else c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def host_ints(t: torch.Tensor) -> list[int]:
    """Values of a small int32 tensor on the host. A CUDA tensor is read through
    msa_read_i32 (a kernel writes mapped pinned memory), so the read waits for
    the tensor's stream but never queues behind bulk copies on other streams;
    a host tensor is read directly."""
    if t.device.type != "cuda":
        return [int(x) for x in t.tolist()]
    src = t.detach().contiguous()
    n = src.numel()
    buf = (ctypes.c_int32 * max(n, 1))()
    with torch.cuda.device(src.device):
        call("msa_read_i32", ptr(src), n, buf, stream_of(src))
    return list(buf[:n])


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t.device.type != "cuda":
            raise RuntimeError("msa_triton_b200 runs on CUDA devices only (no CPU fallback)")
    if not torch.cuda.is_available():
        raise RuntimeError("msa_triton_b200 needs a CUDA device")

# Tensor-core kernel families compiled into this build (flipped on as they land).
HAS_TC_SCORE = True
HAS_TC_ATTENTION = True
