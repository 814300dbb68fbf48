"""CPU checks of the C ABI boundary: the library loads and exports every
entry point that include/msa_b200.h declares, and the ctypes binding covers
them all. No kernel is launched."""

import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for header in (REPO / "include").glob("*.h"):
        text = header.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(msa_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "msa_attn_fwd" in names and "msa_k2q_build" in names and "msa_topk" in names


def test_library_exports_every_declared_symbol():
    from msa_triton_b200 import _lib

    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built (python -m msa_triton_b200.build)")
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    assert set(declared_symbols()) <= set(_lib.exported_symbols()), "ctypes binding misses a declared symbol"
    assert lib.msa_version().decode().startswith("msa_b200")


def test_bad_arguments_return_status_without_gpu():
    """Argument checks run before any CUDA call, so they work on a CPU host."""
    from msa_triton_b200 import _lib

    if not _lib.LIB_PATH.exists():
        pytest.skip("library not built")
    with pytest.raises(_lib.MsaError, match="bad dtype"):
        _lib.call("msa_attn_fwd", None, None, None, 7, None, None, 1, 0, 4, 2, 16, 1, 4, 1.0, None, None, None, None)
    with pytest.raises(_lib.MsaError, match="edge capacity"):
        import ctypes
        host = (ctypes.c_int32 * 2)(0, 1)
        _lib.call("msa_k2q_build", None, None, host, None, 1, 2**20, 64, 2**12, 1, None, None, None, None, 0, None)
