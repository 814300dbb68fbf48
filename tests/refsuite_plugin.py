"""pytest plugin: run the reference's own test suite, unchanged, against this library.

The reference (yeyeyeping/msa_triton) tests its operators through the package
paths ``msa_triton.triton.{index_score,topk,k2q,sparse_attention}`` and picks
the device from ``MSA_TEST_DEVICE`` (tests/test_triton_attention.py:15-24). Its
comparators are its own dense eager ops (``msa_triton.eager``) and its FP64
oracle (``msa_triton.tests.reference_fp64``). This plugin builds the
``msa_triton`` package so that

* ``msa_triton.triton`` and its four operator modules ARE this library's
  modules (``msa_triton_b200``, ``msa_triton_b200.index_score`` ...), so the
  suite calls the CUDA kernels, and its monkeypatch of
  ``msa_triton.triton.k2q.build_k2q_csr`` (test_triton_attention.py:277-286)
  patches the attribute this library's backward looks up;
* everything else (``eager/``, ``layout.py``, ``tests/``) comes from a
  reference checkout, read in place and never modified.

Usage, on a machine with a CUDA device and a reference checkout::

    MSA_TEST_DEVICE=cuda MSA_REFERENCE_ROOT=/path/to/msa_triton \\
        python -m pytest -p tests.refsuite_plugin -p no:cacheprovider \\
        --rootdir "$MSA_REFERENCE_ROOT" -c /dev/null "$MSA_REFERENCE_ROOT/tests"

(run from this repository's root so that ``tests.refsuite_plugin`` and
``msa_triton_b200`` import). One file is not collected:
``tests/test_index_addressing.py`` launches a Triton probe kernel on the
reference's Triton helper ``triton/_addressing.py``, which this library has no
counterpart of; its subject (64-bit element offsets beyond 2^31) is covered by
``tests/test_gpu_fast_path.py::test_offsets_beyond_two_to_the_31_elements``.
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

NOT_COLLECTED = {"test_index_addressing.py": "Triton probe kernel of triton/_addressing.py (no counterpart here)"}


def _install(root: str) -> None:
    import msa_triton_b200 as lib
    from msa_triton_b200 import index_score, k2q, sparse_attention, topk

    pkg = types.ModuleType("msa_triton")
    pkg.__path__ = [root]  # eager/, layout.py, tests/ resolve inside the checkout
    pkg.__file__ = os.path.join(root, "__init__.py")
    sys.modules["msa_triton"] = pkg
    ops = types.ModuleType("msa_triton.triton")
    ops.__path__ = []  # a package whose submodules are all pre-registered below
    ops.__doc__ = "msa_triton_b200 under the reference's import path"
    for name in ("m3_index_score", "m3_topk", "m3_sparse_attention"):
        setattr(ops, name, getattr(lib, name))
    ops.__all__ = ["m3_index_score", "m3_topk", "m3_sparse_attention"]
    for name, mod in (("index_score", index_score), ("topk", topk), ("k2q", k2q),
                      ("sparse_attention", sparse_attention)):
        sys.modules[f"msa_triton.triton.{name}"] = mod
        setattr(ops, name, mod)
    sys.modules["msa_triton.triton"] = ops
    pkg.triton = ops


def pytest_configure(config):
    root = os.environ.get("MSA_REFERENCE_ROOT")
    if not root or not os.path.isdir(os.path.join(root, "tests")):
        raise SystemExit("refsuite_plugin: set MSA_REFERENCE_ROOT to a reference checkout (with tests/)")
    _install(os.path.abspath(root))
    config.addinivalue_line("markers", "strict_accuracy: numerical diagnostics against the strict FP64 oracle")
    config.addinivalue_line("markers", "npu: requires a physical Ascend NPU")


def pytest_ignore_collect(collection_path, config):
    return collection_path.name in NOT_COLLECTED or None


def pytest_report_header(config):
    return [f"refsuite: msa_triton.triton -> msa_triton_b200; not collected: {NOT_COLLECTED}"]
