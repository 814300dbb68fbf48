"""Shared test configuration.

``-m gpu`` tests need a CUDA device and the in-tree CUDA library; everything
else runs on the CPU (oracle pinning, host validation, C-ABI exports, gloo
multi-process sharding logic).
"""

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built CUDA library")
    config.addinivalue_line("markers", "slow: long-running CPU test")


@pytest.fixture(scope="session")
def golden():
    import json
    import numpy as np

    here = REPO / "tests" / "golden"
    manifest = json.loads((here / "manifest.json").read_text())

    class Golden:
        def __init__(self):
            self.manifest = manifest
            self._cache = {}

        def stage(self, name):
            if name not in self._cache:
                self._cache[name] = dict(np.load(here / f"{name}.npz"))
            return self._cache[name]

        def cases(self, stage):
            return manifest[stage]

    return Golden()


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    return torch.device("cuda", 0)
