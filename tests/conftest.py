"""Shared fixtures.  `gpu` tests need a CUDA device and libnxv_b200.so; the
rest run on CPU (the oracle, host-side logic, the C-ABI symbol table)."""
import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = json.loads((ROOT / "tests" / "golden" / "reference_kats.json").read_text())


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    return GOLDEN


@pytest.fixture(scope="session")
def orc():
    from oracle import binding
    binding.lib()
    return binding


@pytest.fixture(scope="session")
def nxv():
    """The Nx.Vulkan mirror on the GPU; fails (not skips) without the library."""
    import torch
    if not torch.cuda.is_available():
        pytest.fail("gpu test collected on a machine without CUDA")
    from nx_vulkan_b200 import vulkan
    assert vulkan.init() == "ok"
    return vulkan


def rng(seed):
    return np.random.default_rng(seed)


def atoms_equal(got, want, tol):
    """Compare a decoded f32 list (with 'nan'/'infinity' atoms) to expectations."""
    assert len(got) == len(want)
    for g, w in zip(got, want):
        if isinstance(w, str):
            assert g == w, (got, want)
        elif tol == 0:
            assert g == w, (got, want)
        else:
            assert abs(g - w) <= tol, (got, want)
