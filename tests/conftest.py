"""Shared test setup: import paths, the ``gpu`` marker, seeded inputs.

``-m "not gpu"`` tests run on any machine (oracle vs golden fixtures, host-side
validation, the C-ABI library's exports, gloo multi-process logic).
``-m gpu`` tests call the sm_100a kernels through the C ABI and compare them
with the CPU oracle in oracle/attention_oracle.py.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "tpu-native-pallas-flashattention_b200"
for p in (str(PKG), str(ROOT), str(ROOT / "tests" / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built library")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        have_gpu = False
    if have_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def randn(shape, seed, dtype=np.float32):
    """Seeded N(0, 1) numpy array (the stand-in for jax.random.normal inputs)."""
    return np.random.default_rng(seed).standard_normal(shape).astype(dtype)


@pytest.fixture(scope="session")
def golden():
    data = np.load(ROOT / "tests" / "golden" / "attention_cases.npz")
    cases = {}
    for key in data.files:
        name, field = key.split("/")
        cases.setdefault(name, {})[field] = data[key]
    return cases


def to_dev(x, dtype=None):
    """numpy -> CUDA tensor (optionally cast, e.g. to torch.bfloat16)."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    return t.to(dtype) if dtype is not None else t


def to_np(t):
    """CUDA tensor -> float64 numpy (bf16/f16 widened exactly)."""
    import torch
    return t.detach().to(torch.float64).cpu().numpy()


def widen(t):
    """Exact float32 values of a (possibly bf16) tensor as numpy, for the oracle."""
    import torch
    return t.detach().to(torch.float32).cpu().numpy()


def rel_err(a, b):
    """max|a-b| / max|b| -- the reference's gradient metric (tests/test_backward.py:25-26)."""
    return float(np.max(np.abs(a - b)) / (np.max(np.abs(b)) + 1e-9))


@pytest.fixture(scope="session")
def ref_golden():
    """Outputs of the reference's own source (tests/golden/make_reference_golden.py).

    Keys are ``group/case/field``; inputs are rebuilt with ``golden_inputs``."""
    data = np.load(ROOT / "tests" / "golden" / "reference_golden.npz")
    return {k: data[k] for k in data.files}


def bf16_bits_to_f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)
