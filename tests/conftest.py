"""Shared pytest configuration for the KV-restore suite.

* ``gpu`` marks tests that need a CUDA device (run with ``-m gpu``); everything
  else runs on a CPU-only machine (``-m "not gpu"``).
* ``golden`` loads the committed fixtures produced by tests/golden/make_golden.py.
* ``scb`` imports the product package (directory ``intelligent-bell_b200``).
"""

from __future__ import annotations

import importlib
import os
import sys

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN_PATH = os.path.join(REPO, "tests", "golden", "golden_path1.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_package():
    """Import the product package from its (hyphenated) directory name."""
    return importlib.import_module("intelligent-bell_b200")


def load_oracle():
    """Import the CPU oracle (test infrastructure only)."""
    return importlib.import_module("oracle.speccache_oracle")


_DT = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}


def as_tensor(arr: np.ndarray, dtype: str | torch.dtype | None = None) -> torch.Tensor:
    """Decode a fixture array; 16-bit float patterns are stored as uint16."""
    if isinstance(dtype, str):
        dtype = _DT[dtype]
    if arr.dtype == np.uint16:
        t = torch.from_numpy(arr.astype(np.int16).copy())
        return t.view(dtype if dtype is not None else torch.float16)
    return torch.from_numpy(np.ascontiguousarray(arr)).clone()


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN_PATH, allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def oracle():
    return load_oracle()


@pytest.fixture(scope="session")
def scb():
    return load_package()


def bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    """Bitwise equality (treats +0/-0 as different, NaN patterns as equal)."""
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    a = a.contiguous().cpu()
    b = b.contiguous().cpu()
    if a.dtype in (torch.float16, torch.bfloat16):
        return torch.equal(a.view(torch.int16), b.view(torch.int16))
    if a.dtype == torch.float32:
        return torch.equal(a.view(torch.int32), b.view(torch.int32))
    return torch.equal(a, b)
