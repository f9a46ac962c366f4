"""Shared fixtures. Tests marked ``gpu`` need a CUDA device (B200); the rest run on CPU."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (run with -m gpu on a B200)")


def load_golden(name: str) -> dict:
    return json.loads((GOLDEN / name).read_text())


_NP_BITS = {"f32": np.uint32, "f16": np.uint16, "bf16": np.uint16, "f64": np.uint64}
_NP_VIEW = {"f32": np.float32, "f16": np.float16, "f64": np.float64}


def golden_values(bits, dtype: str) -> np.ndarray:
    """Golden rows are raw bit patterns; bf16 stays as uint16 bits, others become floats."""
    arr = np.asarray(bits, dtype=_NP_BITS[dtype])
    return arr if dtype == "bf16" else arr.view(_NP_VIEW[dtype])


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle

    return oracle.load()


@pytest.fixture(scope="session")
def cuda_lib():
    """Build (if needed) and load libonyx_b200.so."""
    from onyx_b200 import _lib, build_lib

    build_lib.build()
    return _lib.load()
