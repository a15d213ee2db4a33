"""Shared test setup: the `gpu` marker, repository imports and golden data."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    # GPU tests fail loudly on a machine without a GPU unless deselected with -m "not gpu"
    pass


@pytest.fixture(scope="session")
def validation_vectors():
    return json.loads((GOLDEN / "validation_vectors.json").read_text())


@pytest.fixture(scope="session")
def descriptor_grid():
    return json.loads((GOLDEN / "descriptors.json").read_text())


@pytest.fixture(scope="session")
def sparse_records():
    return json.loads((GOLDEN / "sparse_active.json").read_text())


@pytest.fixture(scope="session")
def golden_paths():
    index = json.loads((GOLDEN / "paths.json").read_text())
    arrays = dict(np.load(GOLDEN / "paths.npz"))
    return index, arrays


def full_desc(desc: dict) -> dict:
    out = dict(a_format="tf32", b_format=None, d_type="f32", saturate=False, scaling=None, scale_vec=None, kind=None)
    out.update({k: v for k, v in desc.items() if k in out})
    return out
