"""Test configuration: import paths, the ``gpu`` marker and shared fixtures.

``-m "not gpu"`` runs on any machine (oracle vs golden vectors, host logic,
the C-ABI library's exports).  ``-m gpu`` needs a CUDA device and the built
``libie_tpq.so``; those tests are the parity tests proper.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO, REPO / "inference-engine_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU and the built libie_tpq.so")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device visible")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    with np.load(GOLDEN / "golden_small.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden_hashes():
    import json

    return json.loads((GOLDEN / "golden_hashes.json").read_text())
