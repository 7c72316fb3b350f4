"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on CPU."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def built():
    """Build the CUDA library (nvcc cross-compiles without a GPU) and the oracle."""
    from edgecore_b200 import build
    from oracle import oracle
    build.build()
    oracle.build(reference=True)
    return True


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(GOLDEN / name)
    return load


@pytest.fixture(scope="session")
def tiny_models(tmp_path_factory, golden):
    """The seeded tiny models of the golden set, regenerated and hash-checked."""
    sys.path.insert(0, str(GOLDEN))
    from make_golden import TINY, sha256
    from edgecore_b200 import synth
    meta = json.loads((GOLDEN / "models.json").read_text())
    cache = tmp_path_factory.mktemp("models")
    paths = {}
    for key, spec in TINY.items():
        p = synth.ensure_model(spec, cache)
        assert sha256(p) == meta[key]["sha256"], f"synthetic model {key} drifted from the golden one"
        paths[key] = (spec, p)
    return paths


@pytest.fixture(scope="session")
def cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch
