"""Shared pytest setup: markers, import paths, synthetic model fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
for sub in ("project-ia_b200", "oracle"):
    p = str(ROOT / sub)
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN / "golden.npz")


@pytest.fixture(scope="session")
def tiny_path(tmp_path_factory):
    import qorus_b200 as Q
    cfg = Q.config(**Q.TINY)
    path = tmp_path_factory.mktemp("models") / "tiny.qorus"
    Q.write_model(str(path), cfg, seed=0, threads=1)
    return str(path)
