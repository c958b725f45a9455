"""Shared pytest configuration.

Markers: ``gpu`` tests need a CUDA device (B200, sm_100a) and the built native
library; everything else runs on a CPU-only host.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the native library")


def golden_cases():
    return json.loads((GOLDEN / "manifest.json").read_text())


def load_golden(case: str):
    d = np.load(GOLDEN / f"{case}.npz")
    return d["x"].astype(np.float64), d["expected"].astype(np.float64)


@pytest.fixture(scope="session")
def fixture_dir(tmp_path_factory):
    return tmp_path_factory.mktemp("onnx_fixtures")


@pytest.fixture(scope="session")
def device():
    return int(os.environ.get("ARTHIP_DEVICE", "0"))
