"""Test bootstrap: in-tree imports, the ``gpu`` marker and golden-vector loading."""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built library")


def load_golden(name: str) -> dict:
    """Arrays of one golden case plus its decoded ``meta`` dict."""
    with np.load(GOLDEN / f"{name}.npz") as data:
        case = {k: data[k] for k in data.files}
    case["meta"] = json.loads(str(case["meta"]))
    return case


def golden_names(prefix: str) -> list[str]:
    return sorted(p.stem for p in GOLDEN.glob(f"{prefix}*.npz"))


@pytest.fixture(scope="session")
def cuda_device():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
