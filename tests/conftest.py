"""Shared fixtures: the `gpu` marker, golden-vector loading, native builds."""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def golden_manifest() -> dict:
    return json.loads((GOLDEN / "MANIFEST.json").read_text())


def golden_cases() -> list[dict]:
    return golden_manifest()["cases"]


def load_golden(case: dict) -> dict[str, np.ndarray]:
    with np.load(GOLDEN / case["file"]) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def native_lib():
    """The product library, built in-tree if missing or stale."""
    from pathtile_b200 import _lib, build

    build.build()
    return _lib.load()


@pytest.fixture(scope="session")
def cuda_device(native_lib):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"GPU tests need compute capability 10.0, found {major}.{minor}")
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    return torch.device("cuda", 0)
