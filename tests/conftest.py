from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built libima_b200.so")


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as z:
        return {k: z[k] for k in z.files}


def golden_cases(data: dict) -> dict[str, dict]:
    """Group 'case/field' keys of a fixture into {case: {field: array}}."""
    out: dict[str, dict] = {}
    for key, val in data.items():
        if "/" in key:
            case, field = key.split("/", 1)
            out.setdefault(case, {})[field] = val
    return out


def json_field(arr) -> dict:
    return json.loads(str(arr))


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU tests need CUDA (run them with -m gpu on a B200)")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"libima_b200.so is built for sm_100a only; found sm_{major}{minor}")
    return torch.device("cuda", 0)
