"""pytest configuration: the ``gpu`` marker and shared fixture loaders."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def load_golden(name: str) -> dict:
    """Load ``tests/golden/<name>.npz``; bf16 bit patterns become float32 values,
    fp16 arrays become float32, other arrays are returned as stored."""
    from oracle.svdq_oracle import bits_to_bf16

    raw = np.load(os.path.join(GOLDEN, name + ".npz"))
    out = {}
    for key in raw.files:
        v = raw[key]
        if key.endswith("__bf16"):
            out[key[: -len("__bf16")]] = bits_to_bf16(v)
            out[key[: -len("__bf16")] + "__bits"] = v
        elif key.endswith("__fp16"):
            out[key[: -len("__fp16")]] = v.astype(np.float32)
            out[key[: -len("__fp16")] + "__fp16raw"] = v
        else:
            out[key] = v
    return out


@pytest.fixture
def golden():
    return load_golden
