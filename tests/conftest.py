"""Shared pytest configuration: the ``gpu`` marker and golden-fixture helpers."""
from __future__ import annotations

import hashlib
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
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def det_bytes(seed: str, n: int) -> bytes:
    """Same SHA-256 counter stream as tests/golden/make_golden.py."""
    out = bytearray()
    counter = 0
    while len(out) < n:
        out += hashlib.sha256(f"{seed}:{counter}".encode()).digest()
        counter += 1
    return bytes(out[:n])


@pytest.fixture(scope="session")
def gcm_kat():
    return json.loads((GOLDEN / "gcm_kat.json").read_text())


@pytest.fixture(scope="session")
def golden_records():
    return json.loads((GOLDEN / "records.json").read_text())


def load_codec(heads: int):
    with np.load(GOLDEN / f"codec_h{heads}.npz") as data:
        return {k: data[k] for k in data.files}
