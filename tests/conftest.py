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


def codec_shapes() -> dict:
    return json.loads((GOLDEN / "codec_shapes.json").read_text())


def codec_shape_source(entry: dict) -> np.ndarray:
    """The bf16 source (uint16 bits [blocks, 128, heads, 128]) of a
    codec_shapes.json entry, regenerated from its seed exactly as
    tests/golden/make_golden.py draws it (numpy PCG64 normals, 1% outliers of
    +-8, round to nearest even), and checked against the stored digest."""
    g = np.random.default_rng(entry["seed"])
    shape = (entry["blocks"], 128, entry["heads"], 128)
    x = g.standard_normal(shape).astype(np.float32)
    if entry["outliers"]:
        mask = g.random(shape) < 0.01
        sign = np.where(g.random(shape) < 0.5, -1.0, 1.0).astype(np.float32)
        x = np.where(mask, 8.0 * sign, x).astype(np.float32)
    u = x.view(np.uint32)
    bits = ((u + ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)) >> np.uint32(16)).astype(np.uint16)
    assert hashlib.sha256(bits.tobytes()).hexdigest() == entry["source_sha256"], \
        "regenerated source differs from the fixture's (numpy draw changed?)"
    return bits


def sha256(data) -> str:
    return hashlib.sha256(np.ascontiguousarray(data).tobytes()).hexdigest()
