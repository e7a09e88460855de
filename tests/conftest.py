"""Shared pytest setup: repo root on sys.path, the ``gpu`` marker, helpers."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def golden_cases():
    """Names of the seeded operator fixtures made from the reference."""
    skip = {"key_dtype", "cache_sequence"}
    return sorted(p.stem for p in GOLDEN.glob("*.npz") if p.stem not in skip)


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def payload_code(case: dict) -> str:
    return {"float32": "f32", "bfloat16": "bf16", "float16": "f16", "float64": "f64"}[str(case["dtype"])]


def payload_as_float64(case: dict) -> np.ndarray:
    """Payload values as float64 (bf16 bits widened exactly)."""
    p = case["payload"]
    code = payload_code(case)
    if code == "bf16":
        return (p.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    if code == "f16":
        return p.view(np.float16).astype(np.float64)
    return p.astype(np.float64)


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    oracle.build()
    return oracle
