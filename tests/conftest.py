"""Shared test set-up: import paths, the ``gpu`` marker, golden fixtures."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_ROOT = REPO / "qsa-fp8-sm89_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(REPO), str(PKG_ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN_CASES = sorted(p.stem for p in GOLDEN.glob("*.npz"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run with -m gpu")


def load_golden(name: str) -> dict:
    z = np.load(GOLDEN / f"{name}.npz")
    return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden():
    return {name: load_golden(name) for name in GOLDEN_CASES}


def fp32_floor(z: dict) -> float:
    """Absolute error floor of an fp32 evaluation of a fixture's softmax
    average: K accumulated terms of at most max|V| * v_scale each, one fp32
    rounding (2^-24) apiece (at least 1e-6). The reference's own torch_eager
    and reference() disagree by about that where the output cancels to near
    zero, as in the dynamic-range case."""
    from oracle import qsa_oracle as O

    vmax = float(np.nanmax(np.abs(O.e4m3fn_table()[z["v"]]))) * float(z["v_scale"])
    return max(1e-6, z["indices"].shape[1] * 2.0 ** -24 * vmax)


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    """Spacing of bf16 numbers around |x| (2^(floor(log2|x|) - 7))."""
    a = np.abs(np.asarray(x, dtype=np.float64))
    e = np.floor(np.log2(np.where(a > 0, a, 1.0)))
    return np.where(a > 0, 2.0 ** (e - 7), 2.0 ** -133)
