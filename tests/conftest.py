"""Shared pytest setup.

Markers: ``gpu`` — needs a B200 (sm_100a) and the built libds3cuda.so; the
CPU suite runs with ``-m "not gpu"``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"

# Tolerances for fp32 outputs (1e-5 relative, 1e-6 absolute).
RTOL, ATOL = 1e-5, 1e-6


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built CUDA library")


def assert_close(got, want, rtol=RTOL, atol=ATOL, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    err = np.abs(got - want)
    lim = atol + rtol * np.abs(want)
    bad = err > lim
    if bad.any():
        i = np.unravel_index(np.argmax(err - lim), err.shape)
        raise AssertionError(f"{what}: {bad.sum()} of {bad.size} outside tol (rtol={rtol}, atol={atol}); "
                             f"worst at {i}: got {got[i]!r} want {want[i]!r}")


def assert_bitexact(got, want, what=""):
    got = np.ascontiguousarray(got)
    want = np.ascontiguousarray(want)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    if got.dtype == np.float32:
        eq = got.view(np.uint32) == want.view(np.uint32)
    else:
        eq = got == want
    if not eq.all():
        i = np.unravel_index(np.argmin(eq), eq.shape)
        raise AssertionError(f"{what}: {(~eq).sum()} of {eq.size} differ; first at {i}: got {got[i]!r} "
                             f"want {want[i]!r}")


def load_golden(name: str):
    with np.load(GOLDEN / name) as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def port():
    import oracle

    return oracle.port()


@pytest.fixture(scope="session")
def ds3():
    """The initialised CUDA backend (GPU tests only). Fails loudly when the
    library or the device is missing: there is no fallback."""
    from qw3_b200 import build, ds3 as d

    build.build()
    rc = d.init()
    if rc != 0:
        pytest.fail("ds3_cuda_init failed: " + d.last_error())
    yield d
