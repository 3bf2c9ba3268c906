"""bench.py's host-side helpers on CPU: the parity measures (bit-exactness,
tolerance ratio), the input-copy count that keeps every config out of L2,
and the config line both arms print."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_bitexact_compares_bits():
    a = np.array([0.0, 1.0, np.nan], np.float32)
    assert bench.bitexact(a, a.copy())
    b = a.copy()
    b[0] = -0.0  # equal as floats, different bits
    assert not bench.bitexact(a, b)
    assert not bench.bitexact(a, a[:2])


def test_tol_ratio_is_error_over_tolerance():
    want = np.ones((3000, 4), np.float32)
    got = want.copy()
    assert bench.tol_ratio(got, want) == 0.0
    got[2999, 3] += np.float32(5.5e-6)  # 1e-6 + 1e-5 * 1 = 1.1e-5 allowed
    r = bench.tol_ratio(got, want)
    assert 0.45 < r < 0.55
    got[0, 0] += np.float32(2.2e-5)
    assert bench.tol_ratio(got, want) > 1.0


def test_parity_ok_reads_flags_and_ratios():
    assert bench.parity_ok({"a_bitexact": True, "b_tol_ratio": 0.9})
    assert not bench.parity_ok({"a_bitexact": True, "b_tol_ratio": 1.2})
    assert not bench.parity_ok({"a_bitexact": False, "b_tol_ratio": 0.1})


def test_n_copies_exceeds_l2_at_every_size():
    for nbytes in (1, 10_000_000, 75_000_000, 126_000_000, 1_073_741_824):
        n = bench.n_copies(nbytes)
        assert n >= 2 and n * nbytes >= 320_000_000 or (nbytes >= 320_000_000 and n == 2)
    assert bench.n_copies(700_000_000, lo=1) == 1


def test_both_arms_print_the_same_config():
    c1, c8 = bench.config_line(1), bench.config_line(8)
    assert c1["workload"] == "fused_layer_T512" and c8["global_tokens"] == 8 * bench.T
    assert "l2" in c1 and set(c1) == set(c8)


def test_step_bytes_match_the_per_token_figures():
    # embed + norm, QK-norm + RoPE, add + norm, router, 8 SwiGLU rows, combine (8 expert rows, the
    # residual, 8 weights, the output)
    per_token = 17_540 + 36_868 + 32_768 + 576 + 8 * 9_220 + 81_952
    assert bench.STEP_BYTES == bench.T * per_token == 124_653_568
