"""bench.py's output contract on CPU: the reference arm (the reference's own
CPU kernels, oracle/_ref) prints exactly one JSON line with the keys the
driver reads, alone and under torchrun with two ranks (rank 0 prints, the
other rank exits 0 without output)."""

from __future__ import annotations

import json
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
        "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _ref_built() -> bool:
    return (ROOT / "oracle" / "_ref" / "libds3ref.so").exists() or (ROOT / "oracle" / "libds3oracle.so").exists()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _check(line: dict, n: int) -> None:
    assert KEYS <= set(line), KEYS - set(line)
    assert line["impl"] == "reference" and line["n_gpus"] == n and line["unit"] == "tokens/s"
    assert line["value"] > 0 and line["higher_is_better"] is True and line["scaling"] == "weak"
    assert line["config"]["workload"] == "fused_layer_T512"
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"]["value"] == line["value"] and line["e2e"]["h2d_bytes_per_step"] == 0


@pytest.fixture(scope="module", autouse=True)
def oracles():
    import oracle

    oracle.build()
    if not _ref_built():
        pytest.skip("no CPU implementation built")


def test_reference_arm_prints_one_json_line():
    res = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "2", "--warmup", "3"],
                         cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, res.stdout
    _check(json.loads(lines[0]), 1)


def test_reference_arm_under_torchrun_two_ranks():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", str(_free_port()), "bench.py", "--impl", "reference", "--gpus", "2",
           "--steps", "2", "--warmup", "3"]
    res = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [l for l in res.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, res.stdout
    _check(json.loads(lines[0]), 2)
