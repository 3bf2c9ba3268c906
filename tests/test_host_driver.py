"""The C host driver (qw3_b200/host/ds3_chunk_pre.c) replays the engine's
chunk-prefill call sequence through include/ds3_cuda.h. On CPU it must build
and skip with the reference tests' exit code 77; on a GPU its fused outputs
must match the oracle and agree with the engine-order sequence."""

from __future__ import annotations

import subprocess

import numpy as np
import pytest

from conftest import assert_bitexact, assert_close
from qw3_b200 import build

H, NQ, NK, HD, E, K = 2048, 32, 4, 128, 128, 8


def driver():
    build.build()
    return build.build_host()


def test_driver_builds_and_skips_without_gpu(tmp_path):
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    res = subprocess.run([str(driver()), str(tmp_path / "o.bin"), "8"], capture_output=True, text=True)
    assert res.returncode == 77, res.stderr


def parse(path):
    raw = open(path, "rb").read()
    hdr = np.frombuffer(raw[:16], np.int32)
    assert hdr[0] == 0x33534433
    M, V, seq_pos = int(hdr[1]), int(hdr[2]), int(hdr[3])
    off = 16
    out = {}

    def take(name, dtype, count, shape):
        nonlocal off
        n = np.dtype(dtype).itemsize * count
        out[name] = np.frombuffer(raw[off:off + n], dtype).reshape(shape).copy()
        off += n

    take("table", np.uint8, V * 1152, (V, 1152))
    take("ids", np.int32, M, (M,))
    take("w", np.float32, 2 * H, (2, H))
    take("hw", np.float32, 2 * HD, (2, HD))
    take("q", np.float32, M * NQ * HD, (M, NQ, HD))
    take("k", np.float32, M * NK * HD, (M, NK, HD))
    take("a", np.float32, M * H, (M, H))
    take("logits", np.float32, M * E, (M, E))
    take("resid", np.float32, M * H, (M, H))
    take("norm", np.float32, M * H, (M, H))
    take("q_out", np.float32, M * NQ * HD, (M, NQ, HD))
    take("k_out", np.float32, M * NK * HD, (M, NK, HD))
    take("idx", np.int32, M * K, (M, K))
    take("scores", np.float32, M * K, (M, K))
    assert off == len(raw)
    return M, V, seq_pos, out


@pytest.mark.gpu
@pytest.mark.parametrize("M,seq_pos", [(64, 0), (17, 4000)])
def test_driver_matches_oracle(tmp_path, port, M, seq_pos):
    f = tmp_path / "o.bin"
    res = subprocess.run([str(driver()), str(f), str(M), str(seq_pos)], capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "agree" in res.stdout
    M, V, seq_pos, d = parse(f)
    _, hid, _ = port.embed_rms_norm(d["table"], 12, 1152, V, d["ids"], H, d["w"][0], 1e-6)
    s, n = port.add_rms_norm(d["a"], hid, d["w"][1], 1e-6)
    assert_bitexact(d["resid"], s, "residual")
    assert_close(d["norm"], n, what="ffn norm")
    pos = np.arange(seq_pos, seq_pos + M, dtype=np.int32)
    qo, ko = port.qk_norm_rope(d["q"], d["k"], d["hw"][0], d["hw"][1], pos, 1e6, 1e-6)
    assert_close(d["q_out"], qo, what="q")
    assert_close(d["k_out"], ko, what="k")
    _, idx, sc = port.router(d["logits"], K, True)
    assert_bitexact(d["idx"], idx, "top-8")
    assert_close(d["scores"], sc, what="scores")
