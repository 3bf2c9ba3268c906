"""GGUF v3 reader of the backend (include/ds3_cuda_gguf.h) against the
engine's reader (src/ds3_gguf.c): the unmodified reference compiled into
oracle/_ref when the sources are present, the committed golden table it
produced (tests/golden/gguf_ref_table.json), and the CPU restatement
oracle/gguf.py. Host code only: no GPU needed."""

from __future__ import annotations

import json
import struct
from pathlib import Path

import pytest

import oracle
from gguf_writer import ARRAY, F32, STRING, U32, GgufFile, synthetic_model
from oracle import gguf as OG
from qw3_b200 import build, ds3

GOLDEN = Path(__file__).resolve().parent / "golden" / "gguf_ref_table.json"


@pytest.fixture(scope="module", autouse=True)
def lib():
    build.build()
    return ds3.lib()


def mine(path) -> dict:
    with ds3.Gguf(path) as g:
        return {"version": g.version, "alignment": g.alignment, "data_offset": g.data_offset,
                "n_metadata": g.n_metadata, "tensors": g.tensors()}


def same_table(a: list[dict], b: list[dict], keys=("name", "n_dims", "ne", "type", "offset", "size")):
    assert len(a) == len(b)
    for x, y in zip(a, b):
        assert {k: x[k] for k in keys} == {k: y[k] for k in keys}, (x, y)


CONFIGS = [dict(), dict(alignment=64), dict(alignment=256, embd_type=14, norm_type=0),
           dict(norm_type=8, n_layer=3, seed=3), dict(alignment=8, n_embd=256, n_vocab=7, seed=5)]


@pytest.mark.parametrize("cfg", CONFIGS)
def test_table_matches_restatement_and_writer(tmp_path, cfg):
    g, _ = synthetic_model(**cfg)
    p = g.write(tmp_path / "m.gguf")
    got, want = mine(p), OG.parse(p.read_bytes())
    for k in ("version", "alignment", "data_offset", "n_metadata"):
        assert got[k] == want[k], k
    same_table(got["tensors"], want["tensors"], keys=("name", "n_dims", "ne", "nb", "type", "offset", "size"))
    same_table(got["tensors"], g.expected_table())


@pytest.mark.parametrize("cfg", CONFIGS)
def test_table_matches_reference_reader(tmp_path, cfg):
    g, _ = synthetic_model(**cfg)
    p = g.write(tmp_path / "m.gguf")
    ref = oracle.reference_gguf(p)
    if ref is None:
        pytest.skip("reference reader not built (needs the reference sources)")
    got = mine(p)
    for k in ("version", "alignment", "data_offset", "n_metadata"):
        assert got[k] == ref[k], k
    same_table(got["tensors"], ref["tensors"])
    for t in ref["tensors"]:
        assert t["data_at"] == ref["data_offset"] + t["offset"]


def test_table_matches_golden_reference_table(tmp_path):
    """Pinned without the reference sources: the reference reader's table for
    the files make_golden.py wrote, regenerated here from the same seeds."""
    gold = json.loads(GOLDEN.read_text())
    for case in gold:
        g, _ = synthetic_model(**case["config"])
        p = g.write(tmp_path / "m.gguf")
        got = mine(p)
        for k in ("version", "alignment", "data_offset", "n_metadata"):
            assert got[k] == case[k], k
        same_table(got["tensors"], case["tensors"])


def test_metadata_getters(tmp_path):
    g, _ = synthetic_model()
    g.add_meta("x.u32_as_f32", F32, 3.0)
    p = g.write(tmp_path / "m.gguf")
    with ds3.Gguf(p) as f:
        assert f.get_u32("qwen3moe.block_count") == 2
        assert f.get_f32("qwen3moe.attention.layer_norm_rms_epsilon") == pytest.approx(1e-6, rel=1e-7)
        assert f.get_string("general.architecture") == b"qwen3moe"
        # typed getters only match the stored type, as in the engine
        assert f.get_u32("x.u32_as_f32") is None and f.get_f32("x.u32_as_f32") == 3.0
        assert f.get_u32("general.architecture") is None
        assert f.get_u32("absent.key") is None and f.get_string("absent.key") is None


def test_find_returns_first_match_and_none_when_absent(tmp_path):
    g = GgufFile()
    g.add_tensor("a", [4], 0, b"\1" * 16)
    g.add_tensor("a", [8], 0, b"\2" * 32)
    p = g.write(tmp_path / "dup.gguf")
    with ds3.Gguf(p) as f:
        assert f.find("a")["ne"][0] == 4
        assert f.find("b") is None and f.find("") is None


def test_empty_file_tables_and_one_dim_strides(tmp_path):
    g = GgufFile()
    p = g.write(tmp_path / "empty.gguf")
    got = mine(p)
    assert got["tensors"] == [] and got["data_offset"] == 32  # 24-byte header padded to 32
    g.add_tensor("v", [256], 12, b"\0" * 144)
    g.add_tensor("s", [], 0, b"\0" * 4)
    p = g.write(tmp_path / "one.gguf")
    v, s = mine(p)["tensors"]
    assert v["nb"] == [144, 0, 0, 0] and v["size"] == 144      # make_tensor leaves nb[1] = 0 for 1-D
    assert s["n_dims"] == 0 and s["ne"] == [1, 1, 1, 1] and s["size"] == 4


def test_partial_block_counts_whole(tmp_path):
    g = GgufFile()
    g.tensors.append(("q", [300], 12, b"\0" * 288))  # 300 elements of Q4_K: two blocks
    p = g.write(tmp_path / "p.gguf")
    assert mine(p)["tensors"][0]["size"] == 288 == OG.parse(p.read_bytes())["tensors"][0]["size"]


def test_nested_arrays_are_skipped(tmp_path):
    g, _ = synthetic_model()
    g.add_meta("x.nested", ARRAY, (ARRAY, [(U32, [1, 2, 3]), (STRING, ["a", "bc"])]))
    g.add_meta("x.after", U32, 7)
    p = g.write(tmp_path / "n.gguf")
    with ds3.Gguf(p) as f:
        assert f.get_u32("x.after") == 7
        same_table(f.tensors(), OG.parse(p.read_bytes())["tensors"])


# ------------------------------------------------------------ rejections

def _base(tmp_path) -> tuple[bytes, GgufFile]:
    g, _ = synthetic_model(n_layer=1, n_embd=256, n_vocab=4)
    return g.to_bytes(), g


def _rejects(tmp_path, data: bytes, name: str) -> str:
    p = tmp_path / name
    p.write_bytes(data)
    with pytest.raises(OSError) as e:
        ds3.Gguf(p)
    with pytest.raises(OG.ParseError):
        OG.parse(data)
    return str(e.value)


def test_rejects_bad_magic_and_old_version(tmp_path):
    data, _ = _base(tmp_path)
    assert "magic" in _rejects(tmp_path, b"GGUX" + data[4:], "m.gguf")
    assert "version" in _rejects(tmp_path, data[:4] + struct.pack("<I", 2) + data[8:], "v.gguf")
    ref = oracle.reference_gguf(tmp_path / "v.gguf")
    assert ref is None or ref == {"error": True}


@pytest.mark.parametrize("cut", [0, 3, 10, 23, 40, 200, 700])
def test_rejects_truncated_headers(tmp_path, cut):
    data, g = _base(tmp_path)
    hdr, _, _ = g.layout()
    assert cut < len(hdr)
    _rejects(tmp_path, data[:cut], f"t{cut}.gguf")
    ref = oracle.reference_gguf(tmp_path / f"t{cut}.gguf")
    assert ref is None or ref == {"error": True}


def test_rejects_tensor_data_past_end(tmp_path):
    data, _ = _base(tmp_path)
    msg = _rejects(tmp_path, data[:-1], "short.gguf")
    assert "past the end" in msg


def test_rejects_more_than_four_dims_unknown_types_and_zero_alignment(tmp_path):
    g = GgufFile()
    g.tensors.append(("x", [1, 1, 1, 1, 2], 0, b"\0" * 8))
    _rejects(tmp_path, g.to_bytes(), "dims.gguf")
    g = GgufFile()
    g.tensors.append(("x", [32], 99, b""))
    _rejects(tmp_path, g.to_bytes(), "type.gguf")
    # one metadata pair with value type 13 (not in the specification)
    _rejects(tmp_path, _header(0, 1) + _key("x.bad") + struct.pack("<I", 13) + b"\0" * 16, "meta.gguf")
    # general.alignment = 0
    _rejects(tmp_path, _header(0, 1) + _key("general.alignment") + struct.pack("<II", U32, 0), "a0.gguf")


def _header(n_tensors: int, n_meta: int) -> bytes:
    return b"GGUF" + struct.pack("<IQQ", 3, n_tensors, n_meta)


def _key(k: str) -> bytes:
    return struct.pack("<Q", len(k)) + k.encode()


def test_c_info_program_prints_the_same_table(tmp_path):
    """qw3_b200/host/ds3_gguf_info (C, through include/ds3_cuda_gguf.h) on CPU."""
    import subprocess

    exe = build.build_host("ds3_gguf_info")
    g, _ = synthetic_model(alignment=64)
    p = g.write(tmp_path / "m.gguf")
    res = subprocess.run([str(exe), str(p)], capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    lines = [l.split() for l in res.stdout.splitlines()]
    want = mine(p)
    assert lines[0] == ["header", "3", "64", str(len(want["tensors"])), str(want["n_metadata"]),
                        str(want["data_offset"])]
    for l, t in zip(lines[1:], want["tensors"]):
        assert l == ["tensor", t["name"], str(t["n_dims"]), *map(str, t["ne"]), str(t["type"]), str(t["offset"]),
                     str(t["size"])]
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUF" + struct.pack("<I", 2))
    assert subprocess.run([str(exe), str(bad)], capture_output=True).returncode == 1


def test_c_info_program_skips_binding_without_gpu(tmp_path):
    import subprocess

    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    g, _ = synthetic_model()
    res = subprocess.run([str(build.build_host("ds3_gguf_info")), str(g.write(tmp_path / "m.gguf")), "-b", "2"],
                         capture_output=True, text=True)
    assert res.returncode == 77, res.stderr
