"""Pins the CPU oracle (oracle/ds3_oracle.c) before anything is checked
against it.

1. Known answers: the hand-derived cases of the reference's own unit test
   program (tests/test_reference.c of wzqhbustb/qw3: RMSNorm, softmax, SiLU,
   NEOX RoPE, top-k, Q4_K both scale branches, Q6_K, Q8_0, F16, dequantize_row)
   restated here against the oracle.
2. Golden fixtures written by the unmodified reference (tests/golden/).
3. When oracle/_ref is built, bit-for-bit agreement with the unmodified
   reference on fresh seeded inputs, and the reference's own test program.
"""

from __future__ import annotations

import ctypes as C
import math
import subprocess

import numpy as np
import pytest

import oracle
from conftest import assert_bitexact, load_golden
from qw3_b200 import inputs as I

EPS_KAT = 1e-4  # tolerance of the reference's known-answer checks


class I_T:
    F32, F16, Q80, Q4K, Q6K = 0, 1, 8, 12, 14


def near(a, b):
    return abs(float(a) - float(b)) <= EPS_KAT


def fp(a):
    return np.ascontiguousarray(a, np.float32)


# ----------------------------------------------------------- known answers
def test_kat_rms_norm(port):
    x = fp([1, 2, 3, 4])
    out = np.empty(4, np.float32)
    port._rms_norm(x.ctypes.data, fp([1, 1, 1, 1]).ctypes.data, 1e-6, 4, out.ctypes.data)
    rms = math.sqrt(7.5)
    assert all(near(out[i], (i + 1) / rms) for i in range(4))
    port._rms_norm(x.ctypes.data, fp([2, 2, 2, 2]).ctypes.data, 1e-6, 4, out.ctypes.data)
    assert near(out[0], 2 / rms) and near(out[3], 8 / rms)


def test_kat_softmax(port):
    x = fp([1, 2, 3, 4])
    port._softmax(x.ctypes.data, 4)
    assert near(x.sum(), 1.0) and near(x[0], 0.0320586) and near(x[3], 0.6439143)
    y = fp([5, 5, 5, 5])
    port._softmax(y.ctypes.data, 4)
    assert near(y[0], 0.25)


def test_kat_silu(port):
    g = fp([[0.0, 1.0, -1.0]])
    out = port.swiglu(g, np.ones_like(g))
    assert near(out[0, 0], 0.0)
    assert near(out[0, 1], 1 / (1 + math.exp(-1)))
    assert near(out[0, 2], -1 / (1 + math.exp(1)))


def test_kat_rope_neox(port):
    # head_dim 4, NEOX pairs (0,2), (1,3); pair 1 frequency theta^(-1/2) = 1e-3.
    q = fp([1, 0, 1, 0])
    k = fp([1, 0, 1, 0])
    port._rope_token(q.ctypes.data, k.ctypes.data, 0, 1, 1, 4, 1e6)
    assert near(q[0], 1) and near(q[1], 0) and near((q * q).sum(), 2.0)
    q2 = fp([1, 0, 0, 1])
    k2 = fp([0, 1, 1, 0])
    port._rope_token(q2.ctypes.data, k2.ctypes.data, 1, 1, 1, 4, 1e6)
    assert near(q2[0], math.cos(1)) and near(q2[2], math.sin(1))
    assert near(q2[1], -math.sin(1e-3)) and near(q2[3], math.cos(1e-3))
    q3 = fp([1, 0, 0, 1, 2, 0, 0, 2])
    k3 = fp([1, 0, 0, 1])
    port._rope_token(q3.ctypes.data, k3.ctypes.data, 1, 2, 1, 4, 1e6)
    assert near(q3[4], 2 * math.cos(1)) and near(q3[5], -2 * math.sin(1e-3)) and near(q3[7], 2.0)


def test_kat_topk(port):
    s = fp([0.1, 0.5, 0.2, 0.9, 0.3, 0.8, 0.0, 0.4])
    idx = np.empty(3, np.int32)
    val = np.empty(3, np.float32)
    port._topk(s.ctypes.data, 8, 3, idx.ctypes.data, val.ctypes.data)
    assert list(idx) == [3, 5, 1]
    assert near(val[0], 0.9) and near(val[2], 0.5)


def test_topk_ties_lowest_index_first(port):
    s = fp([0.5, 0.7, 0.7, 0.1, 0.7])
    idx = np.empty(3, np.int32)
    val = np.empty(3, np.float32)
    port._topk(s.ctypes.data, 5, 3, idx.ctypes.data, val.ctypes.data)
    assert list(idx) == [1, 2, 4]


def _dequant(port, type_, blk, n):
    blk = np.ascontiguousarray(blk, np.uint8)
    out = np.empty(n, np.float32)
    assert port._dequant_row(type_, blk.ctypes.data, n, out.ctypes.data) == 0
    return out


def test_kat_q4k_both_scale_branches(port):
    b = np.zeros(144, np.uint8)
    b[0:2] = [0x00, 0x3C]  # d = 1.0
    b[2:4] = [0x00, 0x3C]  # dmin = 1.0
    scales = b[4:16]
    scales[0] = 1
    scales[1] = 1
    scales[8] = 0x53  # pair 4: sc 3, m 5 (j >= 4 branch)
    scales[9] = 0x02  # pair 5: sc 2, m 0
    qs = b[16:]
    qs[0] = 0xAB
    qs[64] = 0xCD
    y = _dequant(port, I_T.Q4K, b, 256)
    assert near(y[0], 11) and near(y[32], 10) and near(y[1], 0) and near(y[33], 0)
    assert near(y[128], 34) and near(y[160], 24) and near(y[129], -5) and near(y[161], 0)


def test_kat_q6k(port):
    b = np.zeros(210, np.uint8)
    b[192:208] = 1  # scales
    b[208:210] = [0x00, 0x3C]  # d = 1.0
    b[0] = 0x31
    b[32] = 0x42
    b[128] = 0xAA
    y = _dequant(port, I_T.Q6K, b, 256)
    assert near(y[0], 1) and near(y[32], 2) and near(y[64], 3) and near(y[96], 4)
    assert near(y[1], -32)


def test_kat_q8_0_and_f16(port):
    b = np.zeros(34, np.uint8)
    b[0:2] = [0x00, 0x3C]
    b[2] = 5
    b[3] = np.uint8(np.int8(-3).view(np.uint8))
    y = _dequant(port, I_T.Q80, b, 32)
    assert near(y[0], 5) and near(y[1], -3) and near(y[2], 0)
    h = np.array([0x3C00, 0x4000, 0x0000], np.uint16)
    y = _dequant(port, I_T.F16, h.view(np.uint8), 3)
    assert list(y) == [1.0, 2.0, 0.0]


def test_kat_dequantize_row(port):
    f32 = fp([[1, 2, 3], [4, 5, 6]])
    rc, out = port.embed_rows(f32.view(np.uint8), I_T.F32, 12, 2, [1], 3)
    assert rc == 0 and list(out[0]) == [4, 5, 6]
    f16 = np.array([[0x3C00, 0x4000, 0x0000], [0x4200, 0x4400, 0x4500]], np.uint16)
    rc, out = port.embed_rows(f16.view(np.uint8), I_T.F16, 6, 2, [0, 1], 3)
    assert rc == 0 and list(out[0]) == [1, 2, 0] and list(out[1]) == [3, 4, 5]


def test_embed_rejects_out_of_range_ids(port):
    tab = I.q4k_table(4, 256, 1)
    rc, out = port.embed_rows(tab, I_T.Q4K, 144, 4, [0, 4, -1, 3], 256)
    assert rc == -1
    assert not out[1].any() and not out[2].any() and out[0].any()


# --------------------------------------------------------- golden fixtures
@pytest.mark.parametrize("name", ["embed_q4k_512.npz", "embed_q4k_2048.npz", "embed_q6k_512.npz",
                                  "embed_q6k_2048.npz"])
def test_golden_embed(port, name):
    g = load_golden(name)
    n_cols = g["out"].shape[1]
    rc, out = port.embed_rows(g["table"], int(g["type"]), g["table"].shape[1], int(g["n_vocab"]), g["ids"], n_cols)
    assert rc == 0
    assert_bitexact(out, g["out"], name)
    rc, hid, nrm = port.embed_rms_norm(g["table"], int(g["type"]), g["table"].shape[1], int(g["n_vocab"]),
                                       g["ids"], n_cols, g["w"], 1e-6)
    assert_bitexact(nrm, g["norm"], name + " norm")


def test_golden_norms(port):
    g = load_golden("add_rms_norm.npz")
    s, o = port.add_rms_norm(g["x"], g["r"], g["w"], 1e-6)
    assert_bitexact(s, g["sum"], "sum")
    assert_bitexact(o, g["norm"], "norm")
    assert_bitexact(port.rms_norm_rows(g["x"], g["w"], 1e-6), g["plain"], "plain")


def test_golden_qk_norm_rope(port):
    g = load_golden("qk_norm_rope.npz")
    q, k = port.qk_norm_rope(g["q"], g["k"], g["q_w"], g["k_w"], g["pos"], 1e6, 1e-6)
    assert_bitexact(q, g["q_out"], "q")
    assert_bitexact(k, g["k_out"], "k")
    assert_bitexact(port.rope_rows(g["q"], g["pos"], 1e6), g["q_rope_only"], "rope")


def test_golden_router(port):
    g = load_golden("router.npz")
    p, i, s = port.router(g["logits"], 8, True)
    assert_bitexact(p, g["probs"], "probs")
    assert_bitexact(i, g["idx"], "idx")
    assert_bitexact(s, g["scores"], "scores")
    _, i2, s2 = port.router(g["logits"], 8, False)
    assert_bitexact(i2, g["idx_raw"], "idx raw")
    assert_bitexact(s2, g["scores_raw"], "scores raw")


def test_golden_swiglu_combine(port):
    g = load_golden("swiglu.npz")
    assert_bitexact(port.swiglu(g["gate"], g["up"], g["row_w"]), g["out"], "swiglu")
    assert_bitexact(port.swiglu(g["gate"], g["up"], None), g["out_plain"], "silu_mul")
    g = load_golden("combine.npz")
    assert_bitexact(port.combine(g["y"], g["w"], g["residual"]), g["out"], "combine")


def test_thread_count_does_not_change_results(port):
    x = I.normal(1, (64, 2048))
    w = I.gamma(2048, 2)
    assert_bitexact(port.rms_norm_rows(x, w, 1e-6, 1), port.rms_norm_rows(x, w, 1e-6, 4), "threads")


# --------------------------------------------- the unmodified reference
ref = oracle.reference()
needs_ref = pytest.mark.skipif(ref is None, reason="oracle/_ref not built (reference sources absent)")


@needs_ref
def test_port_equals_reference_seeded(port):
    tab = I.q4k_table(500, 2048, 11)
    ids = I.token_ids(96, 12, 500)
    assert_bitexact(port.embed_rows(tab, 12, 1152, 500, ids, 2048)[1], ref.embed_rows(tab, 12, 1152, 500, ids, 2048)[1])
    tab6 = I.q6k_table(500, 2048, 13)
    assert_bitexact(port.embed_rows(tab6, 14, 1680, 500, ids, 2048)[1],
                    ref.embed_rows(tab6, 14, 1680, 500, ids, 2048)[1])
    q = I.normal(14, (8, 32, 128))
    k = I.normal(15, (8, 4, 128))
    pos = I.rng(16).integers(0, 32768, 8).astype(np.int32)
    qw, kw = I.gamma(128, 17), I.gamma(128, 18)
    a = port.qk_norm_rope(q, k, qw, kw, pos, 1e6, 1e-6)
    b = ref.qk_norm_rope(q, k, qw, kw, pos, 1e6, 1e-6)
    assert_bitexact(a[0], b[0])
    assert_bitexact(a[1], b[1])
    lg = I.normal(19, (256, 128), 0, 2)
    for x, y in zip(port.router(lg, 8), ref.router(lg, 8)):
        assert_bitexact(x, y)
    g = I.normal(20, (32, 768), 0, 1.5)
    u = I.normal(21, (32, 768), 0, 1.5)
    rw = I.normal(22, (32,))
    assert_bitexact(port.swiglu(g, u, rw), ref.swiglu(g, u, rw))
    y = I.normal(23, (64, 2048))
    w = I.normal(24, (8, 8))
    r = I.normal(25, (8, 2048))
    rows = I.rng(26).permutation(64).astype(np.int32)
    assert_bitexact(port.combine(y, w, r, rows), ref.combine(y, w, r, rows))


@needs_ref
def test_reference_own_known_answer_program():
    exe = oracle.HERE / "_ref" / "test_reference"
    if not exe.exists():
        pytest.skip("reference test program not built")
    res = subprocess.run([str(exe)], capture_output=True, text=True)
    assert res.returncode == 0, res.stdout[-2000:]
    assert "0 failed" in res.stdout


def test_kv_cache_write_rounds_like_numpy_fp16(port):
    # metal/attention.metal:66-87 stores half(k), half(v) at row seq_pos + t.
    k = I.normal(30, (3, 4, 128), 0.0, 3.0)
    v = I.normal(31, (3, 4, 128), 0.0, 3.0)
    ck = np.full((9, 4, 128), 0x7E00, np.uint16)
    cv = ck.copy()
    oracle.kv_cache_write(port, k, v, ck, cv, seq_pos=5)
    assert np.array_equal(ck[5:8].view(np.float16), k.astype(np.float16))
    assert np.array_equal(cv[5:8].view(np.float16), v.astype(np.float16))
    assert (ck[:5] == 0x7E00).all() and (ck[8:] == 0x7E00).all()
    rows = np.array([8, 0, 3], np.int32)
    oracle.kv_cache_write(port, k, v, ck, cv, row_of=rows)
    assert np.array_equal(ck[rows].view(np.float16), k.astype(np.float16))


def test_moe_expert_lists_engine_layout(port):
    # src/ds3_engine.c:933-954: tokens ascending per expert, strided by M.
    idx = np.array([[2, 0], [0, 1], [2, 1]], np.int32)
    sc = np.array([[0.6, 0.4], [0.7, 0.3], [0.5, 0.5]], np.float32)
    rc, counts, ids, gs, slot = oracle.moe_expert_lists(port, idx, sc, 3, 3)
    assert rc == 0 and list(counts) == [2, 2, 2]
    assert list(ids[0:2]) == [0, 1] and list(ids[3:5]) == [1, 2] and list(ids[6:8]) == [0, 2]
    assert np.allclose(gs[[0, 1, 3, 4, 6, 7]], [0.4, 0.7, 0.3, 0.5, 0.6, 0.5])
    assert list(slot) == [6, 0, 1, 3, 7, 4]
    rc, *_ = oracle.moe_expert_lists(port, np.array([[5, 0]], np.int32), sc[:1], 3, 3)
    assert rc == -1


@needs_ref
def test_router_logits_equal_reference_vec_matmul(port):
    x = I.normal(40, (9, 2048))
    W = I.normal(41, (128, 2048), 0.0, 0.05)
    assert_bitexact(port.router_logits(x, W), ref.router_logits(x, W))
