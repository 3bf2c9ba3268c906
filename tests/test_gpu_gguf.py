"""Real-checkpoint path on the device: ds3_cuda_dequantize_f32 against the
oracle's restatement of ds3_ref_dequantize_tensor (bit-exact), and
ds3_cuda_path_weights_load on synthetic GGUF files (tests/gguf_writer.py)
whose bound tensors must equal the file's contents converted to fp32 and
drive the fused embedding exactly like directly uploaded weights."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_bitexact, assert_close
from gguf_writer import f16_bytes, q8_0_bytes, synthetic_model
from qw3_b200 import inputs as I

pytestmark = pytest.mark.gpu


def oracle_dequant(port, type_: int, raw: bytes, n: int) -> np.ndarray:
    src = np.frombuffer(raw, np.uint8).copy()
    out = np.empty(n, np.float32)
    assert port._dequant_row(type_, src.ctypes.data, n, out.ctypes.data) == 0
    return out


@pytest.fixture
def keep(ds3):
    bufs = []
    yield bufs
    for b in bufs:
        b.free()
    assert ds3.device_errors() == 0


def cases():
    w = I.normal(11, (4096,), 0.0, 1.5)
    return [("f32", 0, w.astype("<f4").tobytes(), 4096),
            ("f16", 1, f16_bytes(w.astype(np.float16)), 4096),
            ("q8_0", 8, q8_0_bytes(w), 4096),
            ("q4_k", 12, I.q4k_table(3, 2048, 12).tobytes(), 3 * 2048),
            ("q6_k", 14, I.q6k_table(3, 2048, 13).tobytes(), 3 * 2048),
            ("f16_odd", 1, f16_bytes(w[:37].astype(np.float16)), 37)]


@pytest.mark.parametrize("name,type_,raw,n", cases(), ids=[c[0] for c in cases()])
def test_dequantize_f32_bitexact(ds3, port, keep, name, type_, raw, n):
    src = ds3.upload(np.frombuffer(raw, np.uint8).copy())
    dst = ds3.empty(n * 4)
    keep += [src, dst]
    assert ds3.dequantize_f32(src, type_, n, dst) == 0, ds3.last_error()
    assert_bitexact(ds3.download(dst, np.float32, (n,)), oracle_dequant(port, type_, raw, n), name)


def test_dequantize_f32_rejects_bad_arguments(ds3, keep):
    src, dst = ds3.empty(1024), ds3.empty(4096)
    keep += [src, dst]
    assert ds3.dequantize_f32(src, 12, 100, dst) == -1      # not a whole Q4_K block
    assert ds3.dequantize_f32(src, 3, 256, dst) == -1       # unsupported type
    assert ds3.dequantize_f32(src, 0, 512, dst) == -1       # src too small (2048 bytes needed)
    assert ds3.dequantize_f32(src, 1, 0, dst) == -1


@pytest.mark.parametrize("cfg", [dict(), dict(norm_type=0, embd_type=14, alignment=256),
                                 dict(norm_type=8, n_layer=3, seed=3, n_embd=1024)])
def test_path_weights_match_file_contents(ds3, port, tmp_path, cfg):
    g, raw = synthetic_model(**cfg)
    p = g.write(tmp_path / "m.gguf")
    n_layer = cfg.get("n_layer", 2)
    with ds3.Gguf(p) as f:
        w = ds3.PathWeights(f, n_layer)
        try:
            c = w.c
            tab = raw["token_embd.weight"]
            n_embd = cfg.get("n_embd", 512)
            assert (c.n_layer, c.n_embd, c.n_vocab, c.head_dim, c.n_expert) == (n_layer, n_embd, tab.shape[0],
                                                                                 128, 16)
            assert c.token_embd_type == cfg.get("embd_type", 12) and c.token_embd_row_stride == tab.shape[1]
            te = ds3._Borrowed(c.token_embd, tab.nbytes)
            assert_bitexact(ds3.download(te, np.uint8, tab.shape), tab, "token_embd bytes")
            norm_t = cfg.get("norm_type", 1)

            def check(buf, name, n, type_):
                data, _ = raw[name]
                want = oracle_dequant(port, type_, data, n)
                assert_bitexact(ds3.download(ds3._Borrowed(buf, n * 4), np.float32, (n,)), want, name)

            check(c.output_norm, "output_norm.weight", c.n_embd, norm_t)
            for l in range(n_layer):
                check(c.attn_norm[l], f"blk.{l}.attn_norm.weight", c.n_embd, norm_t)
                check(c.attn_q_norm[l], f"blk.{l}.attn_q_norm.weight", 128, norm_t)
                check(c.attn_k_norm[l], f"blk.{l}.attn_k_norm.weight", 128, norm_t)
                check(c.ffn_norm[l], f"blk.{l}.ffn_norm.weight", c.n_embd, norm_t)
                check(c.ffn_gate_inp[l], f"blk.{l}.ffn_gate_inp.weight", 16 * c.n_embd, l % 2)
        finally:
            w.free()
    assert ds3.device_errors() == 0


def test_loaded_weights_drive_the_fused_embedding(ds3, port, tmp_path, keep):
    """embed_rms_norm over the bound token_embd and attn_norm equals the oracle
    over the same bytes from the file."""
    g, raw = synthetic_model(n_layer=1, n_embd=2048, n_vocab=96, norm_type=1, seed=9)
    p = g.write(tmp_path / "m.gguf")
    with ds3.Gguf(p) as f:
        w = ds3.PathWeights(f, 1)
        try:
            c = w.c
            ids = I.token_ids(33, 5, c.n_vocab)
            idb = ds3.upload(ids)
            hid, nrm = ds3.empty(33 * 2048 * 4), ds3.empty(33 * 2048 * 4)
            keep += [idb, hid, nrm]
            tabb = ds3._Borrowed(c.token_embd, raw["token_embd.weight"].nbytes)
            gam = ds3._Borrowed(c.attn_norm[0], 2048 * 4)
            rc = ds3.embed_rms_norm(tabb, idb, gam, hid, nrm, 33, 2048, c.n_vocab, c.token_embd_type,
                                    c.token_embd_row_stride, 1e-6)
            assert rc == 0, ds3.last_error()
            tab = raw["token_embd.weight"]
            gw = raw["blk.0.attn_norm.weight"][1]
            rc, want_h, want_n = port.embed_rms_norm(tab, 12, tab.shape[1], c.n_vocab, ids, 2048, gw, 1e-6)
            assert rc == 0
            assert_bitexact(ds3.download(hid, np.float32, (33, 2048)), want_h, "hidden")
            assert_close(ds3.download(nrm, np.float32, (33, 2048)), want_n, what="norm")
        finally:
            w.free()


def test_missing_tensor_fails_the_load(ds3, tmp_path):
    g, _ = synthetic_model(n_layer=1, n_embd=256)
    with ds3.Gguf(g.write(tmp_path / "full.gguf")) as f:
        with pytest.raises(RuntimeError, match="blk.1"):
            ds3.PathWeights(f, 2)   # the file holds one layer
    g.tensors = [t for t in g.tensors if t[0] != "blk.0.ffn_norm.weight"]
    with ds3.Gguf(g.write(tmp_path / "m.gguf")) as f:
        with pytest.raises(RuntimeError, match="blk.0.ffn_norm.weight"):
            ds3.PathWeights(f, 1)
    g2, _ = synthetic_model(n_layer=1, n_embd=256)
    g2.tensors = [t for t in g2.tensors if "attn_q_norm" not in t[0]]
    p2 = g2.write(tmp_path / "noqk.gguf")
    with ds3.Gguf(p2) as f:
        with pytest.raises(RuntimeError, match="attn_q_norm"):
            ds3.PathWeights(f, 1)
        w = ds3.PathWeights(f, 1, require_qk_norm=False)   # the 235B variant has no q/k norms
        assert not w.c.attn_q_norm[0] and w.c.head_dim == 0
        w.free()
    assert ds3.device_errors() == 0


def test_c_info_program_binds_on_the_gpu(tmp_path):
    import subprocess

    from qw3_b200 import build

    g, _ = synthetic_model(n_layer=2, n_embd=512, n_vocab=64)
    res = subprocess.run([str(build.build_host("ds3_gguf_info")), str(g.write(tmp_path / "m.gguf")), "-b", "2"],
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    assert res.stdout.splitlines()[-1].split() == ["bound", "2", "512", "64", "128", "16", "12"]


@pytest.mark.parametrize("norm_type", [1, 8])
def test_loaded_weights_drive_the_layer_ops(ds3, port, tmp_path, keep, norm_type):
    """QK-norm+RoPE, add+RMSNorm and the router projection + top-k, each fed
    with the tensors bound from the file (norms stored F16 or Q8_0, the router
    F32 in layer 0 and F16 in layer 1), against the oracle on the same values."""
    H, T, NQ, NK, HD, E, K = 512, 24, 32, 4, 128, 16, 4
    g, raw = synthetic_model(n_layer=2, n_embd=H, n_vocab=8, norm_type=norm_type, seed=21)
    with ds3.Gguf(g.write(tmp_path / "m.gguf")) as f:
        w = ds3.PathWeights(f, 2)
        try:
            c = w.c

            def wval(name, n, type_):
                return oracle_dequant(port, type_, raw[name][0], n)

            for l in range(2):
                q, k = I.normal(30 + l, (T, NQ, HD)), I.normal(40 + l, (T, NK, HD))
                pos = I.rng(50 + l).integers(0, 4096, T).astype(np.int32)
                qb, kb, pb = ds3.upload(q), ds3.upload(k), ds3.upload(pos)
                keep += [qb, kb, pb]
                qn = ds3._Borrowed(c.attn_q_norm[l], HD * 4)
                kn = ds3._Borrowed(c.attn_k_norm[l], HD * 4)
                assert ds3.qk_norm_rope(qb, kb, qn, kn, pb, T, NQ, NK, HD, 1e6, 1e-6) == 0, ds3.last_error()
                want_q, want_k = port.qk_norm_rope(q, k, wval(f"blk.{l}.attn_q_norm.weight", HD, norm_type),
                                                   wval(f"blk.{l}.attn_k_norm.weight", HD, norm_type), pos,
                                                   1e6, 1e-6)
                assert_close(ds3.download(qb, np.float32, q.shape), want_q, what=f"q layer {l}")
                assert_close(ds3.download(kb, np.float32, k.shape), want_k, what=f"k layer {l}")

                x, r = I.normal(60 + l, (T, H)), I.normal(70 + l, (T, H))
                xb, rb, sb, nb = ds3.upload(x), ds3.upload(r), ds3.empty(T * H * 4), ds3.empty(T * H * 4)
                keep += [xb, rb, sb, nb]
                fw = ds3._Borrowed(c.ffn_norm[l], H * 4)
                assert ds3.add_rms_norm(xb, rb, fw, sb, nb, H, T, 1e-6) == 0, ds3.last_error()
                want_s, want_n = port.add_rms_norm(x, r, wval(f"blk.{l}.ffn_norm.weight", H, norm_type), 1e-6)
                assert_bitexact(ds3.download(sb, np.float32, (T, H)), want_s, f"sum layer {l}")
                assert_close(ds3.download(nb, np.float32, (T, H)), want_n, what=f"norm layer {l}")

                Wr = wval(f"blk.{l}.ffn_gate_inp.weight", E * H, l % 2).reshape(E, H)
                lb, ib, scb = ds3.empty(T * E * 4), ds3.empty(T * K * 4), ds3.empty(T * K * 4)
                keep += [lb, ib, scb]
                gw = ds3._Borrowed(c.ffn_gate_inp[l], E * H * 4)
                assert ds3.router_logits_topk(nb, gw, lb, ib, scb, T, H, E, K, True) == 0, ds3.last_error()
                lg = port.router_logits(ds3.download(nb, np.float32, (T, H)), Wr)
                _, want_i, want_sc = port.router(lg, K, True)
                assert_bitexact(ds3.download(lb, np.float32, (T, E)), lg, f"router logits layer {l}")
                assert_bitexact(ds3.download(ib, np.int32, (T, K)), want_i, f"top-k layer {l}")
                assert_close(ds3.download(scb, np.float32, (T, K)), want_sc, what=f"scores layer {l}")
        finally:
            w.free()
