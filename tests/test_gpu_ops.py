"""GPU parity: every ds3_cuda entry point against the CPU oracle and the
golden fixtures of the unmodified reference, through the C-ABI.

Bars (the tolerances the path is held to): bit-exact for embedding dequant, residual sums, the
weighted combine and router top-k indices (exact ties excluded; the seeded
inputs here have none); within 1e-5 relative / 1e-6 absolute for fp32 norm,
RoPE, SwiGLU and softmax outputs; 2e-3 relative (1e-3 absolute floor) for the
fp16-storage RoPE variant against the oracle run on the fp16-rounded inputs.
Shapes follow the reference's own GPU tests (tests/test_metal.c: [4,2048]
norm, Q [4,32,128] / K [4,4,128] RoPE) plus ragged sizes (T = 1, 3, 17, 511),
widths the fast paths do not take, and bad ids.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_bitexact, assert_close, load_golden
from qw3_b200 import inputs as I

pytestmark = pytest.mark.gpu

F32, F16, Q80, Q4K, Q6K = 0, 1, 8, 12, 14


class Bufs:
    """Uploads numpy arrays and frees everything at the end of a test."""

    def __init__(self, ds3):
        self.d = ds3
        self.all = []

    def up(self, a):
        b = self.d.upload(np.ascontiguousarray(a))
        self.all.append(b)
        return b

    def empty(self, nbytes):
        b = self.d.empty(nbytes)
        self.all.append(b)
        return b

    def close(self):
        for b in self.all:
            b.free()


@pytest.fixture
def B(ds3):
    b = Bufs(ds3)
    yield b
    b.close()
    assert ds3.device_errors() == 0


def f32(b, ds3, shape):
    return ds3.download(b, np.float32, shape)


# ------------------------------------------------------------------ embedding
def run_embed(ds3, B, tab, type_, n_vocab, ids, n_cols, stride=None, w=None):
    stride = stride or tab.shape[1]
    t = B.up(tab)
    i = B.up(np.asarray(ids, np.int32))
    n = len(ids)
    out = B.empty(n * n_cols * 4)
    rc = ds3.embed_rows(t, i, out, n, n_cols, n_vocab, type_, stride)
    res = [rc, f32(out, ds3, (n, n_cols))]
    if w is not None:
        hid, nrm = B.empty(n * n_cols * 4), B.empty(n * n_cols * 4)
        wb = B.up(w)
        rc2 = ds3.embed_rms_norm(t, i, wb, hid, nrm, n, n_cols, n_vocab, type_, stride, 1e-6)
        res += [rc2, f32(hid, ds3, (n, n_cols)), f32(nrm, ds3, (n, n_cols))]
    return res


@pytest.mark.parametrize("name", ["embed_q4k_512.npz", "embed_q4k_2048.npz", "embed_q6k_512.npz",
                                  "embed_q6k_2048.npz"])
def test_embed_golden(ds3, B, name):
    g = load_golden(name)
    n_cols = g["out"].shape[1]
    rc, out, rc2, hid, nrm = run_embed(ds3, B, g["table"], int(g["type"]), int(g["n_vocab"]), g["ids"], n_cols,
                                       w=g["w"])
    assert rc == 0 and rc2 == 0
    assert_bitexact(out, g["out"], name)
    assert_bitexact(hid, g["out"], name + " hidden")
    assert_close(nrm, g["norm"], what=name + " norm")


@pytest.mark.parametrize("type_,maker", [(Q4K, I.q4k_table), (Q6K, I.q6k_table)])
@pytest.mark.parametrize("n_cols", [256, 512, 1024, 2048])
@pytest.mark.parametrize("T", [1, 3, 17, 511])
def test_embed_vs_oracle(ds3, B, port, type_, maker, n_cols, T):
    vocab = 1000
    tab = maker(vocab, n_cols, 10 + n_cols)
    ids = I.token_ids(T, 20 + T, vocab)
    w = I.gamma(n_cols, 30)
    rc, out, rc2, hid, nrm = run_embed(ds3, B, tab, type_, vocab, ids, n_cols, w=w)
    assert rc == 0 and rc2 == 0
    _, want, want_n = port.embed_rms_norm(tab, type_, tab.shape[1], vocab, ids, n_cols, w, 1e-6)
    assert_bitexact(out, want, "embed")
    assert_bitexact(hid, want, "embed hidden")
    assert_close(nrm, want_n, what="embed norm")


@pytest.mark.parametrize("type_", [F32, F16, Q80])
def test_embed_other_types(ds3, B, port, type_):
    n_cols, vocab, T = 256, 50, 19
    g = I.rng(5)
    if type_ == F32:
        tab = I.normal(6, (vocab, n_cols)).view(np.uint8)
    elif type_ == F16:
        tab = I.normal(6, (vocab, n_cols)).astype(np.float16).view(np.uint8)
    else:
        tab = g.integers(0, 256, (vocab, n_cols // 32 * 34), dtype=np.uint8)
        d = g.uniform(0, 0.02, (vocab, n_cols // 32, 1)).astype(np.float16).view(np.uint8)
        t3 = tab.reshape(vocab, n_cols // 32, 34)
        t3[:, :, 0:2] = d
    ids = I.token_ids(T, 7, vocab)
    rc, out = run_embed(ds3, B, tab, type_, vocab, ids, n_cols)
    assert rc == 0
    assert_bitexact(out, port.embed_rows(tab, type_, tab.shape[1], vocab, ids, n_cols)[1])


def test_embed_padded_row_stride(ds3, B, port):
    # Rows padded to 1160 B (not a multiple of 16): the byte-copy staging path.
    vocab, n_cols = 64, 2048
    raw = I.q4k_table(vocab, n_cols, 40)
    tab = np.zeros((vocab, 1160), np.uint8)
    tab[:, :1152] = raw
    ids = I.token_ids(33, 41, vocab)
    rc, out = run_embed(ds3, B, tab, Q4K, vocab, ids, n_cols, stride=1160)
    assert rc == 0
    assert_bitexact(out, port.embed_rows(raw, Q4K, 1152, vocab, ids, n_cols)[1])


def test_embed_bad_ids_fail_loudly(ds3, B, port):
    vocab, n_cols = 100, 2048
    tab = I.q4k_table(vocab, n_cols, 50)
    ids = np.array([3, 100, -1, 99, 7], np.int32)
    rc, out = run_embed(ds3, B, tab, Q4K, vocab, ids, n_cols)
    assert rc == -1
    assert not out[1].any() and not out[2].any()
    _, want = port.embed_rows(tab, Q4K, 1152, vocab, ids, n_cols)
    assert_bitexact(out, want)
    assert ds3.device_errors() == 0  # the failing call consumed the error bits


# ---------------------------------------------------------------- RMSNorm
@pytest.mark.parametrize("rows,n", [(4, 2048), (512, 2048), (7, 128), (3, 4), (5, 1000), (2, 4096), (9, 768)])
def test_rms_norm(ds3, B, port, rows, n):
    x = I.normal(rows * n, (rows, n))
    w = I.gamma(n, 3)
    xb, wb, ob = B.up(x), B.up(w), B.empty(x.nbytes)
    assert ds3.rms_norm(xb, wb, ob, n, rows, 1e-6) == 0
    assert_close(f32(ob, ds3, x.shape), port.rms_norm_rows(x, w, 1e-6))
    # in place, as the engine does for q/k and output_norm
    assert ds3.rms_norm(xb, wb, xb, n, rows, 1e-6) == 0
    assert_close(f32(xb, ds3, x.shape), port.rms_norm_rows(x, w, 1e-6))


@pytest.mark.parametrize("rows,n", [(64, 2048), (1, 2048), (17, 2048), (6, 1000), (3000, 2048), (2500, 1024)])
def test_add_rms_norm(ds3, B, port, rows, n):
    x, r, w = I.normal(1, (rows, n)), I.normal(2, (rows, n)), I.gamma(n, 3)
    s_want, n_want = port.add_rms_norm(x, r, w, 1e-6)
    xb, rb, wb = B.up(x), B.up(r), B.up(w)
    sb, nb = B.empty(x.nbytes), B.empty(x.nbytes)
    assert ds3.add_rms_norm(xb, rb, wb, sb, nb, n, rows, 1e-6) == 0
    assert_bitexact(f32(sb, ds3, x.shape), s_want, "sum")
    assert_close(f32(nb, ds3, x.shape), n_want, what="norm")
    # engine aliasing: residual <- sum, hidden <- norm (src/ds3_engine.c:857-866)
    assert ds3.add_rms_norm(xb, rb, wb, rb, xb, n, rows, 1e-6) == 0
    assert_bitexact(f32(rb, ds3, x.shape), s_want, "sum in place")
    assert_close(f32(xb, ds3, x.shape), n_want, what="norm in place")
    # no sum output
    xb2, rb2, nb2 = B.up(x), B.up(r), B.empty(x.nbytes)
    assert ds3.add_rms_norm(xb2, rb2, wb, None, nb2, n, rows, 1e-6) == 0
    assert_close(f32(nb2, ds3, x.shape), n_want, what="norm no-sum")


# ------------------------------------------------------- QK-norm + RoPE
def test_qk_norm_rope_golden(ds3, B):
    g = load_golden("qk_norm_rope.npz")
    T = g["q"].shape[0]
    qb, kb = B.up(g["q"]), B.up(g["k"])
    rc = ds3.qk_norm_rope(qb, kb, B.up(g["q_w"]), B.up(g["k_w"]), B.up(g["pos"]), T, 32, 4, 128, 1e6, 1e-6)
    assert rc == 0
    assert_close(f32(qb, ds3, g["q"].shape), g["q_out"], what="q")
    assert_close(f32(kb, ds3, g["k"].shape), g["k_out"], what="k")


@pytest.mark.parametrize("T,maxpos", [(4, 22), (64, 512), (17, 4096), (511, 32768)])
def test_qk_norm_rope_vs_oracle(ds3, B, port, T, maxpos):
    q, k = I.normal(T, (T, 32, 128)), I.normal(T + 1, (T, 4, 128))
    qw, kw = I.gamma(128, 2), I.gamma(128, 3)
    pos = I.rng(T + 2).integers(0, maxpos, T).astype(np.int32)
    pos[-1] = maxpos - 1
    qb, kb = B.up(q), B.up(k)
    assert ds3.qk_norm_rope(qb, kb, B.up(qw), B.up(kw), B.up(pos), T, 32, 4, 128, 1e6, 1e-6) == 0
    qo, ko = port.qk_norm_rope(q, k, qw, kw, pos, 1e6, 1e-6)
    assert_close(f32(qb, ds3, q.shape), qo, what="q")
    assert_close(f32(kb, ds3, k.shape), ko, what="k")


@pytest.mark.parametrize("nq,nk,hd", [(2, 1, 4), (8, 2, 64), (5, 3, 128), (4, 0, 256)])
def test_qk_norm_rope_shapes(ds3, B, port, nq, nk, hd):
    T = 9
    q, k = I.normal(1, (T, nq, hd)), I.normal(2, (T, max(nk, 1), hd))[:, :nk]
    qw, kw = I.gamma(hd, 3), I.gamma(hd, 4)
    pos = I.rng(5).integers(0, 1000, T).astype(np.int32)
    qb = B.up(q)
    kb = B.up(k) if nk else None
    assert ds3.qk_norm_rope(qb, kb, B.up(qw), B.up(kw), B.up(pos), T, nq, nk, hd, 1e6, 1e-6) == 0
    qo, ko = port.qk_norm_rope(q, k, qw, kw, pos, 1e6, 1e-6)
    assert_close(f32(qb, ds3, q.shape), qo, what="q")
    if nk:
        assert_close(f32(kb, ds3, k.shape), ko, what="k")


@pytest.mark.parametrize("T", [128, 2049, 4100])
def test_qk_norm_rope_fp16_storage(ds3, B, port, T):
    q = I.normal(7, (T, 32, 128)).astype(np.float16)
    k = I.normal(8, (T, 4, 128)).astype(np.float16)
    qw, kw = I.gamma(128, 9), I.gamma(128, 10)
    pos = (np.arange(T, dtype=np.int32) * 250) % 32768
    qb, kb = B.up(q), B.up(k)
    assert ds3.qk_norm_rope(qb, kb, B.up(qw), B.up(kw), B.up(pos), T, 32, 4, 128, 1e6, 1e-6, F16) == 0
    qo, ko = port.qk_norm_rope(q.astype(np.float32), k.astype(np.float32), qw, kw, pos, 1e6, 1e-6)
    got_q = ds3.download(qb, np.float16, q.shape).astype(np.float32)
    got_k = ds3.download(kb, np.float16, k.shape).astype(np.float32)
    assert_close(got_q, qo, rtol=2e-3, atol=1e-3, what="q fp16")
    assert_close(got_k, ko, rtol=2e-3, atol=1e-3, what="k fp16")


@pytest.mark.parametrize("T,nq,nk", [(2048, 32, 0), (3001, 16, 2), (2050, 5, 3)])
def test_qk_norm_rope_fp16_staged_head_splits(ds3, B, port, T, nq, nk):
    """The warp-specialised fp16 kernel (>= 2048 tokens) with no K heads and
    with other Q/K head splits, including an odd token count (ragged last tile)."""
    q = I.normal(17, (T, nq, 128)).astype(np.float16)
    k = I.normal(18, (T, max(nk, 1), 128))[:, :nk].astype(np.float16)
    qw, kw = I.gamma(128, 19), I.gamma(128, 20)
    pos = (np.arange(T, dtype=np.int32) * 7919) % 32768
    qb = B.up(q)
    kb = B.up(k) if nk else None
    assert ds3.qk_norm_rope(qb, kb, B.up(qw), B.up(kw), B.up(pos), T, nq, nk, 128, 1e6, 1e-6, F16) == 0
    qo, ko = port.qk_norm_rope(q.astype(np.float32), k.astype(np.float32), qw, kw, pos, 1e6, 1e-6)
    assert_close(ds3.download(qb, np.float16, q.shape).astype(np.float32), qo, rtol=2e-3, atol=1e-3, what="q fp16")
    if nk:
        assert_close(ds3.download(kb, np.float16, k.shape).astype(np.float32), ko, rtol=2e-3, atol=1e-3,
                     what="k fp16")


def test_rope_standalone(ds3, B, port):
    g = load_golden("qk_norm_rope.npz")
    T = g["q"].shape[0]
    src, dst, pos = B.up(g["q"]), B.empty(g["q"].nbytes), B.up(g["pos"])
    assert ds3.rope(src, dst, pos, 32, 128, T, 1e6) == 0
    assert_close(f32(dst, ds3, g["q"].shape), g["q_rope_only"], what="rope")
    assert ds3.rope(src, src, pos, 32, 128, T, 1e6) == 0  # src == dst
    assert_close(f32(src, ds3, g["q"].shape), g["q_rope_only"], what="rope in place")
    # reference test_metal.c shape: Q [4,32,128], positions 0,7,14,21
    q = I.normal(11, (4, 32, 128))
    p = np.array([0, 7, 14, 21], np.int32)
    qb = B.up(q)
    assert ds3.rope(qb, qb, B.up(p), 32, 128, 4, 1e6) == 0
    assert_close(f32(qb, ds3, q.shape), port.rope_rows(q, p, 1e6), what="rope 4x32")


# ----------------------------------------------------------------- router
def check_router(got_idx, got_sc, got_p, want_p, want_i, want_s):
    assert_bitexact(got_idx, want_i, "router idx")
    assert_close(got_sc, want_s, what="router scores")
    if got_p is not None:
        assert_close(got_p, want_p, what="router probs")


def test_router_golden(ds3, B):
    g = load_golden("router.npz")
    T = g["logits"].shape[0]
    lb, pb, ib, sb = B.up(g["logits"]), B.empty(T * 128 * 4), B.empty(T * 32), B.empty(T * 32)
    assert ds3.router_softmax_topk(lb, pb, ib, sb, T, 128, 8, True) == 0
    check_router(ds3.download(ib, np.int32, (T, 8)), f32(sb, ds3, (T, 8)), f32(pb, ds3, (T, 128)), g["probs"],
                 g["idx"], g["scores"])
    assert ds3.router_softmax_topk(lb, None, ib, sb, T, 128, 8, False) == 0
    check_router(ds3.download(ib, np.int32, (T, 8)), f32(sb, ds3, (T, 8)), None, None, g["idx_raw"],
                 g["scores_raw"])


@pytest.mark.parametrize("T,E,K", [(512, 128, 8), (1, 128, 8), (64, 128, 8), (33, 64, 4), (20, 256, 8),
                                   (9, 100, 8), (5, 128, 40), (7, 32, 32)])
def test_router_vs_oracle(ds3, B, port, T, E, K):
    lg = I.normal(T * E, (T, E), 0.0, 2.0)
    lb, pb, ib, sb = B.up(lg), B.empty(lg.nbytes), B.empty(T * K * 4), B.empty(T * K * 4)
    assert ds3.router_softmax_topk(lb, pb, ib, sb, T, E, K, True) == 0
    want = port.router(lg, K, True)
    check_router(ds3.download(ib, np.int32, (T, K)), f32(sb, ds3, (T, K)), f32(pb, ds3, (T, E)), *want)


def test_router_metal_batch_entry_points(ds3, B, port):
    L, T = 3, 10
    lg = I.normal(90, (L, T, 128), 0.0, 2.0)
    lb, ib, sb = B.up(lg), B.empty(L * T * 32), B.empty(L * T * 32)
    assert ds3.moe_router_topk_batch_tokens(lb, ib, sb, L, T, 128, 8, True) == 0
    _, wi, ws = port.router(lg.reshape(L * T, 128), 8, True)
    assert_bitexact(ds3.download(ib, np.int32, (L * T, 8)), wi)
    assert_close(f32(sb, ds3, (L * T, 8)), ws)
    assert ds3.moe_router_topk_batch(lb, ib, sb, L, 128, 8, True) == 0
    _, wi, ws = port.router(lg.reshape(L * T, 128)[:L], 8, True)  # [n_layers][n_expert] view
    assert_bitexact(ds3.download(ib, np.int32, (L, 8)), wi)


def test_router_ties_take_lowest_index(ds3, B, port):
    lg = np.zeros((2, 128), np.float32)
    lg[0, [5, 9, 77, 100]] = 3.0
    lg[1, :] = 1.0
    lb, ib, sb = B.up(lg), B.empty(2 * 32), B.empty(2 * 32)
    assert ds3.router_softmax_topk(lb, None, ib, sb, 2, 128, 8, True) == 0
    _, wi, ws = port.router(lg, 8, True)
    assert_bitexact(ds3.download(ib, np.int32, (2, 8)), wi)
    assert_close(f32(sb, ds3, (2, 8)), ws)


# ------------------------------------------------------------ SwiGLU / combine
@pytest.mark.parametrize("R,Cc,weighted", [(4096, 768, True), (512, 6144, False), (3, 5, True), (1, 1023, False),
                                         (7, 12, True), (40000, 768, True)])
def test_swiglu(ds3, B, port, R, Cc, weighted):
    g, u = I.normal(1, (R, Cc), 0, 1.5), I.normal(2, (R, Cc), 0, 1.5)
    rw = I.rng(3).uniform(0, 1, R).astype(np.float32) if weighted else None
    gb, ub, ob = B.up(g), B.up(u), B.empty(g.nbytes)
    assert ds3.swiglu(gb, ub, B.up(rw) if weighted else None, ob, R, Cc) == 0
    assert_close(f32(ob, ds3, g.shape), port.swiglu(g, u, rw), what="swiglu")


def test_swiglu_golden_and_silu_mul(ds3, B):
    g = load_golden("swiglu.npz")
    R, Cc = g["gate"].shape
    gb, ub, ob = B.up(g["gate"]), B.up(g["up"]), B.empty(g["gate"].nbytes)
    assert ds3.swiglu(gb, ub, B.up(g["row_w"]), ob, R, Cc) == 0
    assert_close(f32(ob, ds3, (R, Cc)), g["out"])
    assert ds3.silu_mul_f32(gb, ub, ob, R * Cc) == 0
    assert_close(f32(ob, ds3, (R, Cc)), g["out_plain"])


@pytest.mark.parametrize("T,K,Cc,mapped", [(512, 8, 2048, False), (64, 8, 2048, True), (5, 4, 256, False),
                                           (3, 8, 6, True), (7, 8, 2056, False), (1, 8, 36, False)])
def test_combine(ds3, B, port, T, K, Cc, mapped):
    y = I.normal(1, (T * K, Cc))
    w = I.rng(2).uniform(0, 1, (T, K)).astype(np.float32)
    r = I.normal(3, (T, Cc))
    rows = I.rng(4).permutation(T * K).astype(np.int32) if mapped else None
    yb, wb, rb, ob = B.up(y), B.up(w), B.up(r), B.empty(r.nbytes)
    assert ds3.moe_combine_residual(yb, B.up(rows) if mapped else None, wb, rb, ob, T, K, Cc) == 0
    assert_bitexact(f32(ob, ds3, r.shape), port.combine(y, w, r, rows), "combine")
    assert ds3.moe_combine_residual(yb, B.up(rows) if mapped else None, wb, rb, rb, T, K, Cc) == 0  # in place
    assert_bitexact(f32(rb, ds3, r.shape), port.combine(y, w, r, rows), "combine in place")


def test_combine_golden(ds3, B):
    g = load_golden("combine.npz")
    T, K = g["w"].shape
    Cc = g["residual"].shape[1]
    ob = B.empty(g["residual"].nbytes)
    assert ds3.moe_combine_residual(B.up(g["y"]), None, B.up(g["w"]), B.up(g["residual"]), ob, T, K, Cc) == 0
    assert_bitexact(f32(ob, ds3, (T, Cc)), g["out"])


# ------------------------------------------------------ Metal elementwise mirror
def test_elementwise_helpers(ds3, B, port):
    n = 1027
    a, b = I.normal(1, (n,)), I.normal(2, (n,))
    ab, bb, cb = B.up(a), B.up(b), B.empty(n * 4)
    assert ds3.vec_add(ab, bb, cb, n) == 0
    assert_bitexact(f32(cb, ds3, (n,)), a + b)
    assert ds3.vec_add_inplace(bb, ab, n) == 0
    assert_bitexact(f32(bb, ds3, (n,)), a + b)
    assert ds3.buffer_copy_f32(ab, cb, n * 4) == 0
    assert_bitexact(f32(cb, ds3, (n,)), a)
    assert ds3.buffer_zero_f32(cb, n * 4) == 0
    assert not f32(cb, ds3, (n,)).any()
    assert ds3.buffer_copy_f32(ab, cb, 6) == -1  # not a multiple of 4 bytes

    src = I.normal(3, (20, 64))
    ids = np.array([4, 0, 19, 4, 7, 3], np.int32)
    sb, ib, db = B.up(src), B.up(ids), B.empty(4 * 64 * 4)
    assert ds3.gather_rows_f32(sb, ib, db, 64, 4, 2) == 0  # rows ids[2:6]
    assert_bitexact(f32(db, ds3, (4, 64)), src[ids[2:6]])

    rows = I.normal(4, (3, 64))
    sc = np.array([0.5, 0.25, 2.0, -1.0], np.float32)
    uids = np.array([9, 2, 5, 11], np.int32)
    dst = I.normal(5, (12, 64))
    db2 = B.up(dst)
    assert ds3.scatter_add_weighted_f32(B.up(rows), B.up(sc), B.up(uids), db2, 64, 3, 1) == 0
    want = dst.copy()
    for i in range(3):
        want[uids[1 + i]] = want[uids[1 + i]] + sc[1 + i] * rows[i]
    assert_bitexact(f32(db2, ds3, (12, 64)), want)


# ------------------------------------------------ batch / graph / errors / timers
def test_batch_and_graph(ds3, B, port):
    x, r, w = I.normal(1, (32, 2048)), I.normal(2, (32, 2048)), I.gamma(2048, 3)
    xb, rb, wb, sb, nb = B.up(x), B.up(r), B.up(w), B.empty(x.nbytes), B.empty(x.nbytes)
    assert ds3.begin_batch() == 0
    assert ds3.begin_batch() == -1  # nested batch refused
    assert ds3.add_rms_norm(xb, rb, wb, sb, nb, 2048, 32, 1e-6) == 0
    assert ds3.rms_norm(nb, wb, nb, 2048, 32, 1e-6) == 0
    assert ds3.end_batch() == 0
    s_want, n_want = port.add_rms_norm(x, r, w, 1e-6)
    assert_close(f32(nb, ds3, x.shape), port.rms_norm_rows(n_want, w, 1e-6), rtol=3e-5)

    assert ds3.graph_begin() == 0
    assert ds3.timer_mark(0) == 0
    assert ds3.add_rms_norm(xb, rb, wb, sb, nb, 2048, 32, 1e-6) == 0
    assert ds3.timer_mark(1) == 0
    g = ds3.graph_end()
    ds3.buffer_zero_f32(sb, x.nbytes)
    for _ in range(3):
        assert ds3.graph_launch(g) == 0
    ds3.synchronize()
    assert ds3.timer_elapsed_ms(0, 1) > 0
    assert_bitexact(f32(sb, ds3, x.shape), s_want)
    ds3.graph_free(g)


def test_argument_errors(ds3, B):
    x = B.up(I.normal(1, (4, 128)))
    small = B.empty(16)
    w = B.up(I.gamma(128, 2))
    assert ds3.rms_norm(x, w, None, 128, 4, 1e-6) == -1
    assert ds3.rms_norm(x, w, small, 128, 4, 1e-6) == -1
    assert "needs" in ds3.last_error()
    assert ds3.rope(x, x, small, 1, 127, 4, 1e6) == -1  # odd head_dim
    assert ds3.router_softmax_topk(x, None, small, small, 4, 128, 0, True) == -1
    ro = ds3.buffer_from_mmap(np.zeros(64, np.uint8))
    try:
        assert ds3.buffer_write(ro, 0, np.ones(4, np.uint8)) == -1  # read-only
        assert ds3.rms_norm(x, w, ro, 16, 1, 1e-6) == -1
    finally:
        ro.free()
    v = ds3.buffer_view(x, 512, 512)
    try:
        assert ds3.download(v, np.float32, (128,)).shape == (128,)
        with pytest.raises(RuntimeError):
            ds3.buffer_view(x, 1024, 2048)  # past the end: NULL
    finally:
        v.free()


def test_kernels_are_sm100_code(ds3):
    # What the CUDA runtime reports for a kernel it loaded from the library.
    assert ds3.kernel_binary_version() == 100


def test_bounded_wait_gives_up_and_reports(ds3):
    # A wait on an mbarrier nothing completes must return after its poll
    # budget and raise the timeout bit, leaving the context usable.
    assert ds3.selftest_bounded_wait(2000) == 0
    assert ds3.device_errors() == 0
    x = ds3.upload(I.normal(1, (2, 128)))
    w = ds3.upload(I.gamma(128, 2))
    try:
        assert ds3.rms_norm(x, w, x, 128, 2, 1e-6) == 0  # context still healthy
    finally:
        x.free()
        w.free()


def test_async_copies_in_a_batch(ds3, B):
    x = I.normal(3, (64, 2048))
    w = I.gamma(2048, 4)
    xb, wb, ob = B.empty(x.nbytes), B.up(w), B.empty(x.nbytes)
    out = np.empty_like(x)
    assert ds3.begin_batch() == 0
    assert ds3.buffer_write_async(xb, 0, x) == 0
    assert ds3.rms_norm(xb, wb, ob, 2048, 64, 1e-6) == 0
    assert ds3.buffer_read_async(ob, 0, out) == 0
    assert ds3.end_batch() == 0
    assert_bitexact(out, f32(ob, ds3, x.shape), "async read")
    assert ds3.buffer_write_async(xb, 8, x) == -1  # past the end


@pytest.mark.parametrize("read_only_table", [False, True])
def test_embed_ids_written_by_the_previous_kernel(ds3, B, port, read_only_table):
    """The gather reads a hint of each id before its PDL wait. When the ids are
    the output of
    the kernel just before it (here a vec_add that copies new ids over old
    ones, bit patterns added to zero), a hint may be stale; the rows must
    still be those of the final ids."""
    vocab, T, n_cols = 4000, 512, 2048
    tab = I.q4k_table(vocab, n_cols, 71)
    if read_only_table:
        t = ds3.buffer_from_mmap(tab)
        B.all.append(t)
    else:
        t = B.up(tab)
    zeros = B.up(np.zeros(T, np.float32))
    dst = B.up(I.token_ids(T, 72, vocab))  # stale ids, valid but different
    out = B.empty(T * n_cols * 4)
    for rep in range(6):
        new = I.token_ids(T, 80 + rep, vocab)
        src = B.up(new)
        assert ds3.begin_batch() == 0
        assert ds3.vec_add(src, zeros, dst, T) == 0
        assert ds3.embed_rows(t, dst, out, T, n_cols, vocab, ds3.TYPE_Q4_K, 1152) == 0
        assert ds3.end_batch() == 0, ds3.last_error()
        want = port.embed_rows(tab, 12, 1152, vocab, new, n_cols)[1]
        assert_bitexact(f32(out, ds3, (T, n_cols)), want, f"rep {rep}")
        ds3.buffer_write(dst, 0, I.token_ids(T, 90 + rep, vocab))


def test_copy_lanes_pipeline(ds3, B, port):
    """Copy lanes: inputs uploaded on lane 1, the op on lane 0 after an event,
    results read on lane 2 after another, two buffer sets alternating, as
    bench.py's e2e pipeline does; every step's result equals the oracle's."""
    import torch

    n, steps = 1 << 16, 6
    xs = [torch.from_numpy(I.normal(300 + i, (n // 2048, 2048))).pin_memory().numpy() for i in range(steps)]
    rs = [torch.from_numpy(I.normal(400 + i, (n // 2048, 2048))).pin_memory().numpy() for i in range(steps)]
    w = B.up(I.gamma(2048, 5))
    outs = [torch.empty((n // 2048, 2048), dtype=torch.float32).pin_memory().numpy() for _ in range(steps)]
    sets = [(B.empty(n * 4), B.empty(n * 4), B.empty(n * 4)) for _ in range(2)]
    assert ds3.begin_batch() == 0
    for i in range(steps):
        s = i % 2
        x, r, o = sets[s]
        if i >= 2:
            assert ds3.lane_wait(1, 210 + s) == 0
        assert ds3.lane_write(1, x, 0, xs[i]) == 0 and ds3.lane_write(1, r, 0, rs[i]) == 0
        assert ds3.lane_record(1, 200 + s) == 0
        assert ds3.lane_wait(0, 200 + s) == 0
        if i >= 2:
            assert ds3.lane_wait(0, 220 + s) == 0
        assert ds3.add_rms_norm(x, r, w, None, o, 2048, n // 2048, 1e-6) == 0
        assert ds3.lane_record(0, 210 + s) == 0
        assert ds3.lane_wait(2, 210 + s) == 0
        assert ds3.lane_read(2, o, 0, outs[i]) == 0
        assert ds3.lane_record(2, 220 + s) == 0
    assert ds3.end_batch() == 0, ds3.last_error()
    for i in range(steps):
        _, want = port.add_rms_norm(xs[i], rs[i], I.gamma(2048, 5), 1e-6)
        assert_close(outs[i], want, what=f"step {i}")
    assert ds3.lane_write(3, sets[0][0], 0, xs[0]) == -1  # no such lane
