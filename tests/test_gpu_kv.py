"""GPU parity of the KV-cache writers: the standalone batch write (mirror of
ds3_metal_kv_cache_write_batch) and the write fused into QK-norm + RoPE.
Cache contents are fp16 and compared bit for bit; rows the call does not own
must keep their previous contents."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import assert_bitexact, assert_close
from qw3_b200 import inputs as I

pytestmark = pytest.mark.gpu
SENT = 0x7E00  # fp16 NaN pattern marking untouched cache rows


@pytest.fixture
def bufs(ds3):
    keep = []

    def up(a):
        b = ds3.upload(np.ascontiguousarray(a))
        keep.append(b)
        return b

    yield up
    for b in keep:
        b.free()
    assert ds3.device_errors() == 0


@pytest.mark.parametrize("seq_pos,T,max_seq", [(0, 64, 64), (100, 17, 4096), (7, 1, 8)])
def test_kv_cache_write_batch(ds3, bufs, port, seq_pos, T, max_seq):
    k, v = I.normal(1, (T, 4, 128), 0, 3), I.normal(2, (T, 4, 128), 0, 3)
    ck = np.full((max_seq, 4, 128), SENT, np.uint16)
    cv = ck.copy()
    kc, vc = bufs(ck), bufs(cv)
    assert ds3.kv_cache_write_batch(bufs(k), bufs(v), kc, vc, seq_pos, T, max_seq, 32, 4, 128) == 0
    oracle.kv_cache_write(port, k, v, ck, cv, seq_pos=seq_pos)
    assert_bitexact(ds3.download(kc, np.uint16, ck.shape), ck, "k cache")
    assert_bitexact(ds3.download(vc, np.uint16, cv.shape), cv, "v cache")
    assert ds3.kv_cache_write_batch(bufs(k), bufs(v), kc, vc, max_seq - T + 1, T, max_seq, 32, 4, 128) == -1


@pytest.mark.parametrize("T,storage", [(64, 0), (17, 0), (512, 0), (33, 1)])
def test_qk_norm_rope_kv(ds3, bufs, port, T, storage):
    dt = np.float16 if storage else np.float32
    max_seq = 4096
    q, k, v = I.normal(3, (T, 32, 128)), I.normal(4, (T, 4, 128)), I.normal(5, (T, 4, 128))
    q, k, v = q.astype(dt), k.astype(dt), v.astype(dt)
    qw, kw = I.gamma(128, 6), I.gamma(128, 7)
    pos = I.rng(8).permutation(max_seq)[:T].astype(np.int32)  # distinct cache rows
    ck = np.full((max_seq, 4, 128), SENT, np.uint16)
    cv = ck.copy()
    qb, kb, vb, kc, vc = bufs(q), bufs(k), bufs(v), bufs(ck), bufs(cv)
    rc = ds3.qk_norm_rope_kv(qb, kb, vb, bufs(qw), bufs(kw), bufs(pos), kc, vc, T, 32, 4, 128, max_seq, 1e6, 1e-6,
                             storage)
    assert rc == 0, ds3.last_error()
    qo, ko = port.qk_norm_rope(q.astype(np.float32), k.astype(np.float32), qw, kw, pos, 1e6, 1e-6)
    got_q = ds3.download(qb, dt, q.shape).astype(np.float32)
    got_k = ds3.download(kb, dt, k.shape)
    tol = dict(rtol=2e-3, atol=1e-3) if storage else {}
    assert_close(got_q, qo, what="q", **tol)
    assert_close(got_k.astype(np.float32), ko, what="k", **tol)
    assert_bitexact(ds3.download(vb, dt, v.shape), v, "v untouched")
    # The cache holds exactly the fp16 rounding of the k the call returned,
    # and of v; every other row is untouched.
    want_k = np.full_like(ck, SENT)
    want_v = np.full_like(cv, SENT)
    oracle.kv_cache_write(port, got_k.astype(np.float32), v.astype(np.float32), want_k, want_v, row_of=pos)
    assert_bitexact(ds3.download(kc, np.uint16, ck.shape), want_k, "k cache")
    assert_bitexact(ds3.download(vc, np.uint16, cv.shape), want_v, "v cache")


def test_qk_norm_rope_kv_rejects_bad_positions(ds3, bufs):
    T, max_seq = 4, 16
    q, k, v = I.normal(3, (T, 32, 128)), I.normal(4, (T, 4, 128)), I.normal(5, (T, 4, 128))
    pos = np.array([0, 3, 16, 2], np.int32)  # 16 is past the cache
    ck = np.full((max_seq, 4, 128), SENT, np.uint16)
    kc = bufs(ck)
    rc = ds3.qk_norm_rope_kv(bufs(q), bufs(k), bufs(v), bufs(I.gamma(128, 6)), bufs(I.gamma(128, 7)), bufs(pos), kc,
                             bufs(ck), T, 32, 4, 128, max_seq, 1e6, 1e-6)
    assert rc == -1
    got = ds3.download(kc, np.uint16, ck.shape)
    assert (got[[0, 3, 2]] != SENT).all() and (got[[1] + list(range(4, 16))] == SENT).all()
    assert ds3.qk_norm_rope_kv(bufs(q), bufs(k), bufs(v), bufs(I.gamma(128, 6)), bufs(I.gamma(128, 7)), bufs(pos),
                               kc, bufs(ck), T, 32, 4, 64, max_seq, 1e6, 1e-6) == -1  # head_dim 64
