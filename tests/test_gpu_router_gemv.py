"""Router projection fused with softmax/top-k (ds3_cuda_router_logits_topk):
logits bit-exact with the reference's sequential vec_matmul (restated in the
oracle), top-k indices exact, scores within the fp32 tolerance."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_bitexact, assert_close
from qw3_b200 import inputs as I

pytestmark = pytest.mark.gpu


@pytest.fixture
def up(ds3):
    keep = []

    def f(a):
        b = ds3.upload(np.ascontiguousarray(a))
        keep.append(b)
        return b

    yield f
    for b in keep:
        b.free()
    assert ds3.device_errors() == 0


@pytest.mark.parametrize("T,K,E,n_used,with_logits", [(512, 2048, 128, 8, True), (512, 2048, 128, 8, False),
                                                      (1, 2048, 128, 8, True), (67, 1024, 128, 8, True),
                                                      (13, 100, 64, 4, True), (5, 2048, 32, 8, True),
                                                      (70, 2080, 128, 8, True), (1000, 2048, 128, 8, True)])
def test_router_logits_topk(ds3, up, port, T, K, E, n_used, with_logits):
    x = I.normal(T + K, (T, K))
    W = I.normal(E + 7, (E, K), 0.0, 0.05)
    lg = port.router_logits(x, W, 8)
    _, want_i, want_s = port.router(lg, n_used, True)
    lb = up(np.zeros((T, E), np.float32)) if with_logits else None
    ib, sb = up(np.zeros((T, n_used), np.int32)), up(np.zeros((T, n_used), np.float32))
    rc = ds3.router_logits_topk(up(x), up(W), lb, ib, sb, T, K, E, n_used, True)
    assert rc == 0, ds3.last_error()
    if with_logits:
        assert_bitexact(ds3.download(lb, np.float32, (T, E)), lg, "logits")
    assert_bitexact(ds3.download(ib, np.int32, (T, n_used)), want_i, "top-k")
    assert_close(ds3.download(sb, np.float32, (T, n_used)), want_s, what="scores")


def test_router_logits_topk_needs_logits_off_the_fast_path(ds3, up):
    x, W = I.normal(1, (4, 100)), I.normal(2, (64, 100))
    ib, sb = up(np.zeros((4, 4), np.int32)), up(np.zeros((4, 4), np.float32))
    assert ds3.router_logits_topk(up(x), up(W), None, ib, sb, 4, 100, 64, 4, True) == -1
    # 128 experts but n_embd not a multiple of 64: also the general path.
    x2, W2 = I.normal(3, (4, 2080)), I.normal(4, (128, 2080))
    ib2, sb2 = up(np.zeros((4, 8), np.int32)), up(np.zeros((4, 8), np.float32))
    assert ds3.router_logits_topk(up(x2), up(W2), None, ib2, sb2, 4, 2080, 128, 8, True) == -1
