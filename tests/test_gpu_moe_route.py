"""Device-side per-expert token lists (ds3_cuda_moe_expert_lists) against the
engine's host loop (restated in the oracle), and the gathered-MoE flow they
enable: lists -> gather rows per expert -> expert outputs -> combine through
the slot map, equal to the combine of token-major expert outputs."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import assert_bitexact
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


def route(ds3, up, port, T, E, K, seed):
    lg = I.normal(seed, (T, E), 0.0, 2.0)
    _, idx, sc = port.router(lg, K, True)
    cap = T
    fill = np.full(E * cap, -7, np.int32)
    fills = np.full(E * cap, np.nan, np.float32)
    cb, ib, gb, sb = up(np.zeros(E, np.int32)), up(fill), up(fills), up(np.zeros(T * K, np.int32))
    assert ds3.moe_expert_lists(up(idx), up(sc), cb, ib, gb, sb, T, E, K, cap) == 0, ds3.last_error()
    got = (ds3.download(cb, np.int32, (E,)), ds3.download(ib, np.int32, (E * cap,)),
           ds3.download(gb, np.float32, (E * cap,)), ds3.download(sb, np.int32, (T * K,)))
    want = oracle.moe_expert_lists(port, idx, sc, E, cap)
    return idx, sc, got, want


@pytest.mark.parametrize("T,E,K", [(512, 128, 8), (1, 128, 8), (3000, 128, 8), (37, 64, 4), (130, 256, 8)])
def test_expert_lists_match_engine_loop(ds3, up, port, T, E, K):
    _, _, got, want = route(ds3, up, port, T, E, K, seed=T + E)
    assert want[0] == 0
    for g, w, name in zip(got, want[1:], ("counts", "ids", "gscores", "slot_of")):
        assert_bitexact(g, w, name)


def test_expert_lists_reject_bad_ids(ds3, up):
    idx = np.array([[1, 300]], np.int32)
    sc = np.ones((1, 2), np.float32)
    rc = ds3.moe_expert_lists(up(idx), up(sc), up(np.zeros(128, np.int32)), up(np.zeros(128, np.int32)),
                              up(np.zeros(128, np.float32)), None, 1, 128, 2, 1)
    assert rc == -1


def test_gathered_flow_equals_token_major_combine(ds3, up, port):
    T, E, K, H = 64, 128, 8, 256
    idx, sc, (counts, ids, gs, slot), _ = route(ds3, up, port, T, E, K, seed=9)
    x = I.normal(10, (T, H))
    xb = up(x)
    cap = T
    # Gather each expert's token rows into the per-expert layout (engine :973).
    gathered = up(np.zeros((E * cap, H), np.float32))
    idsb = up(ids)
    for ex in range(E):
        c = int(counts[ex])
        if c:
            view = ds3.buffer_view(gathered, ex * cap * H * 4, c * H * 4)
            assert ds3.gather_rows_f32(xb, idsb, view, H, c, ex * cap) == 0
            view.free()
    g = ds3.download(gathered, np.float32, (E * cap, H))
    # Stand-in expert: y = row * (1 + ex); compute both layouts on the host.
    ex_of_slot = np.repeat(np.arange(E), cap)
    y_exp = (g * (1.0 + ex_of_slot)[:, None]).astype(np.float32)
    y_tok = (x[np.repeat(np.arange(T), K)] * (1.0 + idx.reshape(-1))[:, None]).astype(np.float32)
    r = I.normal(11, (T, H))
    o1, o2 = up(np.zeros((T, H), np.float32)), up(np.zeros((T, H), np.float32))
    assert ds3.moe_combine_residual(up(y_exp), up(slot), up(sc), up(r), o1, T, K, H) == 0
    assert ds3.moe_combine_residual(up(y_tok), None, up(sc), up(r), o2, T, K, H) == 0
    assert_bitexact(ds3.download(o1, np.float32, (T, H)), ds3.download(o2, np.float32, (T, H)), "combine")
    assert_bitexact(ds3.download(o2, np.float32, (T, H)), port.combine(y_tok, sc, r), "oracle")
