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


def test_combine_row_map_out_of_range(ds3, up, port):
    """A row map holding -1 (what moe_expert_lists leaves for a bad id or a
    full list) or an index past y's last row: those rows count as zero, y is
    never read outside its buffer, and the call returns -1."""
    T, K, H = 6, 8, 256
    n_y = T * K
    y = I.normal(21, (n_y, H))
    w = I.rng(22).uniform(0, 1, (T, K)).astype(np.float32)
    r = I.normal(23, (T, H))
    rows = I.rng(24).permutation(n_y).astype(np.int32).reshape(T, K)
    rows[1, 3] = -1
    rows[4, 0] = n_y
    rows[5, 7] = 1 << 30
    o = up(np.zeros((T, H), np.float32))
    assert ds3.moe_combine_residual(up(y), up(rows), up(w), up(r), o, T, K, H) == -1
    # Expected: the bad entries read an all-zero row appended to y.
    y_ext = np.concatenate([y, np.zeros((1, H), np.float32)])
    fixed = np.where((rows < 0) | (rows >= n_y), n_y, rows).astype(np.int32)
    assert_bitexact(ds3.download(o, np.float32, (T, H)), port.combine(y_ext, w, r, fixed.reshape(-1)), "zero rows")
    # The error word was consumed by the failing call; a good call succeeds.
    assert ds3.moe_combine_residual(up(y), up(fixed % n_y), up(w), up(r), o, T, K, H) == 0


def test_expert_lists_counts_clamped_to_cap(ds3, up, port):
    """A list that overflows its capacity: counts[ex] stays <= cap, the
    overflowing slots get -1 and the call returns -1."""
    T, E, K, cap = 8, 16, 2, 4
    idx = np.tile(np.array([[3, 5]], np.int32), (T, 1))  # expert 3 and 5 chosen by all 8 tokens
    sc = np.full((T, K), 0.5, np.float32)
    cb, ib, gb, sb = (up(np.zeros(E, np.int32)), up(np.zeros(E * cap, np.int32)), up(np.zeros(E * cap, np.float32)),
                      up(np.zeros(T * K, np.int32)))
    assert ds3.moe_expert_lists(up(idx), up(sc), cb, ib, gb, sb, T, E, K, cap) == -1
    counts = ds3.download(cb, np.int32, (E,))
    assert counts[3] == cap and counts[5] == cap and counts.max() == cap
    slot = ds3.download(sb, np.int32, (T, K))
    assert (slot[:cap, 0] == 3 * cap + np.arange(cap)).all() and (slot[cap:, :] == -1).all()
    rc, want_counts, _, _, want_slot = oracle.moe_expert_lists(port, idx, sc, E, cap)
    assert rc == -1
    assert_bitexact(counts, want_counts, "counts")
    assert_bitexact(slot.reshape(-1), want_slot, "slot_of")
