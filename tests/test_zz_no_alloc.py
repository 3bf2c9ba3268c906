"""The allocation-free router entry point (ds3_cuda_moe_ffn_router_topk_noalloc)
against the regular one (ds3_cuda_moe_ffn_router_topk), through the C-ABI.

The no-alloc entry exists for callers that cannot let the library allocate
device memory (a host whose GPU memory is reserved up front by its own
allocator, or one that must not trigger an allocation mid-step). It keeps the
fp32 copy of a stored router weight in a fixed scratch array inside the
library instead of a workspace it allocates. Both entries must give the same
logits, top-8 indices and scores. Two calls in a row, with different weights
and stored types, check that the shared scratch is fully rewritten by each
call. This file is collected last, so a run that stops at the first failure
has already run every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import assert_bitexact, assert_close
from qw3_b200 import inputs as I

pytestmark = pytest.mark.gpu

F32, F16, Q80 = 0, 1, 8
E, K, N_USED = 128, 2048, 8


def stored(type_, seed):
    if type_ == F16:
        return I.normal(seed, (E, K), 0.0, 0.05).astype(np.float16).view(np.uint8)
    g = I.rng(seed)
    rows = g.integers(0, 256, (E, K // 32, 34), dtype=np.uint8)
    rows[:, :, 0:2] = g.uniform(0, 0.002, (E, K // 32, 1)).astype(np.float16).view(np.uint8)
    return rows.reshape(E, -1)


def test_noalloc_router_matches_regular_entry(ds3):
    keep = []

    def up(a):
        b = ds3.upload(np.ascontiguousarray(a))
        keep.append(b)
        return b

    try:
        for call, (type_, T) in enumerate([(Q80, 512), (F16, 64)]):
            x = I.normal(900 + call, (T, K))
            w = stored(type_, 910 + call)
            xb, wb = up(x), up(w)
            outs = []
            for fn in (ds3.moe_ffn_router_topk, ds3.moe_ffn_router_topk_noalloc):
                lb = up(np.zeros((T, E), np.float32))
                ib, sb = up(np.zeros((T, N_USED), np.int32)), up(np.zeros((T, N_USED), np.float32))
                assert fn(xb, wb, w.shape[1], type_, lb, ib, sb, T, K, E, N_USED, True) == 0, ds3.last_error()
                outs.append((ds3.download(lb, np.float32, (T, E)), ds3.download(ib, np.int32, (T, N_USED)),
                             ds3.download(sb, np.float32, (T, N_USED))))
            (l0, i0, s0), (l1, i1, s1) = outs
            assert_bitexact(l1, l0, f"logits, call {call}")
            assert_bitexact(i1, i0, f"top-8, call {call}")
            assert_close(s1, s0, what=f"scores, call {call}")
        # Beyond the fixed scratch: refused with a message, nothing launched.
        big_w = up(np.zeros((256, 4096 // 32 * 34), np.uint8))
        xb = up(np.zeros((1, 4096), np.float32))
        ib, sb = up(np.zeros((1, N_USED), np.int32)), up(np.zeros((1, N_USED), np.float32))
        assert ds3.moe_ffn_router_topk_noalloc(xb, big_w, 4096 // 32 * 34, Q80, None, ib, sb, 1, 4096, 256, N_USED,
                                               True) == -1
        assert "scratch" in ds3.last_error()
    finally:
        for b in keep:
            b.free()
    assert ds3.device_errors() == 0
