"""Multi-GPU row sharding on real devices: each rank runs its contiguous
slice of tokens through the C-ABI on its own GPU, and the verification
all-gather (NCCL) reassembles outputs equal to the oracle's over all rows.
Skipped when fewer than two GPUs are visible."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, n_rows, out):
    import torch
    import torch.distributed as dist

    from qw3_b200 import ds3, inputs as I
    from qw3_b200.shard import gather_rows, shard_range

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    assert ds3.set_device(rank) == 0 and ds3.init() == 0, ds3.last_error()
    a, b = shard_range(n_rows, world, rank)
    m = b - a
    tab = I.q4k_table(2000, 2048, 1)
    ids = I.token_ids(n_rows, 2, 2000)[a:b]
    w = I.gamma(2048, 3)
    q = I.normal(4, (n_rows, 32, 128))[a:b]
    k = I.normal(5, (n_rows, 4, 128))[a:b]
    pos = np.arange(a, b, dtype=np.int32)
    hid = torch.empty((m, 2048), device="cuda")
    nrm = torch.empty((m, 2048), device="cuda")
    qt = torch.from_numpy(np.ascontiguousarray(q)).cuda()
    kt = torch.from_numpy(np.ascontiguousarray(k)).cuda()
    torch.cuda.synchronize()
    T = ds3.buffer_from_mmap(tab)
    ib, wb, pb = ds3.upload(ids), ds3.upload(w), ds3.upload(pos)
    hb, nb = ds3.buffer_wrap(hid.data_ptr(), hid.numel() * 4), ds3.buffer_wrap(nrm.data_ptr(), nrm.numel() * 4)
    qb, kb = ds3.buffer_wrap(qt.data_ptr(), qt.numel() * 4), ds3.buffer_wrap(kt.data_ptr(), kt.numel() * 4)
    qw, kw = ds3.upload(I.gamma(128, 6)), ds3.upload(I.gamma(128, 7))
    assert ds3.embed_rms_norm(T, ib, wb, hb, nb, m, 2048, 2000, ds3.TYPE_Q4_K, 1152, 1e-6) == 0
    assert ds3.qk_norm_rope(qb, kb, qw, kw, pb, m, 32, 4, 128, 1e6, 1e-6) == 0
    full_h = gather_rows(hid, n_rows).cpu().numpy()
    full_q = gather_rows(qt, n_rows).cpu().numpy()
    if rank == 0:
        np.savez(out, hidden=full_h, q=full_q)
    dist.destroy_process_group()


def test_two_gpus_row_shard_matches_oracle(tmp_path, port):
    import torch
    import torch.multiprocessing as mp

    from qw3_b200 import inputs as I

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    n_rows = 301
    out = tmp_path / "m.npz"
    mp.spawn(_rank, args=(2, _free_port(), n_rows, str(out)), nprocs=2, join=True)
    got = np.load(out)
    tab = I.q4k_table(2000, 2048, 1)
    _, hid = port.embed_rows(tab, 12, 1152, 2000, I.token_ids(n_rows, 2, 2000), 2048)
    assert np.array_equal(got["hidden"], hid)
    qo, _ = port.qk_norm_rope(I.normal(4, (n_rows, 32, 128)), I.normal(5, (n_rows, 4, 128)), I.gamma(128, 6),
                              I.gamma(128, 7), np.arange(n_rows, dtype=np.int32), 1e6, 1e-6)
    err = np.abs(got["q"] - qo) / (1e-6 + 1e-5 * np.abs(qo))
    assert err.max() <= 1.0
