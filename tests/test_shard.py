"""Row sharding across ranks (qw3_b200/shard.py): ranges cover every row
once, and a world_size-2 gloo run — each rank computing its slice with the
oracle, then the verification all-gather — reproduces the single-process
result bit for bit. Rows are independent, so no other exchange exists."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from qw3_b200.shard import shard_range, shard_sizes


@pytest.mark.parametrize("n,world", [(512, 8), (32768, 8), (64, 8), (7, 3), (0, 2), (5, 8)])
def test_ranges_partition_rows(n, world):
    seen = []
    for r in range(world):
        a, b = shard_range(n, world, r)
        assert 0 <= a <= b <= n
        seen.extend(range(a, b))
    assert seen == list(range(n))
    assert max(shard_sizes(n, world)) - min(shard_sizes(n, world)) <= 1


def test_bad_rank_rejected():
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, n_rows, out_path):
    import torch
    import torch.distributed as dist

    import oracle
    from qw3_b200 import inputs as I
    from qw3_b200.shard import gather_rows

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    P = oracle.port()
    x, r, w = I.normal(1, (n_rows, 2048)), I.normal(2, (n_rows, 2048)), I.gamma(2048, 3)
    q, k = I.normal(4, (n_rows, 32, 128)), I.normal(5, (n_rows, 4, 128))
    pos = np.arange(n_rows, dtype=np.int32)
    a, b = shard_range(n_rows, world, rank)
    _, nrm = P.add_rms_norm(x[a:b], r[a:b], w, 1e-6)
    qo, _ = P.qk_norm_rope(q[a:b], k[a:b], I.gamma(128, 6), I.gamma(128, 7), pos[a:b], 1e6, 1e-6)
    full_n = gather_rows(torch.from_numpy(nrm), n_rows).numpy()
    full_q = gather_rows(torch.from_numpy(qo), n_rows).numpy()
    if rank == 0:
        np.savez(out_path, norm=full_n, q=full_q)
    dist.destroy_process_group()


def test_gloo_two_ranks_match_single_process(tmp_path, port):
    import oracle  # noqa: F401
    from qw3_b200 import inputs as I

    n_rows = 37  # uneven split
    out = tmp_path / "g.npz"
    mp.spawn(_worker, args=(2, _free_port(), n_rows, str(out)), nprocs=2, join=True)
    got = np.load(out)
    x, r, w = I.normal(1, (n_rows, 2048)), I.normal(2, (n_rows, 2048)), I.gamma(2048, 3)
    _, want_n = port.add_rms_norm(x, r, w, 1e-6)
    q, k = I.normal(4, (n_rows, 32, 128)), I.normal(5, (n_rows, 4, 128))
    want_q, _ = port.qk_norm_rope(q, k, I.gamma(128, 6), I.gamma(128, 7), np.arange(n_rows, dtype=np.int32), 1e6,
                                  1e-6)
    assert np.array_equal(got["norm"], want_n)
    assert np.array_equal(got["q"], want_q)


def _quitter(rank, world, port, out_path):
    import datetime

    import torch
    import torch.distributed as dist

    from qw3_b200.shard import gather_rows

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        return  # leaves between steps, without joining the gather
    try:
        gather_rows(torch.zeros((3, 4)), 6)
        status = "completed"
    except Exception as e:  # the survivor must see an error, not hang
        status = "error: " + type(e).__name__
    with open(out_path, "w") as f:
        f.write(status)


def test_rank_that_quits_makes_the_gather_fail_not_hang(tmp_path):
    out = tmp_path / "status.txt"
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_quitter, args=(r, 2, port, str(out))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode is not None for p in procs), "a rank hung"
    assert out.read_text().startswith("error"), out.read_text()
