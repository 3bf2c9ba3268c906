"""Row (token) sharding across GPUs for the per-layer path.

Every op of the path is independent per token row (per (token, head) for
QK-norm + RoPE), so N GPUs each run the unchanged kernels on a contiguous
slice of rows and nothing is exchanged while they run. A collective is used
only to bring the slices back together for verification (``gather_rows``).
"""

from __future__ import annotations


def shard_range(n_rows: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) of ``n_rows`` owned by ``rank`` of ``world``;
    the first ``n_rows % world`` ranks take one extra row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    if n_rows < 0:
        raise ValueError("n_rows must be >= 0")
    base, extra = divmod(n_rows, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


def shard_sizes(n_rows: int, world: int) -> list[int]:
    return [b - a for a, b in (shard_range(n_rows, world, r) for r in range(world))]


def gather_rows(local, n_rows: int, group=None):
    """All-gather row shards of a torch tensor ``local`` ([rows_r, ...]) into
    the full [n_rows, ...] tensor on every rank (verification only; uneven
    shards are padded to the largest one for the collective)."""
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    sizes = shard_sizes(n_rows, world)
    m = max(sizes)
    pad = torch.zeros((m,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return torch.cat([p[:s] for p, s in zip(parts, sizes)], dim=0)
