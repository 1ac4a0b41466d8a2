"""Market sharding across ranks (one process per GPU) and the to-root gather.

Markets are independent, so a multi-GPU run is G engines, one per rank, each
owning a contiguous block of global market ids; the matching step has no
collective.  The only collective is the optional gather of per-market outputs
(best bid/offer and int64 position/cash) to rank 0, which a learner would
consume; it runs over whatever backend the process group has (NCCL over
NVLink for CUDA tensors, gloo for CPU tensors in tests).

The reference has no multi-GPU layer beyond one VecMarket per device
(src/tests/integration/test_vec_market.py:361-413).
"""
from __future__ import annotations

import torch


def shard_range(rank: int, world: int, total: int) -> tuple[int, int]:
    """Global market ids [start, stop) owned by `rank` when `total` markets are
    split into `world` contiguous shards (the first total % world ranks hold
    one more)."""
    if not (0 <= rank < world):
        raise ValueError(f"rank {rank} outside [0, {world})")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _as_bytes(t: torch.Tensor) -> torch.Tensor:
    """Flat bytes of `t`, zero-padded to a multiple of 16 so every part of the
    payload starts aligned for its dtype."""
    b = t.contiguous().reshape(-1).view(torch.uint8)
    pad = (-b.numel()) % 16
    if pad:
        b = torch.cat([b, torch.zeros(pad, dtype=torch.uint8, device=b.device)])
    return b


def gather_to_root(parts, group=None, dst: int = 0):
    """Gather each rank's tensors to rank `dst` in one collective.

    `parts` is a list of tensors with the same shapes and dtypes on every rank,
    market-major along dimension 0 except for tensors marked market-minor by
    passing ``(tensor, 1)``.  On `dst` returns the list of concatenations over
    ranks (rank order) along each tensor's market dimension; elsewhere None.
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    norm = [(p, 0) if isinstance(p, torch.Tensor) else (p[0], int(p[1])) for p in parts]
    payload = torch.cat([_as_bytes(t) for t, _ in norm])
    bufs = [torch.empty_like(payload) for _ in range(world)] if rank == dst else None
    dist.gather(payload, bufs, dst=dst, group=group)
    if rank != dst:
        return None
    out = []
    off = 0
    for t, dim in norm:
        nb = t.numel() * t.element_size()
        pieces = [b[off:off + nb].view(t.dtype).view(t.shape) for b in bufs]
        out.append(torch.cat(pieces, dim=dim))
        off += nb + (-nb) % 16
    return out
