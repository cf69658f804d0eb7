"""(batch x head) sharding across ranks.

Every (b, KV head) unit is independent through the whole path (coarsening, FRC, top-k and
attention touch one head's Q/K/V only; for GQA the query heads of one KV group stay
together), so ranks take contiguous ranges of units and exchange nothing. The only
collective is the optional gather of per-rank outputs for a caller that needs the whole
tensor on every rank.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def unit_range(num_units: int, world_size: int, rank: int):
    """Contiguous, balanced [start, end) range of units for ``rank``."""
    if not 0 <= rank < world_size:
        raise ValueError("rank outside [0, world_size)")
    base, extra = divmod(num_units, world_size)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def units_to_slices(start: int, end: int, Hkv: int):
    """Split a flat unit range (unit = b * Hkv + g) into per-batch (b, g0, g1) slices."""
    out = []
    u = start
    while u < end:
        b, g0 = divmod(u, Hkv)
        g1 = min(Hkv, g0 + (end - u))
        out.append((b, g0, g1))
        u += g1 - g0
    return out


def gather_units(local: torch.Tensor, num_units: int, group=None) -> torch.Tensor:
    """All-gather per-rank unit slabs ``local [n_local, ...]`` into ``[num_units, ...]``
    (ranks hold contiguous ranges from ``unit_range``; uneven ranges are padded)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    counts = [unit_range(num_units, world, r)[1] - unit_range(num_units, world, r)[0]
              for r in range(world)]
    assert local.shape[0] == counts[rank]
    cmax = max(counts)
    padded = torch.zeros((cmax,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    bufs = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(bufs, padded, group=group)
    return torch.cat([bufs[r][: counts[r]] for r in range(world)], dim=0)
