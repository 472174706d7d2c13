"""Tensor-parallel layout of the shift path: KV heads per rank and the shared segment table.

vLLM tensor parallelism gives rank ``r`` of ``tp`` the KV heads
``[r*H/tp, (r+1)*H/tp)`` of every layer, in its own paged cache; the store a
rank keeps for a session holds the same heads.  A shift load therefore touches
only rank-local memory: every rank runs the same segment table over its own
head shard and nothing crosses NVLink.  The only thing ranks must agree on is
the segment table itself.  Inside vLLM it arrives with the connector metadata
that vLLM broadcasts to every worker; a driver outside vLLM (the benchmark)
sends it once with :func:`broadcast_table`, a few hundred bytes.

The reference kept one store per worker and never ran under TP
(``src/marathon/vllm_shift_connector.py:49-50``); it had no collective at all.
"""

from __future__ import annotations

from datetime import timedelta

import numpy as np
import torch

#: columns of a packed segment table row
TABLE_COLUMNS = ("session", "store_start", "length", "delta", "paged_start")


def head_shard(heads: int, rank: int, world: int) -> tuple[int, int]:
    """``[lo, hi)`` KV heads of ``rank``; heads must divide evenly, as in vLLM TP."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if heads % world:
        raise ValueError(f"{heads} KV heads do not split over {world} ranks")
    per = heads // world
    return rank * per, (rank + 1) * per


def pack_table(runs) -> torch.Tensor:
    """Segment table of ``RunSpec``-like objects as an int64 ``[n, 5]`` tensor."""
    rows = [[int(getattr(r, c)) for c in TABLE_COLUMNS] for r in runs]
    return torch.tensor(rows, dtype=torch.int64).reshape(-1, len(TABLE_COLUMNS))


def unpack_table(t: torch.Tensor) -> list[dict]:
    return [dict(zip(TABLE_COLUMNS, map(int, row), strict=True)) for row in t.cpu().tolist()]


def broadcast_table(table: torch.Tensor | None, n_rows: int, *, src: int = 0, group=None,
                    device: torch.device | str = "cpu") -> torch.Tensor:
    """Every rank returns ``src``'s table; non-source ranks may pass ``None``.

    ``n_rows`` must be known on every rank (it is part of the step's plan); the
    call is one ``broadcast`` of ``n_rows * 5`` int64 values and raises if the
    process group's timeout expires (a rank that never arrives).
    """
    import torch.distributed as dist

    if dist.get_rank(group) == src:
        if table is None or table.shape != (n_rows, len(TABLE_COLUMNS)):
            raise ValueError("the source rank must pass the table it broadcasts")
        buf = table.to(device=device, dtype=torch.int64).contiguous()
    else:
        buf = torch.empty((n_rows, len(TABLE_COLUMNS)), dtype=torch.int64, device=device)
    dist.broadcast(buf, src=src, group=group)
    return buf


def shard_rows(x: np.ndarray | torch.Tensor, lo: int, hi: int, head_axis: int = -2):
    """Slice heads ``[lo, hi)`` out of a ``[..., heads, row]`` array (test / harness helper)."""
    index = [slice(None)] * x.ndim
    index[head_axis] = slice(lo, hi)
    return x[tuple(index)]


def default_timeout(seconds: float = 120.0) -> timedelta:
    """Process-group timeout used by the harnesses: a missing rank ends in an error."""
    return timedelta(seconds=seconds)
