"""Row sharding of a projection across GPUs, one process per GPU.

Rows of a GGUF matrix are independent and each row is a whole number of quant
blocks, so a projection splits into contiguous row ranges: rank r owns rows
[start, end) — whole blocks — and computes y[:, start:end]; the full output is
assembled with one all-gather (NCCL over NVLink on B200, gloo in CPU tests).

The helpers here are the plumbing; the per-rank compute is any backend call
(``DeviceWeight.matmul`` or ``frc_gemv`` on the rank's GPU).
"""

from __future__ import annotations

from typing import Any

import numpy as np

from .synth import row_bytes


def row_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced row range of `rank` (sizes differ by at most 1)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    return (n * rank) // world, (n * (rank + 1)) // world


def shard_bytes(raw: np.ndarray, quant: str, n: int, k: int, world: int, rank: int) -> np.ndarray:
    """The raw GGUF bytes of rank's rows: a contiguous slice (no copy)."""
    rb = row_bytes(quant, k)
    start, end = row_range(n, world, rank)
    flat = np.asarray(raw).reshape(-1)
    if flat.size != n * rb:
        raise ValueError(f"{quant}: expected {n * rb} bytes for ({n}, {k}), got {flat.size}")
    return flat[start * rb:end * rb]


def assemble(gathered: Any, world: int, batch: int, n_local: int) -> Any:
    """(world * batch * n_local) gathered in rank order -> (batch, world * n_local).

    ``all_gather_into_tensor`` concatenates the ranks' (batch, n_local) blocks
    along the first axis; rows of y belong to ranks, so the rank axis moves
    inside each batch row.  Works on torch tensors and NumPy arrays."""
    if isinstance(gathered, np.ndarray):
        return gathered.reshape(world, batch, n_local).transpose(1, 0, 2).reshape(batch, world * n_local)
    return gathered.reshape(world, batch, n_local).permute(1, 0, 2).reshape(batch, world * n_local)


def sharded_matmul(local_matmul, x: Any, n: int, world: int, group=None):
    """y = W x with W row-sharded: `local_matmul(x)` returns this rank's
    (batch, n_local) block (equal shards required); the blocks are
    all-gathered with torch.distributed and assembled to (batch, n)."""
    import torch
    import torch.distributed as dist

    y_local = local_matmul(x)
    y_local = y_local if isinstance(y_local, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(y_local))
    y2 = y_local.reshape(-1, y_local.shape[-1]).contiguous()
    batch, n_local = y2.shape
    if n_local * world != n:
        raise ValueError(f"equal shards required: {n_local} x {world} != {n}")
    out = torch.empty(world * batch * n_local, dtype=y2.dtype, device=y2.device)
    dist.all_gather_into_tensor(out, y2.reshape(-1), group=group)
    return assemble(out, world, batch, n_local)


__all__ = ["row_range", "shard_bytes", "assemble", "sharded_matmul"]
