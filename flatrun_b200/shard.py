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


class _DevArray:
    """A raw device allocation described by __cuda_array_interface__."""

    def __init__(self, ptr: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3}


class FusedGather:
    """Row-sharded outputs assembled by the GEMV itself over NVLink.

    One per projection group and rank.  Every rank owns `shard_floats` floats
    of output (its rows of the group's matrices, laid out contiguously in a
    local buffer); the gathered buffer holds `world` such shards in rank
    order.  Set-up exchanges CUDA IPC handles of the gathered buffers and flag
    arrays over `group` (any torch.distributed backend) and maps the peers'.
    Per use: `gemv(...)` (the fused batch-1 launch that stores every y value
    into all ranks' gathered buffers) then `wait(stream)`.  Every rank must
    issue the same sequence of calls.
    """

    def __init__(self, lib, world: int, rank: int, shard_floats: int, group=None):
        import ctypes

        import torch.distributed as dist

        from . import _lib

        self._lib, self.world, self.rank, self.shard_floats = lib, world, rank, shard_floats
        self._own, self._peers, self.handle = [], [], None
        hb = ctypes.create_string_buffer(64)
        hf = ctypes.create_string_buffer(64)
        buf, flg = ctypes.c_void_p(), ctypes.c_void_p()
        _lib.check(lib.frc_ipc_alloc(world * shard_floats * 4, ctypes.byref(buf), hb), lib)
        self._own.append(buf.value)
        _lib.check(lib.frc_ipc_alloc(world * 4, ctypes.byref(flg), hf), lib)
        self._own.append(flg.value)
        self.buffer_ptr = buf.value
        handles = [None] * world
        dist.all_gather_object(handles, (hb.raw, hf.raw), group=group)
        shard_dst, flags = [], []
        for r in range(world):
            if r == rank:
                b, f = buf.value, flg.value
            else:
                pb, pf = ctypes.c_void_p(), ctypes.c_void_p()
                _lib.check(lib.frc_ipc_open(handles[r][0], ctypes.byref(pb)), lib)
                self._peers.append(pb.value)
                _lib.check(lib.frc_ipc_open(handles[r][1], ctypes.byref(pf)), lib)
                self._peers.append(pf.value)
                b, f = pb.value, pf.value
            shard_dst.append(b + rank * shard_floats * 4)
            flags.append(f)
        g = ctypes.c_void_p()
        _lib.check(lib.frc_gather_create(world, rank, (ctypes.c_void_p * world)(*shard_dst),
                                         (ctypes.c_void_p * world)(*flags), ctypes.byref(g)), lib)
        self.handle = g

    def gathered(self):
        """The gathered buffer (world * shard_floats floats) as a torch tensor view."""
        import torch
        return torch.as_tensor(_DevArray(self.buffer_ptr, (self.world * self.shard_floats,), "<f4"), device="cuda")

    def gemv(self, quant_id: int, w_ptrs, w_bytes, ns, k: int, x_ptr: int, y_ptrs, y_base: int, stream: int,
             wait_for: "FusedGather | None" = None) -> int:
        """frc_gemv_gather: returns the status (FRC_ERR_UNSUPPORTED when the
        shape has no fused path).  `wait_for`: an earlier gather whose result
        the GEMV waits for before reading x."""
        import ctypes
        c = len(w_ptrs)
        return self._lib.frc_gemv_gather(quant_id, c, (ctypes.c_void_p * c)(*w_ptrs), (ctypes.c_size_t * c)(*w_bytes),
                                         (ctypes.c_int64 * c)(*ns), k, x_ptr, (ctypes.c_void_p * c)(*y_ptrs), y_base,
                                         self.handle, wait_for.handle if wait_for is not None else None,
                                         ctypes.c_void_p(stream))

    def wait(self, stream: int) -> None:
        import ctypes

        from . import _lib
        _lib.check(self._lib.frc_gather_wait(self.handle, ctypes.c_void_p(stream)), self._lib)

    def close(self) -> None:
        """Frees the gather; call on every rank after a device synchronise and
        a barrier, so no peer still writes into this rank's buffers."""
        if self.handle is not None:
            self._lib.frc_gather_free(self.handle)
            self.handle = None
        for p in self._peers:
            self._lib.frc_ipc_close(p)
        for p in self._own:
            self._lib.frc_ipc_free(p)
        self._peers, self._own = [], []


__all__ = ["row_range", "shard_bytes", "assemble", "sharded_matmul", "FusedGather"]
