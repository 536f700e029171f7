"""Row sharding + all-gather assembly on two gloo ranks (CPU).

Each rank computes its row shard with the CPU oracle (standing in for the
rank's GPU), the blocks are all-gathered and assembled, and the result must
equal the unsharded product (the rows are computed identically)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from flatrun_b200 import shard, synth


def test_row_range_covers_rows():
    for n, w in [(3584, 8), (512, 3), (7, 4), (152064, 8)]:
        ranges = [shard.row_range(n, w, r) for r in range(w)]
        assert ranges[0][0] == 0 and ranges[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        sizes = [e - s for s, e in ranges]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.row_range(10, 2, 2)


def test_shard_bytes_are_whole_rows():
    n, k = 12, 512
    raw = synth.make_weight("Q6_K", n, k, seed=3)
    parts = [shard.shard_bytes(raw, "Q6_K", n, k, 4, r) for r in range(4)]
    assert b"".join(p.tobytes() for p in parts) == raw.tobytes()
    assert all(p.size == 3 * synth.row_bytes("Q6_K", k) for p in parts)


def test_assemble_layout_numpy():
    world, batch, nl = 3, 2, 4
    blocks = [np.arange(batch * nl).reshape(batch, nl) + 100 * r for r in range(world)]
    full = shard.assemble(np.concatenate([b.reshape(-1) for b in blocks]), world, batch, nl)
    np.testing.assert_array_equal(full, np.concatenate(blocks, axis=1))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, fmt, n, k, batch, q):
    import torch.distributed as dist
    from oracle import gguf_oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        raw = synth.make_weight(fmt, n, k, seed=9)
        x = synth.make_x(k, batch=batch, seed=10)
        local = shard.shard_bytes(raw, fmt, n, k, world, rank)
        s, e = shard.row_range(n, world, rank)
        y = shard.sharded_matmul(lambda xx: O.matvec_fp32(fmt, local, xx, e - s, k), x, n, world)
        q.put((rank, np.asarray(y)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fmt,n,k,batch", [("Q4_K", 64, 512, 3), ("Q8_0", 32, 64, 1)])
def test_sharded_matmul_two_gloo_ranks(fmt, n, k, batch):
    import multiprocessing as mp
    from oracle import gguf_oracle as O
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, fmt, n, k, batch, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    raw = synth.make_weight(fmt, n, k, seed=9)
    x = synth.make_x(k, batch=batch, seed=10)
    full = O.matvec_fp32(fmt, raw, x, n, k).reshape(batch, n)
    for r in range(2):
        np.testing.assert_allclose(results[r], full, rtol=0, atol=1e-5 * np.abs(full).max())
