"""All-gather fused into the batch-1 GEMV, on two GPUs (one process each).

Each rank owns half the rows of two projection groups: a q/k/v-like launch
(three Q4_K matrices sharing x) and a single Q6_K matrix.  Three rounds chain
the groups as a forward pass would (each GEMV waits for the previous group's
gather before reading x; the last gather of a round is waited for with
frc_gather_wait); after every round both gathered buffers on every rank must
hold every rank's shard, bit for bit equal to the same rows computed by
frc_gemv_multi without the gather.  Handles are exchanged over a gloo process
group.  Skipped with fewer than two GPUs."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GROUPS = [("Q4_K", [512, 128, 128], 1024), ("Q6_K", [300], 3584)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    import ctypes

    import torch
    import torch.distributed as dist

    from flatrun_b200 import _lib, shard, synth

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    results = []
    gathers = []
    try:
        groups = []
        for gi, (fmt, ns_full, k) in enumerate(GROUPS):
            raws = [synth.make_weight(fmt, n, k, seed=70 + 10 * gi + i) for i, n in enumerate(ns_full)]
            shards = [[torch.from_numpy(np.ascontiguousarray(shard.shard_bytes(raw, fmt, n, k, world, r))).cuda()
                       for raw, n in zip(raws, ns_full)] for r in range(world)]
            n_loc = [[shard.row_range(n, world, r)[1] - shard.row_range(n, world, r)[0] for n in ns_full]
                     for r in range(world)]
            floats = sum(n_loc[rank])
            assert all(sum(n_loc[r]) == floats for r in range(world))
            g = shard.FusedGather(lib, world, rank, floats)
            gathers.append(g)
            local = torch.empty(floats, device="cuda")
            ys, off = [], 0
            for nl in n_loc[rank]:
                ys.append(local[off:off + nl])
                off += nl
            groups.append(dict(fmt=fmt, k=k, qid=_lib.QUANT_IDS[fmt], shards=shards, n_loc=n_loc, g=g,
                               local=local, ys=ys))
        for it in range(3):
            xs = [torch.from_numpy(synth.make_x(gr["k"], seed=100 + 10 * it + gi)).cuda()
                  for gi, gr in enumerate(groups)]
            for gi, gr in enumerate(groups):
                prev = groups[gi - 1]["g"] if (it > 0 or gi > 0) else None
                rc = gr["g"].gemv(gr["qid"], [t.data_ptr() for t in gr["shards"][rank]],
                                  [t.numel() for t in gr["shards"][rank]], gr["n_loc"][rank], gr["k"],
                                  xs[gi].data_ptr(), [t.data_ptr() for t in gr["ys"]], gr["local"].data_ptr(),
                                  stream, wait_for=prev)
                _lib.check(rc, lib)
            groups[-1]["g"].wait(stream)
            torch.cuda.synchronize()
            for gi, gr in enumerate(groups):
                got = gr["g"].gathered().cpu().numpy().copy()
                expect = []
                c = len(gr["n_loc"][rank])
                for r in range(world):
                    yr = [torch.empty(nl, device="cuda") for nl in gr["n_loc"][r]]
                    _lib.check(lib.frc_gemv_multi(
                        gr["qid"], c, (ctypes.c_void_p * c)(*[t.data_ptr() for t in gr["shards"][r]]),
                        (ctypes.c_size_t * c)(*[t.numel() for t in gr["shards"][r]]),
                        (ctypes.c_int64 * c)(*gr["n_loc"][r]), gr["k"], xs[gi].data_ptr(), 1,
                        (ctypes.c_void_p * c)(*[t.data_ptr() for t in yr]), ctypes.c_void_p(stream)), lib)
                    expect.extend(yr)
                torch.cuda.synchronize()
                results.append((it, gr["fmt"], bool(np.array_equal(got, torch.cat(expect).cpu().numpy()))))
        flags = ctypes.c_uint32()
        _lib.check(lib.frc_device_status(rank, ctypes.byref(flags)), lib)
        torch.cuda.synchronize()
        dist.barrier()
        for g in gathers:
            g.close()
        q.put((rank, results, int(flags.value)))
    finally:
        dist.destroy_process_group()


def test_fused_gather_two_gpus():
    import multiprocessing as mp

    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in procs:
        rank, results, flags = q.get(timeout=300)
        out[rank] = (results, flags)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        results, flags = out[r]
        assert len(results) == 3 * len(GROUPS)
        assert all(ok for _, _, ok in results), (r, results)
        assert flags == 0, (r, hex(flags))
