"""The fused all-gather's bounded waits on one GPU (no fault, no hang): a
"world" of two ranks whose second rank never publishes, so every wait on its
flag runs out after the 1 s limit.  The wait kernel and the GEMV that waits
before reading x must return, record the timeout in the device status word,
and the GEMV must then keep its outputs local (a peer may still be reading
its buffer) instead of storing into the other rank's buffer."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from flatrun_b200 import _lib, synth
from oracle import gguf_oracle as O

pytestmark = pytest.mark.gpu

GATHER_TIMEOUT = 1 << 4  # kStatusGatherTimeout


def test_gather_waits_run_out_and_are_reported(cuda_backend):
    import torch
    lib = _lib.load()
    stream = torch.cuda.current_stream()
    st = ctypes.c_void_p(stream.cuda_stream)
    fmt, n, k = "Q4_K", 256, 512
    raw = synth.make_weight(fmt, n, k, seed=91)
    x = synth.make_x(k, seed=92)
    w = torch.from_numpy(raw).cuda()
    xd = torch.from_numpy(x).cuda()
    # rank 0 and an absent rank 1: each owns a gathered buffer of 2 shards
    # and a flag array of 2 words, all on this GPU
    bufs = [torch.full((2 * n,), -7.0, device="cuda") for _ in range(2)]
    flags = [torch.zeros(2, dtype=torch.int32, device="cuda") for _ in range(2)]
    y = bufs[0][:n]  # rank 0's own shard of its gathered buffer
    g = ctypes.c_void_p()
    _lib.check(lib.frc_gather_create(2, 0, (ctypes.c_void_p * 2)(bufs[0].data_ptr(), bufs[1].data_ptr()),
                                     (ctypes.c_void_p * 2)(flags[0].data_ptr(), flags[1].data_ptr()),
                                     ctypes.byref(g)), lib)
    clear = ctypes.c_uint32()
    _lib.check(lib.frc_device_status(0, ctypes.byref(clear)), lib)

    def gemv(wait_for):
        return lib.frc_gemv_gather(_lib.QUANT_IDS[fmt], 1, (ctypes.c_void_p * 1)(w.data_ptr()),
                                   (ctypes.c_size_t * 1)(raw.nbytes), (ctypes.c_int64 * 1)(n), k, xd.data_ptr(),
                                   (ctypes.c_void_p * 1)(y.data_ptr()), y.data_ptr(), g, wait_for, st)

    ref = O.matvec_fp64(fmt, raw, x, n, k)
    # 1: no wait; stores into both buffers and publishes epoch 1 to both flag arrays
    _lib.check(gemv(None), lib)
    torch.cuda.synchronize()
    assert O.rel_err(bufs[0][:n].cpu().numpy(), ref) < 2e-5
    assert np.array_equal(bufs[1][:n].cpu().numpy(), bufs[0][:n].cpu().numpy())
    assert flags[0].cpu().tolist() == [1, 0] and flags[1].cpu().tolist() == [1, 0]
    # 2: the wait kernel for the gather: rank 1 never publishes -> runs out
    _lib.check(lib.frc_gather_wait(g, st), lib)
    status = ctypes.c_uint32()
    _lib.check(lib.frc_device_status(0, ctypes.byref(status)), lib)
    assert status.value & GATHER_TIMEOUT
    # 3: a GEMV that waits for the gather before reading x: the wait runs out,
    # the outputs stay local, nothing is published, the timeout is reported
    bufs[1].fill_(-7.0)
    y.fill_(0.0)
    _lib.check(gemv(g), lib)
    _lib.check(lib.frc_device_status(0, ctypes.byref(status)), lib)
    assert status.value & GATHER_TIMEOUT
    assert O.rel_err(y.cpu().numpy(), ref) < 2e-5
    assert np.all(bufs[1].cpu().numpy() == -7.0)
    assert flags[0].cpu().tolist() == [1, 0] and flags[1].cpu().tolist() == [1, 0]
    _lib.check(lib.frc_device_status(0, ctypes.byref(status)), lib)
    assert status.value == 0
    lib.frc_gather_free(g)
