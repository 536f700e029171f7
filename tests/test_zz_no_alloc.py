"""frc_gemv_noalloc: the batched GEMV for callers that may not allocate
device memory while they run, over a fixed static activation-record region
(GPU).  Compared with frc_gemv, which stages the same records in a buffer it
allocates, on two calls in a row; checked to leave the device's free memory
unchanged; its status word read back clear; plus its argument limits.  Kept
in its own file, collected last, so a run that stops at the first failure has
run every other test first; it passes both after the rest of the suite and
on its own (`pytest tests/test_zz_no_alloc.py -m gpu`)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from flatrun_b200 import _lib, synth
from oracle import gguf_oracle as O

pytestmark = pytest.mark.gpu

TOL_I8 = 1e-4  # the integer-grid tolerance of the batched kernels against fp64


def _call(lib, name, fmt, w, nbytes, n, k, x, batch, y, stream):
    return getattr(lib, name)(_lib.QUANT_IDS[fmt], w.data_ptr(), nbytes, n, k, x.data_ptr(), batch, y.data_ptr(),
                              ctypes.c_void_p(stream.cuda_stream))


@pytest.mark.parametrize("fmt,n,k,batch", [("Q4_K", 300, 3584, 4), ("Q6_K", 517, 3584, 16), ("Q5_K", 96, 18944, 9),
                                           ("Q8_0", 333, 4096, 2), ("Q1_0", 64, 4096, 7), ("Q6_K", 7, 768, 3)])
def test_noalloc_matches_frc_gemv_twice(fmt, n, k, batch):
    import torch
    lib = _lib.load()
    raw = synth.make_weight(fmt, n, k, seed=500 + n)
    x = synth.make_x(k, batch=batch, seed=600 + n)
    w_d = torch.from_numpy(raw).cuda()
    x_d = torch.from_numpy(x).cuda()
    stream = torch.cuda.current_stream()
    y_ref = torch.full((batch, n), float("nan"), device="cuda")
    _lib.check(_call(lib, "frc_gemv", fmt, w_d, raw.nbytes, n, k, x_d, batch, y_ref, stream), lib)
    ys = []
    for _ in range(2):
        y = torch.full((batch, n), float("nan"), device="cuda")
        _lib.check(_call(lib, "frc_gemv_noalloc", fmt, w_d, raw.nbytes, n, k, x_d, batch, y, stream), lib)
        ys.append(y)
    torch.cuda.synchronize()
    ref = y_ref.cpu().numpy()
    ref64 = O.matvec_fp64(fmt, raw, x, n, k)
    scale = O.term_scale(fmt, raw, x, n, k)
    for y in ys:
        got = y.cpu().numpy()
        assert np.isfinite(got).all()
        np.testing.assert_allclose(got, ref, rtol=0, atol=TOL_I8 * np.abs(ref).max())
        assert O.norm_err(got, ref64, scale) < 5e-5
    _assert_status_clear(lib)


def _assert_status_clear(lib):
    flags = ctypes.c_uint32(0xFFFFFFFF)
    _lib.check(lib.frc_noalloc_status(0, ctypes.byref(flags)), lib)
    assert flags.value == 0


def test_noalloc_allocates_nothing():
    """The property the entry point exists for: once the first call on the
    device has looked up the static region (and the kernels are loaded),
    further calls at several formats, k and batch sizes leave the device's
    free memory exactly as it was.  Every buffer is allocated before the
    measurement and no frc_gemv call runs in this test."""
    import torch
    lib = _lib.load()
    stream = torch.cuda.current_stream()
    cases = []
    for fmt, n, k, batch in [("Q4_K", 300, 3584, 4), ("Q6_K", 64, 3584, 16), ("Q8_0", 96, 4096, 9),
                             ("Q5_K", 40, 18944, 2)]:
        raw = synth.make_weight(fmt, n, k, seed=700 + n)
        x = synth.make_x(k, batch=batch, seed=800 + n)
        cases.append((fmt, n, k, batch, raw, torch.from_numpy(raw).cuda(), torch.from_numpy(x).cuda(),
                      torch.empty((batch, n), device="cuda")))

    def run_all():
        for fmt, n, k, batch, raw, w_d, x_d, y_d in cases:
            _lib.check(_call(lib, "frc_gemv_noalloc", fmt, w_d, raw.nbytes, n, k, x_d, batch, y_d, stream), lib)

    run_all()  # first calls: symbol lookup and module loading
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        run_all()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    _assert_status_clear(lib)


def test_noalloc_limits_are_errors():
    import torch
    lib = _lib.load()
    stream = torch.cuda.current_stream()
    fmt = "Q4_K"
    # batch 16 allows k <= 41472; one 512-chunk more is refused with a message
    n, k = 8, 41472 + 512
    w_d = torch.zeros(synth.weight_bytes(fmt, n, k), dtype=torch.uint8, device="cuda")
    x_d = torch.zeros((16, k), device="cuda")
    y_d = torch.zeros((16, n), device="cuda")
    rc = _call(lib, "frc_gemv_noalloc", fmt, w_d, w_d.numel(), n, k, x_d, 16, y_d, stream)
    assert rc == _lib.FRC_ERR_INVALID
    assert "41472" in _lib.last_error(lib)
    nb = synth.weight_bytes(fmt, n, 512)
    for batch in (1, 17):
        rc = _call(lib, "frc_gemv_noalloc", fmt, w_d, nb, n, 512, x_d, batch, y_d, stream)
        assert rc == _lib.FRC_ERR_INVALID
        assert "batch must be 2..16" in _lib.last_error(lib)
    torch.cuda.synchronize()
