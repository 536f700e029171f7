"""The C-ABI library: loads, exports every symbol include/frcuda.h declares,
and rejects bad arguments before any CUDA call (CPU only, no GPU needed)."""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

from flatrun_b200 import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "frcuda.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\bint\s+(frc_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(_lib.LIB_PATH):
        from flatrun_b200 import build
        build.build()
    return _lib.load()


def test_header_declares_reference_mirrors():
    names = set(_declared())
    for q in ("q4_k", "q8_0", "q6_k"):  # flatrun_native._C (_C.cpp:455-488)
        assert {f"frc_matmul_{q}", f"frc_matmul_{q}_batched", f"frc_dequant_{q}"} <= names
    assert {"frc_version", "frc_is_neon", "frc_gemv", "frc_weight_matmul"} <= names


def test_every_declared_symbol_is_exported(lib):
    names = _declared()
    assert len(names) >= 30
    for name in names:
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_geometry_without_gpu(lib):
    assert "sm_100a" in _lib.version()
    assert lib.frc_is_neon() == 0
    qk, ts = ctypes.c_int(), ctypes.c_int()
    for name, qid in _lib.QUANT_IDS.items():
        assert lib.frc_block_geometry(qid, ctypes.byref(qk), ctypes.byref(ts)) == 0
        from flatrun_b200.synth import FORMATS
        assert (qk.value, ts.value) == FORMATS[name]
    assert lib.frc_block_geometry(99, ctypes.byref(qk), ctypes.byref(ts)) == _lib.FRC_ERR_INVALID
    nb = ctypes.c_size_t()
    assert lib.frc_weight_nbytes(12, 18944, 3584, ctypes.byref(nb)) == 0
    assert nb.value == 38_191_104
    assert lib.frc_weight_nbytes(12, 4, 100, ctypes.byref(nb)) == _lib.FRC_ERR_INVALID


@pytest.mark.parametrize("fn,args,msg", [
    ("frc_matmul_q4_k", (None, None, 144, 1, 255, None), "multiple of 256"),
    ("frc_matmul_q4_k", (None, None, 143, 1, 256, None), "byte size mismatch"),
    ("frc_matmul_q8_0", (None, None, 34, 1, 33, None), "multiple of 32"),
    ("frc_matmul_q6_k", (None, None, 209, 1, 256, None), "byte size mismatch"),
    ("frc_dequant_q4_k", (None, 144, 1, 255, None), "multiple of 256"),
    ("frc_dequant_q8_0", (None, 33, 1, 32, None), "byte size mismatch"),
])
def test_reference_error_paths_before_cuda(lib, fn, args, msg):
    rc = getattr(lib, fn)(*args)
    assert rc == _lib.FRC_ERR_INVALID
    assert msg in _lib.last_error(lib)


def test_gemv_rejects_misaligned_and_empty_batch(lib):
    assert lib.frc_gemv(12, 1, 144, 1, 256, 16, 1, 16, None) == _lib.FRC_ERR_INVALID
    assert "aligned" in _lib.last_error(lib)
    assert lib.frc_gemv(12, 16, 144, 1, 256, 16, 0, 16, None) == _lib.FRC_ERR_INVALID
    assert lib.frc_gemv(7, 16, 144, 1, 256, 16, 1, 16, None) == _lib.FRC_ERR_INVALID


def test_gemv_multi_argument_checks(lib):
    two = (ctypes.c_void_p * 2)(16, 32)
    sizes = (ctypes.c_size_t * 2)(144, 144)
    ns = (ctypes.c_int64 * 2)(1, 1)
    ys = (ctypes.c_void_p * 2)(16, 32)
    assert lib.frc_gemv_multi(12, 5, two, sizes, ns, 256, 16, 1, ys, None) == _lib.FRC_ERR_INVALID
    assert "count" in _lib.last_error(lib)
    bad = (ctypes.c_size_t * 2)(144, 143)
    assert lib.frc_gemv_multi(12, 2, two, bad, ns, 256, 16, 1, ys, None) == _lib.FRC_ERR_INVALID
    assert "mismatch" in _lib.last_error(lib)


def test_q1_0_dequant_accepts_numpy_tail_rule(lib):
    """Q1_0 follows the NumPy rule (ceil blocks, tail dropped, gguf.py:266-299):
    130 elements need 2 blocks; a 1-block buffer is a size mismatch."""
    rc = lib.frc_dequant_q1_0(None, 18, 130, 1, None)
    assert rc == _lib.FRC_ERR_INVALID and "mismatch" in _lib.last_error(lib)


def test_backend_unavailable_raises_without_fallback():
    from flatrun_b200 import CudaBackend
    be = CudaBackend(device=0, lib_path=os.path.join(REPO, "does-not-exist.so"))
    assert not be.available and be.supported_quants == set()
    with pytest.raises(RuntimeError):
        be.matmul_q4k(np.zeros(256, np.float32), np.zeros(144, np.uint8), 1, 256)
