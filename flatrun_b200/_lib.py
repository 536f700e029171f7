"""ctypes binding of libfrcuda.so (the C ABI in include/frcuda.h).

The library is built in-tree by ``python -m flatrun_b200.build``.  Loading
fails loudly when it is missing: there is no CPU fallback behind this module.
"""

from __future__ import annotations

import ctypes
import os
import threading

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libfrcuda.so")

FRC_OK = 0
FRC_ERR_INVALID = 1
FRC_ERR_CUDA = 2
FRC_ERR_NOMEM = 3
FRC_ERR_DEVICE = 4
FRC_ERR_UNSUPPORTED = 5

QUANT_IDS = {"Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "Q1_0": 41}
QUANT_NAMES = {v: k for k, v in QUANT_IDS.items()}

FRC_GEMV_ACCUMULATE = 1  # frc_gemv_ex flag

# frc_set_option ids (include/frcuda.h FRC_OPT_*)
OPTIONS = {"batch1_int16": 1, "batched_fp32": 2, "prefill_tc": 3, "prefill_splits": 4, "inject_oom": 5,
           "batch1_tc": 6}

_i = ctypes.c_int
_i64 = ctypes.c_int64
_sz = ctypes.c_size_t
_p = ctypes.c_void_p
_fp = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_cp = ctypes.c_char_p

# name -> argtypes (every function returns int)
SIGNATURES: dict[str, list] = {
    "frc_version": [_cp, _sz],
    "frc_is_neon": [],
    "frc_last_error": [_cp, _sz],
    "frc_device_count": [ctypes.POINTER(_i)],
    "frc_block_geometry": [_i, ctypes.POINTER(_i), ctypes.POINTER(_i)],
    "frc_weight_nbytes": [_i, _i64, _i64, ctypes.POINTER(_sz)],
    "frc_device_status": [_i, ctypes.POINTER(ctypes.c_uint32)],
    "frc_set_option": [_i, _i],
    "frc_get_option": [_i, ctypes.POINTER(_i)],
    "frc_batch1_kernel": [_i, ctypes.c_int64, ctypes.POINTER(_i)],
    "frc_batch1_plan": [_i, _i64, _i64, _i, ctypes.POINTER(_i64)],
    "frc_noalloc_status": [_i, ctypes.POINTER(ctypes.c_uint32)],
    "frc_gemv_ex": [_i, _i, ctypes.POINTER(_p), ctypes.POINTER(_sz), ctypes.POINTER(_i64), _i64, _p, _p, _p,
                    ctypes.c_float, _i, ctypes.POINTER(_p), _p],
    "frc_rmsnorm": [_p, _p, _i64, _i64, ctypes.c_float, _p, _p],
    "frc_rope_append": [_p, _p, _i, _i, _i, _p, _p, _p, _p, _p, _p],
    "frc_attention_workspace": [_i, _i, _i, ctypes.POINTER(_sz)],
    "frc_attention_decode": [_p, _p, _p, _p, _i, _i, _i, ctypes.c_float, _i, _p, _p, _p],
    "frc_argmax_workspace": [_i64, ctypes.POINTER(_sz)],
    "frc_argmax": [_p, _i64, _p, _p, _p],
    "frc_embed_row": [_i, _p, _i64, _p, _p, _p],
    "frc_pos_advance": [_p, _p],
    "frc_gemv": [_i, _p, _sz, _i64, _i64, _p, _i64, _p, _p],
    "frc_gemv_noalloc": [_i, _p, _sz, _i64, _i64, _p, _i64, _p, _p],
    "frc_ipc_alloc": [_sz, ctypes.POINTER(_p), _p],
    "frc_ipc_open": [_p, ctypes.POINTER(_p)],
    "frc_ipc_close": [_p],
    "frc_ipc_free": [_p],
    "frc_gather_create": [_i, _i, ctypes.POINTER(_p), ctypes.POINTER(_p), ctypes.POINTER(_p)],
    "frc_gather_free": [_p],
    "frc_gemv_gather": [_i, _i, ctypes.POINTER(_p), ctypes.POINTER(_sz), ctypes.POINTER(_i64), _i64, _p,
                        ctypes.POINTER(_p), _p, _p, _p, _p],
    "frc_gather_wait": [_p, _p],
    "frc_dequant_dev": [_i, _p, _sz, _i64, _p, _p],
    "frc_gemv_multi": [_i, _i, ctypes.POINTER(_p), ctypes.POINTER(_sz), ctypes.POINTER(_i64), _i64, _p, _i64,
                       ctypes.POINTER(_p), _p],
    "frc_weight_create": [_i, _i, _p, _sz, _i64, _i64, ctypes.POINTER(_p)],
    "frc_weight_free": [_p],
    "frc_weight_info": [_p, ctypes.POINTER(_p), ctypes.POINTER(_sz), ctypes.POINTER(_i),
                        ctypes.POINTER(_i64), ctypes.POINTER(_i64), ctypes.POINTER(_i)],
    "frc_weight_matmul": [_p, _p, _i64, _p],
    "frc_weight_matmul_dev": [_p, _p, _i64, _p, _p],
    "frc_weight_dequant": [_p, _p],
}
for _q in ("q4_k", "q8_0", "q6_k", "q5_k", "q1_0"):
    SIGNATURES[f"frc_matmul_{_q}"] = [_p, _p, _sz, _i64, _i64, _p]
    SIGNATURES[f"frc_matmul_{_q}_batched"] = [_p, _i64, _p, _sz, _i64, _i64, _p]
    SIGNATURES[f"frc_dequant_{_q}"] = [_p, _sz, _i64, _i64, _p]


class FrcError(RuntimeError):
    """A C-ABI call returned a nonzero status (the reference raises
    RuntimeError from its pybind11 kernels in the same situations)."""

    def __init__(self, code: int, message: str):
        super().__init__(f"[frcuda status {code}] {message}")
        self.code = code


class LibraryMissing(ImportError):
    pass


_lib = None
_lock = threading.Lock()


def load(path: str | None = None) -> ctypes.CDLL:
    """Load (once) and return the library with typed signatures."""
    global _lib
    with _lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise LibraryMissing(
                f"{p} not found: build it with `python -m flatrun_b200.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(p)
        for name, argtypes in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
        if path is None:
            _lib = lib
        return lib


def last_error(lib: ctypes.CDLL | None = None) -> str:
    lib = lib or load()
    buf = ctypes.create_string_buffer(1024)
    lib.frc_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int, lib: ctypes.CDLL | None = None) -> None:
    if rc != FRC_OK:
        raise FrcError(rc, last_error(lib))


def version() -> str:
    lib = load()
    buf = ctypes.create_string_buffer(256)
    check(lib.frc_version(buf, len(buf)), lib)
    return buf.value.decode()


def device_count() -> int:
    lib = load()
    n = ctypes.c_int(0)
    rc = lib.frc_device_count(ctypes.byref(n))
    if rc != FRC_OK:
        return 0
    return int(n.value)


def set_option(name: str, value: int) -> int:
    """Set a library option (frc_set_option); returns the previous value."""
    lib = load()
    old = ctypes.c_int(0)
    check(lib.frc_get_option(OPTIONS[name], ctypes.byref(old)), lib)
    check(lib.frc_set_option(OPTIONS[name], int(value)), lib)
    return int(old.value)


def get_option(name: str) -> int:
    lib = load()
    v = ctypes.c_int(0)
    check(lib.frc_get_option(OPTIONS[name], ctypes.byref(v)), lib)
    return int(v.value)


BATCH1_KERNELS = {0: "cuda_core_fp32", 1: "tensor_fp32", 2: "int16"}


def batch1_kernel(quant: str, k: int) -> str:
    """Which batch-1 kernel a launch of (quant, k) runs under the current
    options: "tensor_fp32" (gemv_tc1), "cuda_core_fp32" or "int16"."""
    lib = load()
    v = ctypes.c_int(-1)
    check(lib.frc_batch1_kernel(QUANT_IDS[quant], int(k), ctypes.byref(v)), lib)
    return BATCH1_KERNELS[int(v.value)]


PLAN_FIELDS = ("kernel", "warps", "chunks", "part_chunks", "split", "ranges", "ctas", "builders", "stages",
               "rows_max", "smem", "tiles_per_warp")


def batch1_plan(quant: str, n: int, k: int, sms: int = 148) -> dict:
    """The batch-1 launch plan of an (n, k) matrix on a device of `sms` SMs
    (frc_batch1_plan; host-side, no GPU needed)."""
    lib = load()
    arr = (ctypes.c_int64 * len(PLAN_FIELDS))()
    check(lib.frc_batch1_plan(QUANT_IDS[quant], int(n), int(k), int(sms), arr), lib)
    plan = dict(zip(PLAN_FIELDS, (int(v) for v in arr)))
    plan["kernel"] = BATCH1_KERNELS[plan["kernel"]]
    return plan


class option:
    """Context manager: `with option("batch1_int16", 1): ...` sets a library
    option for the block and restores the previous value after it."""

    def __init__(self, name: str, value: int):
        self.name, self.value, self.old = name, value, None

    def __enter__(self):
        self.old = set_option(self.name, self.value)
        return self

    def __exit__(self, *exc):
        set_option(self.name, self.old)
        return False
