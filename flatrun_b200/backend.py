"""``CudaBackend``: the B200 projection backend in the reference's backend slot.

Mirrors the interface of ``BackendBase`` (src/flatrun/runtime/backend.py:59-156)
and the facade ``flatrun_native.NativeBackend``
(src/flatrun_native/python/__init__.py:85-227):

* properties ``name``, ``available``, ``supported_quants``;
* ``matmul_q4k``, ``matmul_q6k``, ``matmul_q8_0`` (and the formats the
  reference decodes only in NumPy, ``matmul_q5k``, ``matmul_q1_0``) taking
  ``(x, weight, n, k)``: x fp32 (k,) -> (n,), or (seq, k) -> (seq, n);
  ``weight`` a 1-D uint8 view of the raw GGUF blocks or a handle with
  ``.as_numpy()`` (backend.py:251-257);
* ``dispatch(x, weight, n, k, quant)`` (backend.py:131-156);
* ``dequant_q4k(weight, shape)`` and friends (python/__init__.py:211-227).

Errors: a bad x rank or length raises ``ValueError`` as the facade does
(python/__init__.py:147-153); a shape or byte-size mismatch raises
``RuntimeError`` (``FrcError``) as the pybind11 kernels do (_C.cpp:105-120).
Unlike ``NativeBackend._try_kernel`` (backend.py:259-268) nothing falls back to
NumPy: a failed kernel is an error.

Weights are uploaded to HBM once, keyed by the address and size of the host
bytes (the GGUF mmap view, stable while the model is open), and the source
array is referenced by the cache entry so the address cannot be reused while
the copy lives.  Each call then moves only x in and y out.
"""

from __future__ import annotations

import ctypes
import threading
from typing import Any

import numpy as np

from . import _lib
from .synth import FORMATS

_METHOD_QUANT = {
    "matmul_q4k": "Q4_K",
    "matmul_q6k": "Q6_K",
    "matmul_q8_0": "Q8_0",
    "matmul_q5k": "Q5_K",
    "matmul_q1_0": "Q1_0",
}
QUANT_DISPATCH = {q: m for m, q in _METHOD_QUANT.items()}


def _raw_bytes(weight: Any) -> np.ndarray:
    raw = weight.as_numpy() if hasattr(weight, "as_numpy") else weight
    if isinstance(raw, (bytes, bytearray, memoryview)):
        raw = np.frombuffer(raw, dtype=np.uint8)
    raw = np.asarray(raw)
    if raw.dtype != np.uint8:
        raw = raw.view(np.uint8) if raw.flags.c_contiguous else np.ascontiguousarray(raw).view(np.uint8)
    if not raw.flags.c_contiguous:
        raw = np.ascontiguousarray(raw)
    return raw.reshape(-1)


class DeviceWeight:
    """Raw GGUF blocks of one (n, k) weight resident in HBM."""

    def __init__(self, lib, device: int, quant: str, raw: np.ndarray, n: int, k: int):
        self._lib = lib
        self.quant, self.n, self.k, self.device = quant, int(n), int(k), int(device)
        self.nbytes = int(raw.nbytes)
        h = ctypes.c_void_p()
        _lib.check(lib.frc_weight_create(device, _lib.QUANT_IDS[quant], raw.ctypes.data, raw.nbytes,
                                         self.n, self.k, ctypes.byref(h)), lib)
        self.handle = h

    def matmul(self, x: np.ndarray) -> np.ndarray:
        seq = 1 if x.ndim == 1 else x.shape[0]
        y = np.empty((self.n,) if x.ndim == 1 else (seq, self.n), dtype=np.float32)
        _lib.check(self._lib.frc_weight_matmul(self.handle, x.ctypes.data, seq, y.ctypes.data), self._lib)
        return y

    def dequant(self) -> np.ndarray:
        out = np.empty((self.n, self.k), dtype=np.float32)
        _lib.check(self._lib.frc_weight_dequant(self.handle, out.ctypes.data), self._lib)
        return out

    def device_ptr(self) -> int:
        p = ctypes.c_void_p()
        _lib.check(self._lib.frc_weight_info(self.handle, ctypes.byref(p), None, None, None, None, None),
                   self._lib)
        return int(p.value or 0)

    def free(self) -> None:
        if self.handle is not None and self.handle.value:
            self._lib.frc_weight_free(self.handle)
        self.handle = None

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.free()
        except Exception:
            pass


class ShardedWeight:
    """One (n, k) weight whose rows are split over several GPUs in one process.

    Rows are independent and every row is a whole number of quant blocks, so
    device i holds the contiguous rows ``shard.row_range(n, len(devices), i)``
    (the same split as the one-process-per-GPU path).  A call runs every
    shard at once (one host thread per device; the C ABI releases the GIL)
    and writes each shard's outputs straight into its columns of y: the
    assembly is the host copy the reference's API needs anyway.
    """

    def __init__(self, lib, devices: list, quant: str, raw: np.ndarray, n: int, k: int):
        from concurrent.futures import ThreadPoolExecutor

        from .shard import row_range
        from .synth import row_bytes

        self.quant, self.n, self.k, self.nbytes = quant, int(n), int(k), int(raw.nbytes)
        rb = row_bytes(quant, k)
        self.parts = []
        for i, dev in enumerate(devices):
            r0, r1 = row_range(self.n, len(devices), i)
            if r1 > r0:
                self.parts.append((DeviceWeight(lib, dev, quant, raw[r0 * rb:r1 * rb], r1 - r0, k), r0, r1))
        self._pool = ThreadPoolExecutor(max_workers=max(1, len(self.parts)))

    def matmul(self, x: np.ndarray) -> np.ndarray:
        y = np.empty((self.n,) if x.ndim == 1 else (x.shape[0], self.n), dtype=np.float32)

        def run(part):
            dw, r0, r1 = part
            y[..., r0:r1] = dw.matmul(x)

        for f in [self._pool.submit(run, p) for p in self.parts]:
            f.result()
        return y

    def dequant(self) -> np.ndarray:
        return np.concatenate([dw.dequant() for dw, _, _ in self.parts], axis=0)

    def free(self) -> None:
        for dw, _, _ in self.parts:
            dw.free()
        self._pool.shutdown(wait=False)

    @property
    def handle(self):
        return self.parts[0][0].handle if self.parts else None


def devices_from_env(default: int = 0) -> list:
    """GPUs named by FLATRUN_CUDA_DEVICES (comma-separated ids), else [default]."""
    import os
    spec = os.environ.get("FLATRUN_CUDA_DEVICES", "").strip()
    return [int(d) for d in spec.split(",") if d.strip()] if spec else [default]


class CudaBackend:
    """B200 fused dequant + matvec backend (``--backend cuda``).

    `devices`: GPUs to row-shard every projection over (one process); by
    default the single `device`."""

    def __init__(self, device: int = 0, lib_path: str | None = None, devices: list | None = None):
        self.device = int(device)
        self.devices = [int(d) for d in devices] if devices else [self.device]
        self._load_error: BaseException | None = None
        try:
            self._lib = _lib.load(lib_path)
            self._ndev = _lib.device_count()
        except (OSError, ImportError) as exc:
            self._lib = None
            self._ndev = 0
            self._load_error = exc
        if self.devices != [self.device]:
            self.device = max(self.devices)  # availability checks the highest id
        self._cache: dict[tuple, tuple[DeviceWeight, np.ndarray]] = {}
        self._by_id: dict[int, tuple] = {}
        self._mu = threading.Lock()

    # --- BackendBase properties (backend.py:62-81) ---------------------------
    @property
    def name(self) -> str:
        return "cuda"

    @property
    def available(self) -> bool:
        return self._lib is not None and self.device < self._ndev

    @property
    def supported_quants(self) -> set[str]:
        return set(_METHOD_QUANT.values()) if self.available else set()

    # --- plumbing -----------------------------------------------------------
    def _require(self):
        if self._lib is None:
            raise RuntimeError(f"flatrun_b200 CUDA library is not available: {self._load_error}")
        if self.device >= self._ndev:
            raise RuntimeError(f"CUDA device {self.device} not available ({self._ndev} visible)")
        return self._lib

    def weight(self, weight: Any, n: int, k: int, quant: str) -> DeviceWeight:
        """Device copy of `weight`, uploaded on first use."""
        # fast path: the same array object as a cached entry (the entry holds
        # a reference to it, so its id cannot be reused while cached)
        hit = self._by_id.get(id(weight))
        if hit is not None and hit[1] is weight and hit[0].handle is not None and hit[2] == (quant, n, k):
            return hit[0]
        lib = self._require()
        raw = _raw_bytes(weight)
        key = (raw.ctypes.data, raw.nbytes, quant, int(n), int(k))
        with self._mu:
            entry = self._cache.get(key)
            if entry is None:
                dw = DeviceWeight(lib, self.devices[0], quant, raw, n, k) if len(self.devices) == 1 else \
                    ShardedWeight(lib, self.devices, quant, raw, n, k)
                entry = (dw, raw)
                self._cache[key] = entry
            self._by_id[id(weight)] = (entry[0], weight, (quant, n, k))
            return entry[0]

    def close(self) -> None:
        with self._mu:
            for dw, _ in self._cache.values():
                dw.free()
            self._cache.clear()
            self._by_id.clear()

    @property
    def resident_bytes(self) -> int:
        return sum(dw.nbytes for dw, _ in self._cache.values())

    def _matmul(self, quant: str, x, weight, n: int, k: int) -> np.ndarray:
        if self._lib is None or self.device >= self._ndev:
            self._require()
        x_c = x if (type(x) is np.ndarray and x.dtype == np.float32 and x.flags.c_contiguous) \
            else np.ascontiguousarray(x, dtype=np.float32)
        if x_c.ndim == 1:
            if x_c.shape[0] != k:
                raise ValueError(f"x.shape[0]={x_c.shape[0]} != k={k}")
        elif x_c.ndim == 2:
            if x_c.shape[1] != k:
                raise RuntimeError(f"{quant} matmul (batched): x.shape[1] != k")
            if x_c.shape[0] == 0:
                return np.empty((0, int(n)), dtype=np.float32)
        else:
            raise ValueError(f"x must be 1-D or 2-D, got shape {x_c.shape}")
        return self.weight(weight, n, k, quant).matmul(x_c)

    # --- projections --------------------------------------------------------
    def matmul_q4k(self, x, weight, n, k):
        return self._matmul("Q4_K", x, weight, n, k)

    def matmul_q6k(self, x, weight, n, k):
        return self._matmul("Q6_K", x, weight, n, k)

    # the reference facade spells this one matmul_q6_k (python/__init__.py:184)
    matmul_q6_k = matmul_q6k

    def matmul_q8_0(self, x, weight, n, k):
        return self._matmul("Q8_0", x, weight, n, k)

    def matmul_q5k(self, x, weight, n, k):
        return self._matmul("Q5_K", x, weight, n, k)

    def matmul_q1_0(self, x, weight, n, k):
        return self._matmul("Q1_0", x, weight, n, k)

    def dispatch(self, x, weight, n, k, quant):
        """Route by on-disk quant tag (backend.py:131-156); F32/unknown tags
        keep the reference's ``weight @ x``."""
        method = QUANT_DISPATCH.get(quant or "")
        if method is None:
            return weight @ x
        return getattr(self, method)(x, weight, n, k)

    # --- dequant (validation path) ------------------------------------------
    def dequant(self, weight, shape, quant: str) -> np.ndarray:
        """Bit-exact dequant of a whole tensor on the GPU, as the reference
        NumPy decoders (dequant/gguf.py) compute it."""
        lib = self._require()
        raw = _raw_bytes(weight)
        shape = tuple(int(s) for s in shape)
        n_elems = int(np.prod(shape)) if shape else 1
        out = np.empty(n_elems, dtype=np.float32)
        fn = getattr(lib, f"frc_dequant_{quant.lower()}")
        _lib.check(fn(raw.ctypes.data, raw.nbytes, n_elems, 1, out.ctypes.data), lib)
        return out.reshape(shape)

    def dequant_q4k(self, weight, shape):
        return self.dequant(weight, shape, "Q4_K")

    def dequant_q6k(self, weight, shape):
        return self.dequant(weight, shape, "Q6_K")

    def dequant_q8_0(self, weight, shape):
        return self.dequant(weight, shape, "Q8_0")

    def dequant_q5k(self, weight, shape):
        return self.dequant(weight, shape, "Q5_K")

    def dequant_q1_0(self, weight, shape):
        return self.dequant(weight, shape, "Q1_0")


def block_geometry(quant: str) -> tuple[int, int]:
    return FORMATS[quant]


__all__ = ["CudaBackend", "DeviceWeight", "ShardedWeight", "QUANT_DISPATCH", "devices_from_env"]
