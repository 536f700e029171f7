"""Plug ``CudaBackend`` into an unchanged Flatrun installation.

The reference selects its projection backend by name through
``flatrun.runtime.backend.get_backend`` and the ``_BACKENDS`` registry
(src/flatrun/runtime/backend.py:284-315); ``flatrun run/chat/serve`` pass
``--backend`` to it (src/flatrun/cli.py:1032-1042, :1610).  The NumPy
forwarder only dispatches a layer's projections to a backend whose ``name``
is ``"native"`` and whose quant tags are all in its local ``{Q4_K, Q6_K,
Q8_0}`` set (src/flatrun/model/qwen2.py:1452-1472, :2247-2252).

``register()`` adds two registry entries without editing the reference:

* ``"cuda"``        -> :class:`CudaSlotBackend`: a ``BackendBase`` whose
  ``name`` is ``"cuda"`` (what ``get_backend("cuda")`` and tooling see);
* ``"native-cuda"`` -> :class:`NativeSlotAdapter`: the same backend answering
  ``name == "native"``, the spelling the unchanged forwarder's gate checks, so
  ``make_qwen2_forwarder(..., backend=get_backend("native-cuda"))`` routes every
  supported projection to the GPU.

Neither falls back to NumPy: a kernel error raises (the reference's
``NativeBackend._try_kernel`` would fall back, backend.py:259-268).
"""

from __future__ import annotations

from typing import Any

from .backend import CudaBackend, devices_from_env


def _make_classes(rb):
    class CudaSlotBackend(rb.BackendBase):
        """``BackendBase`` implementation over :class:`CudaBackend`."""

        def __init__(self, device: int | None = None) -> None:
            # the reference's get_backend(name) passes no arguments: the GPUs
            # come from FLATRUN_CUDA_DEVICES (several ids: every projection's
            # rows are split over them), else device 0
            devs = [device] if device is not None else devices_from_env()
            self._cuda = CudaBackend(devs[0], devices=devs)

        @property
        def name(self) -> str:
            return "cuda"

        @property
        def available(self) -> bool:
            return self._cuda.available

        @property
        def supported_quants(self) -> set[str]:
            return self._cuda.supported_quants

        def matmul_q4k(self, x: Any, weight: Any, n: int, k: int):
            return self._cuda.matmul_q4k(x, weight, n, k)

        def matmul_q6k(self, x: Any, weight: Any, n: int, k: int):
            return self._cuda.matmul_q6k(x, weight, n, k)

        def matmul_q8_0(self, x: Any, weight: Any, n: int, k: int):
            return self._cuda.matmul_q8_0(x, weight, n, k)

        def matmul_q5k(self, x: Any, weight: Any, n: int, k: int):
            return self._cuda.matmul_q5k(x, weight, n, k)

        def matmul_q1_0(self, x: Any, weight: Any, n: int, k: int):
            return self._cuda.matmul_q1_0(x, weight, n, k)

        def dispatch(self, x: Any, weight: Any, n: int, k: int, quant: str | None):
            return self._cuda.dispatch(x, weight, n, k, quant)

        def close(self) -> None:
            self._cuda.close()

    class NativeSlotAdapter(CudaSlotBackend):
        """The CUDA backend under the name the forwarder's gate expects."""

        @property
        def name(self) -> str:
            return "native"

    return CudaSlotBackend, NativeSlotAdapter


def register(backend_module: Any = None) -> tuple[type, type]:
    """Register ``"cuda"`` and ``"native-cuda"`` in the reference's backend
    registry (``flatrun.runtime.backend._BACKENDS``) and return the classes."""
    if backend_module is None:
        from flatrun.runtime import backend as backend_module  # type: ignore[import-not-found]
    slot, adapter = _make_classes(backend_module)
    backend_module._BACKENDS["cuda"] = slot
    backend_module._BACKENDS["native-cuda"] = adapter
    return slot, adapter


def extend_forwarder_method_table(qwen2_module: Any = None) -> None:
    """Add Q5_K and Q1_0 to the forwarder's module-level quant -> method table
    (src/flatrun/model/qwen2.py:756-760).  The per-layer gate also consults a
    set local to ``_decoder_block`` (qwen2.py:1452) that cannot be patched from
    outside, so layers with Q5_K/Q1_0 projections still take the NumPy path;
    the LM head (qwen2.py:2247-2252) uses the table and does reach the GPU."""
    if qwen2_module is None:
        from flatrun.model import qwen2 as qwen2_module  # type: ignore[import-not-found]
    qwen2_module._NATIVE_METHOD.setdefault("Q5_K", "matmul_q5k")
    qwen2_module._NATIVE_METHOD.setdefault("Q1_0", "matmul_q1_0")


__all__ = ["register", "extend_forwarder_method_table"]
