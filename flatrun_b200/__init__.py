"""flatrun_b200: B200 (sm_100a) backend for Flatrun's fused GGUF
block-dequantise + matrix-vector product (Q8_0, Q4_K, Q5_K, Q6_K, Q1_0).

``CudaBackend`` takes the slot of the reference's ``NativeBackend``
(src/flatrun/runtime/backend.py); ``flatrun_b200.integration`` registers it
as ``--backend cuda`` when the reference package is importable.
"""

from .backend import CudaBackend, DeviceWeight

__all__ = ["CudaBackend", "DeviceWeight"]
