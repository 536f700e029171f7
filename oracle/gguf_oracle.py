"""CPU oracle for the GGUF block-dequantise + matvec path.

TEST INFRASTRUCTURE ONLY. This module is the checker that the CUDA path is
compared against; it is never called by the product (``flatrun_b200``). Only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg and
``--impl reference`` arm of ``bench.py`` may import it.

It restates, in NumPy, the reference's pure-NumPy decoders in
``src/flatrun/dequant/gguf.py`` and the fp32 projection path of
``src/flatrun/runtime/backend.py`` (``PythonBackend``: dequant to F32, then a
BLAS product). The restatement keeps the reference's floating-point operation
order exactly, so the decoded weights are bit-identical to the reference's:

* Q8_0  ``q * d``                                  (gguf.py:112-127)
* Q4_K  ``((d * sc) * q) - (dmin * m)`` in fp32     (gguf.py:166-220)
* Q5_K  the same expression evaluated in float64 and rounded once to fp32:
  the reference adds ``np.where(qh & bit, 16.0, 0.0)`` (a float64 array) to the
  fp32 nibble, which promotes the whole expression (gguf.py:257-262)
* Q6_K  ``(d * sc) * q`` in fp32 with ``q`` in [-32, 31] (gguf.py:365-420)
* Q1_0  ``(+1 | -1) * d``, bits taken LSB-first       (gguf.py:266-299)

Parity pin: ``tests/golden/make_golden.py`` generated the fixtures in
``tests/golden/`` by importing the reference itself; ``tests/test_oracle.py``
checks this module against them bit for bit, and against the hand-derived
vectors in the reference's ``src/flatrun/tests/test_dequant.py``.
"""

from __future__ import annotations

import numpy as np

# name -> (elements per block, bytes per block); GGML type table in
# src/flatrun/backend/gguf.py:59-86.
FORMATS: dict[str, tuple[int, int]] = {
    "Q8_0": (32, 34),
    "Q4_K": (256, 144),
    "Q5_K": (256, 176),
    "Q6_K": (256, 210),
    "Q1_0": (128, 18),
}


def _blocks(raw, n_elems: int, fmt: str) -> np.ndarray:
    """View ``raw`` as (n_blocks, block_bytes) uint8, padding blocks included
    (gguf.py:29-47 accepts bytes or a uint8 array)."""
    qk, ts = FORMATS[fmt]
    nb = -(-n_elems // qk)
    arr = np.frombuffer(raw, dtype=np.uint8) if isinstance(raw, (bytes, bytearray, memoryview)) \
        else np.asarray(raw).view(np.uint8).reshape(-1)
    if arr.size != nb * ts:
        raise ValueError(f"{fmt}: expected {nb * ts} bytes for {n_elems} elements, got {arr.size}")
    return arr.reshape(nb, ts)


def _half(blk: np.ndarray, off: int) -> np.ndarray:
    """Little-endian IEEE binary16 at byte ``off`` of each block, as fp32
    (gguf.py:50-58). Subnormals, inf and NaN convert exactly."""
    return np.ascontiguousarray(blk[:, off:off + 2]).view("<f2").reshape(-1).astype(np.float32)


def unpack_scale_min_k4(sb: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """12 packed bytes -> 8 six-bit scales and 8 six-bit mins, fp32
    (gguf.py:135-163; ggml ``get_scale_min_k4``)."""
    b = sb.astype(np.uint32)
    lo, mid, hi = b[:, 0:4], b[:, 4:8], b[:, 8:12]
    sc = np.concatenate([lo & 63, (hi & 15) | ((lo >> 6) << 4)], axis=1)
    mn = np.concatenate([mid & 63, (hi >> 4) | ((mid >> 6) << 4)], axis=1)
    return sc.astype(np.float32), mn.astype(np.float32)


def _nibble_planes(qs: np.ndarray) -> np.ndarray:
    """(nb, 128) packed bytes -> (nb, 4, 2, 32) nibble values: group g holds
    the low nibbles of bytes 32g..32g+31 (elements 64g..64g+31) then the high
    nibbles (elements 64g+32..64g+63), gguf.py:205-219."""
    q = qs.reshape(-1, 4, 32)
    return np.stack([q & 0x0F, q >> 4], axis=2)


def dequant_q8_0(raw, shape) -> np.ndarray:
    n = int(np.prod(shape))
    blk = _blocks(raw, n, "Q8_0")
    d = _half(blk, 0)
    w = blk[:, 2:].view(np.int8).astype(np.float32) * d[:, None]
    return w.reshape(-1)[:n].reshape(shape)


def dequant_q4_k(raw, shape) -> np.ndarray:
    n = int(np.prod(shape))
    blk = _blocks(raw, n, "Q4_K")
    d, dmin = _half(blk, 0), _half(blk, 2)
    sc, mn = unpack_scale_min_k4(blk[:, 4:16])
    q = _nibble_planes(blk[:, 16:144]).astype(np.float32)          # (nb,4,2,32)
    scale = (d[:, None] * sc).reshape(-1, 4, 2, 1)                  # fp32(d*sc)
    offset = (dmin[:, None] * mn).reshape(-1, 4, 2, 1)              # fp32(dmin*m)
    w = scale * q - offset                                          # fp32 ops
    return w.reshape(-1)[:n].reshape(shape)


def dequant_q5_k(raw, shape) -> np.ndarray:
    n = int(np.prod(shape))
    blk = _blocks(raw, n, "Q5_K")
    d, dmin = _half(blk, 0), _half(blk, 2)
    sc, mn = unpack_scale_min_k4(blk[:, 4:16])
    qh = blk[:, 16:48]                                              # (nb,32)
    q = _nibble_planes(blk[:, 48:176]).astype(np.float64)          # (nb,4,2,32)
    bit = (1 << np.arange(8, dtype=np.uint8)).reshape(4, 2, 1)      # bit 2g / 2g+1
    q += np.where((qh[:, None, None, :] & bit) != 0, 16.0, 0.0)
    scale = (d[:, None] * sc).reshape(-1, 4, 2, 1)                  # fp32(d*sc)
    offset = (dmin[:, None] * mn).reshape(-1, 4, 2, 1)              # fp32(dmin*m)
    w = scale.astype(np.float64) * q - offset.astype(np.float64)    # float64, as the reference
    return w.astype(np.float32).reshape(-1)[:n].reshape(shape)


def dequant_q6_k(raw, shape) -> np.ndarray:
    n = int(np.prod(shape))
    blk = _blocks(raw, n, "Q6_K")
    ql = blk[:, 0:128].reshape(-1, 2, 2, 32)     # [half][ql lo 32 | ql hi 32][l]
    qh = blk[:, 128:192].reshape(-1, 2, 1, 32)   # [half][.][l]
    sc = blk[:, 192:208].view(np.int8).astype(np.float32).reshape(-1, 2, 4, 2)  # [half][j][l//16]
    d = _half(blk, 208)
    # quarter j of a 128-element half: low nibble of ql[l] (j=0), of ql[l+32]
    # (j=1), high nibble of ql[l] (j=2), of ql[l+32] (j=3); top two bits from
    # qh[l] >> 2j (gguf.py:409-419).
    nib = np.concatenate([ql & 0x0F, ql >> 4], axis=2)             # (nb,2,4,32)
    hi2 = (qh >> (2 * np.arange(4, dtype=np.uint8)).reshape(1, 1, 4, 1)) & 3
    q = nib.astype(np.float32) + (hi2 << 4).astype(np.float32) - np.float32(32.0)
    scale = d[:, None, None, None] * sc                             # fp32(d*sc) (nb,2,4,2)
    w = np.repeat(scale, 16, axis=3) * q                            # l//16 picks the scale
    return w.reshape(-1)[:n].reshape(shape)


def dequant_q1_0(raw, shape) -> np.ndarray:
    n = int(np.prod(shape))
    blk = _blocks(raw, n, "Q1_0")
    d = _half(blk, 0)
    bits = (blk[:, 2:18, None] >> np.arange(8, dtype=np.uint8)) & 1   # LSB first
    sign = np.where(bits.reshape(-1, 128) != 0, np.float32(1.0), np.float32(-1.0))
    w = sign * d[:, None]
    return w.reshape(-1)[:n].reshape(shape)


DEQUANT = {
    "Q8_0": dequant_q8_0,
    "Q4_K": dequant_q4_k,
    "Q5_K": dequant_q5_k,
    "Q6_K": dequant_q6_k,
    "Q1_0": dequant_q1_0,
}


def dequant(fmt: str, raw, n: int, k: int) -> np.ndarray:
    return DEQUANT[fmt](raw, (n, k))


def matvec_fp32(fmt: str, raw, x: np.ndarray, n: int, k: int) -> np.ndarray:
    """The reference fp32 projection: dequant to F32 then a BLAS product
    (runtime/backend.py:180-213). 1-D x (k,) -> (n,); 2-D x (seq, k) ->
    (seq, n), the orientation of the native batched entry points
    (flatrun_native/_C.cpp:154-197)."""
    w = dequant(fmt, raw, n, k)
    x = np.asarray(x, dtype=np.float32)
    return w @ x if x.ndim == 1 else x @ w.T


def matvec_fp64(fmt: str, raw, x: np.ndarray, n: int, k: int) -> np.ndarray:
    """Same product with fp64 accumulation, the error yardstick."""
    w = dequant(fmt, raw, n, k).astype(np.float64)
    x = np.asarray(x, dtype=np.float64)
    return w @ x if x.ndim == 1 else x @ w.T


def rel_err(y, y_ref) -> float:
    """max|y - y_ref| / max|y_ref|: the gate metric for matvec outputs."""
    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    denom = float(np.max(np.abs(y_ref))) if y_ref.size else 0.0
    if denom == 0.0:
        return float(np.max(np.abs(y))) if y.size else 0.0
    return float(np.max(np.abs(y - y_ref))) / denom


def term_scale(fmt: str, raw, x: np.ndarray, n: int, k: int) -> float:
    """max over rows of sum_j |w_ij x_j|: the magnitude of the terms a row
    sums, a denominator that stays meaningful when outputs cancel (few rows)."""
    w = np.abs(dequant(fmt, raw, n, k).astype(np.float64))
    xa = np.abs(np.asarray(x, dtype=np.float64))
    s = w @ xa if xa.ndim == 1 else xa @ w.T
    return float(np.max(s)) if s.size else 0.0


def norm_err(y, y_ref, scale: float) -> float:
    """max|y - y_ref| / scale (see term_scale)."""
    d = np.max(np.abs(np.asarray(y, np.float64) - np.asarray(y_ref, np.float64))) if np.size(y_ref) else 0.0
    return float(d / scale) if scale > 0 else float(d)


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    """Bit-for-bit float32 equality, with every NaN treated as equal."""
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    if a.shape != b.shape:
        return False
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all((a.view(np.uint32) == b.view(np.uint32)) | nan))
