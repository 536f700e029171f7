"""Seeded synthetic GGUF weights and activations.

The workloads have no dataset: the shapes and value distributions are those
the benchmark configurations name (GGUF block layouts as in the reference's
``src/flatrun/dequant/gguf.py``):

* Q8_0  d = fp16(|N(0,1)| * 0.01); 32 int8 quants uniform in [-127, 127]
* Q4_K  d, dmin = fp16(|N(0,1)| * 0.01); the 12 packed scale/min bytes uniform
        in [0, 255] (a bijection onto uniform 6-bit scales and mins); the 128
        quant bytes uniform (both nibbles exercised)
* Q5_K  as Q4_K plus 32 uniform high-bit bytes
* Q6_K  ql, qh uniform bytes; 16 int8 sub-scales uniform in [-32, 31];
        d = fp16(|N(0,1)| * 0.005)
* Q1_0  d = fp16(|N(0,1)| * 0.01); 16 uniform sign-bit bytes
* x     fp32 ~ N(0, 1)

Every byte of every quant field is drawn at full width, unlike the reference's
own parity generators (which leave high nibbles and upper qh bits at zero).
"""

from __future__ import annotations

import numpy as np

FORMATS: dict[str, tuple[int, int]] = {
    "Q8_0": (32, 34),
    "Q4_K": (256, 144),
    "Q5_K": (256, 176),
    "Q6_K": (256, 210),
    "Q1_0": (128, 18),
}


def row_bytes(fmt: str, k: int) -> int:
    qk, ts = FORMATS[fmt]
    if k % qk:
        raise ValueError(f"{fmt}: k={k} is not a multiple of {qk}")
    return (k // qk) * ts


def weight_bytes(fmt: str, n: int, k: int) -> int:
    return n * row_bytes(fmt, k)


def _scale(rng: np.random.Generator, nb: int, mult: float) -> np.ndarray:
    return (np.abs(rng.standard_normal(nb)) * mult).astype(np.float16).view(np.uint8).reshape(nb, 2)


def make_weight(fmt: str, n: int, k: int, seed: int = 0) -> np.ndarray:
    """Raw GGUF bytes (1-D uint8) of an (n, k) row-major weight."""
    qk, ts = FORMATS[fmt]
    nb = n * (k // qk)
    row_bytes(fmt, k)
    rng = np.random.default_rng(seed)
    blk = np.empty((nb, ts), dtype=np.uint8)
    if fmt == "Q8_0":
        blk[:, 0:2] = _scale(rng, nb, 0.01)
        blk[:, 2:34] = rng.integers(-127, 128, size=(nb, 32), dtype=np.int8).view(np.uint8)
    elif fmt in ("Q4_K", "Q5_K"):
        blk[:, 0:2] = _scale(rng, nb, 0.01)
        blk[:, 2:4] = _scale(rng, nb, 0.01)
        blk[:, 4:ts] = rng.integers(0, 256, size=(nb, ts - 4), dtype=np.uint8)
    elif fmt == "Q6_K":
        blk[:, 0:192] = rng.integers(0, 256, size=(nb, 192), dtype=np.uint8)
        blk[:, 192:208] = rng.integers(-32, 32, size=(nb, 16), dtype=np.int8).view(np.uint8)
        blk[:, 208:210] = _scale(rng, nb, 0.005)
    elif fmt == "Q1_0":
        blk[:, 0:2] = _scale(rng, nb, 0.01)
        blk[:, 2:18] = rng.integers(0, 256, size=(nb, 16), dtype=np.uint8)
    else:
        raise ValueError(f"unknown format {fmt!r}")
    return blk.reshape(-1)


def pack_k_scales(sc: np.ndarray, m: np.ndarray) -> np.ndarray:
    """The 12 packed bytes of 8 six-bit scales and mins per K-quant block
    (the inverse of the unpack in dequant/gguf.py:135-163): for j < 4 byte j
    is sc[j] with the top two bits of sc[j+4] in bits 6-7, byte j+4 is m[j]
    with the top bits of m[j+4]; byte j+8 holds the low nibbles of sc[j+4]
    and m[j+4]."""
    sc = sc.astype(np.uint8)
    m = m.astype(np.uint8)
    out = np.empty(sc.shape[:-1] + (12,), np.uint8)
    out[..., 0:4] = sc[..., 0:4] | ((sc[..., 4:8] >> 4) << 6)
    out[..., 4:8] = m[..., 0:4] | ((m[..., 4:8] >> 4) << 6)
    out[..., 8:12] = (sc[..., 4:8] & 0x0F) | ((m[..., 4:8] & 0x0F) << 4)
    return out


def make_centered_q4_k(n: int, k: int, seed: int = 0) -> np.ndarray:
    """Q4_K blocks whose weights have mean ~0, as trained K-quants do (for
    random-init models run for many layers): dmin = d = fp16(|N(0,1)| *
    0.01), scales uniform in [1, 8], mins round(7.5 * scale), so
    d*sc*q - dmin*m is centred on the nibble range's middle; quant bytes
    uniform.  The matvec benchmarks' distribution (uniform scales and mins,
    make_weight) has mean ~1.6 per weight, which makes a residual stream
    grow without bound over many layers."""
    nb = n * (k // 256)
    row_bytes("Q4_K", k)
    rng = np.random.default_rng(seed)
    blk = np.empty((nb, 144), np.uint8)
    d = (np.abs(rng.standard_normal(nb)) * 0.01).astype(np.float16).view(np.uint8).reshape(nb, 2)
    blk[:, 0:2] = d
    blk[:, 2:4] = d
    sc = rng.integers(1, 9, size=(nb, 8))
    blk[:, 4:16] = pack_k_scales(sc, np.rint(7.5 * sc))
    blk[:, 16:144] = rng.integers(0, 256, size=(nb, 128), dtype=np.uint8)
    return blk.reshape(-1)


def make_random_blocks(fmt: str, n_blocks: int, seed: int = 0) -> np.ndarray:
    """Fully random bytes, scale fields included (so fp16 subnormals, inf and
    NaN scales occur): an edge-case generator for bit-exact dequant checks."""
    _, ts = FORMATS[fmt]
    rng = np.random.default_rng(seed)
    return rng.integers(0, 256, size=n_blocks * ts, dtype=np.uint8)


def make_x(k: int, batch: int | None = None, seed: int = 1) -> np.ndarray:
    rng = np.random.default_rng(seed)
    shape = (k,) if batch is None else (batch, k)
    return rng.standard_normal(shape).astype(np.float32)
