"""Generate the golden fixtures in this directory from the reference itself.

Run in a checkout that has the reference source tree (its ``src`` directory is
put on ``sys.path``) and the reference native extension built by
``make -C oracle`` (``oracle/_ref``):

    python tests/golden/make_golden.py --ref <reference checkout>

For every format it stores, per case, the raw block bytes, an activation, and
what the reference computes on them:

* ``deq``   ``flatrun.dequant.gguf.dequant_<fmt>(raw, (n, k), np.float32)``
* ``mv``    the reference fp32 projection ``PythonBackend.matmul_*`` (Q4_K,
            Q6_K, Q8_0) or ``dequant_<fmt>(...) @ x`` (Q5_K, Q1_0, which have no
            backend method)
* ``mvb``   the batched orientation ``x2 @ dequant(...).T`` for x2 (3, k)
* ``nat``   the reference native C++ ``_C.matmul_*`` (Q4_K, Q6_K, Q8_0 only)

Cases: ``syn`` uses the benchmark distributions (flatrun_b200.synth); ``raw``
draws every byte at random, fp16 scale fields included, so subnormal, inf and
NaN scales occur (dequant only).
"""

from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from flatrun_b200 import synth  # noqa: E402

SHAPES = {  # (n, k) small enough for a few-KB fixture
    "Q8_0": (8, 256),
    "Q4_K": (6, 512),
    "Q5_K": (6, 512),
    "Q6_K": (6, 512),
    "Q1_0": (6, 512),
}


def _load_native(path: str):
    for name in os.listdir(path):
        if name.startswith("_C") and name.endswith(".so"):
            spec = importlib.util.spec_from_file_location("_C", os.path.join(path, name))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            return mod
    return None


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("FLATRUN_REFERENCE") or os.path.join(os.path.dirname(REPO), "reference"))
    args = ap.parse_args()
    sys.path.insert(0, os.path.join(args.ref, "src"))
    from flatrun.dequant import gguf
    from flatrun.runtime.backend import PythonBackend

    native = _load_native(os.path.join(REPO, "oracle", "_ref"))
    py = PythonBackend()
    deq = {
        "Q8_0": gguf.dequant_q8_0, "Q4_K": gguf.dequant_q4_k, "Q5_K": gguf.dequant_q5_k,
        "Q6_K": gguf.dequant_q6_k, "Q1_0": gguf.dequant_q1_0,
    }
    pym = {"Q8_0": py.matmul_q8_0, "Q4_K": py.matmul_q4k, "Q6_K": py.matmul_q6k}
    natm = {"Q8_0": "matmul_q8_0", "Q4_K": "matmul_q4_k", "Q6_K": "matmul_q6_k"}

    for fmt, (n, k) in SHAPES.items():
        qk, ts = synth.FORMATS[fmt]
        out = {"n": np.int64(n), "k": np.int64(k)}
        raw = synth.make_weight(fmt, n, k, seed=11)
        x = synth.make_x(k, seed=12)
        x2 = synth.make_x(k, batch=3, seed=13)
        w = deq[fmt](raw, (n, k), np.float32)
        out["syn_raw"], out["syn_x"], out["syn_x2"] = raw, x, x2
        out["syn_deq"] = w
        out["syn_mv"] = (pym[fmt](x, raw, n, k) if fmt in pym else w @ x).astype(np.float32)
        out["syn_mvb"] = (x2 @ w.T).astype(np.float32)
        if native is not None and fmt in natm:
            out["syn_nat"] = getattr(native, natm[fmt])(x, raw, n, k)
        nb_raw = 64
        rraw = synth.make_random_blocks(fmt, nb_raw, seed=21)
        out["raw_raw"] = rraw
        with np.errstate(all="ignore"):
            out["raw_deq"] = deq[fmt](rraw, (nb_raw * qk,), np.float32)
        path = os.path.join(HERE, f"golden_{fmt.lower()}.npz")
        np.savez_compressed(path, **out)
        print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
