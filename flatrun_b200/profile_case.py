"""Launch one GEMV configuration a fixed number of times (for ncu captures).

    python -m flatrun_b200.profile_case --quant Q4_K --n 18944 --k 3584 \
        [--batch 1] [--launches 6] [--copies 4]

Weights are synthetic (flatrun_b200.synth), resident on cuda:0, rotated over
`copies` distinct device copies; nothing else runs, so an ncu capture with
``-k regex:gemv -s <skip> -c <count>`` sees exactly these launches.
"""

from __future__ import annotations

import argparse
import ctypes

import numpy as np


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--quant", default="Q4_K")
    ap.add_argument("--n", type=int, default=18944)
    ap.add_argument("--k", type=int, default=3584)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--launches", type=int, default=6)
    ap.add_argument("--copies", type=int, default=4)
    a = ap.parse_args()

    import torch

    from flatrun_b200 import _lib, synth

    lib = _lib.load()
    raw = synth.make_weight(a.quant, a.n, a.k, seed=0)
    x = synth.make_x(a.k, batch=None if a.batch == 1 else a.batch, seed=1)
    stride = (raw.nbytes + 255) // 256 * 256
    buf = torch.empty(a.copies * stride, dtype=torch.uint8, device="cuda")
    src = torch.from_numpy(raw).cuda()
    for j in range(a.copies):
        buf[j * stride:j * stride + raw.nbytes].copy_(src)
    x_d = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    y_d = torch.empty((a.batch, a.n), device="cuda")
    stream = torch.cuda.current_stream()
    for i in range(a.launches):
        rc = lib.frc_gemv(_lib.QUANT_IDS[a.quant], buf.data_ptr() + (i % a.copies) * stride, raw.nbytes, a.n, a.k,
                          x_d.data_ptr(), a.batch, y_d.data_ptr(), ctypes.c_void_p(stream.cuda_stream))
        _lib.check(rc, lib)
    torch.cuda.synchronize()
    print(f"ok {a.quant} n={a.n} k={a.k} batch={a.batch} launches={a.launches}")


if __name__ == "__main__":
    main()
