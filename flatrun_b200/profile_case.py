"""Launch one GEMV configuration a fixed number of times (for ncu captures).

    python -m flatrun_b200.profile_case --quant Q4_K --n 18944 --k 3584 \
        [--batch 1] [--launches 6] [--copies 4] [--mats 2]

Weights are synthetic (flatrun_b200.synth), resident on cuda:0, rotated over
`copies` distinct device copies; nothing else runs, so an ncu capture with
``-k regex:gemv -s <skip> -c <count>`` sees exactly these launches.  With
``--mats M`` each launch is one fused frc_gemv_multi over M (n, k) matrices
sharing x (the gate+up launch of a layer is ``--n 18944 --k 3584 --mats 2``).
With ``--batch`` above 16 (prefill) the weights are uploaded with
frc_weight_create and each launch is frc_weight_matmul_dev (the tensor-core
GEMM: an fp16 conversion of x, then ``gemm_tc``).
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
    ap.add_argument("--mats", type=int, default=1)
    a = ap.parse_args()

    import torch

    from flatrun_b200 import _lib, synth

    lib = _lib.load()
    raw = synth.make_weight(a.quant, a.n, a.k, seed=0)
    x = synth.make_x(a.k, batch=None if a.batch == 1 else a.batch, seed=1)
    if a.batch > 16:
        handles = []
        for _ in range(a.copies):
            h = ctypes.c_void_p()
            _lib.check(lib.frc_weight_create(0, _lib.QUANT_IDS[a.quant], raw.ctypes.data, raw.nbytes, a.n, a.k,
                                             ctypes.byref(h)), lib)
            handles.append(h)
        x_d = torch.from_numpy(np.ascontiguousarray(x)).cuda()
        y_d = torch.empty((a.batch, a.n), device="cuda")
        stream = torch.cuda.current_stream()
        for i in range(a.launches):
            _lib.check(lib.frc_weight_matmul_dev(handles[i % a.copies], x_d.data_ptr(), a.batch, y_d.data_ptr(),
                                                 ctypes.c_void_p(stream.cuda_stream)), lib)
        torch.cuda.synchronize()
        for h in handles:
            lib.frc_weight_free(h)
        print(f"ok {a.quant} n={a.n} k={a.k} batch={a.batch} launches={a.launches}")
        return
    stride = (raw.nbytes + 255) // 256 * 256
    nbuf = a.copies * a.mats
    buf = torch.empty(nbuf * stride, dtype=torch.uint8, device="cuda")
    src = torch.from_numpy(raw).cuda()
    for j in range(nbuf):
        buf[j * stride:j * stride + raw.nbytes].copy_(src)
    x_d = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    ys = [torch.empty((a.batch, a.n), device="cuda") for _ in range(a.mats)]
    stream = torch.cuda.current_stream()
    q = _lib.QUANT_IDS[a.quant]
    for i in range(a.launches):
        c = i % a.copies
        if a.mats == 1:
            rc = lib.frc_gemv(q, buf.data_ptr() + c * stride, raw.nbytes, a.n, a.k, x_d.data_ptr(), a.batch,
                              ys[0].data_ptr(), ctypes.c_void_p(stream.cuda_stream))
        else:
            m = a.mats
            wp = (ctypes.c_void_p * m)(*[buf.data_ptr() + (c * m + j) * stride for j in range(m)])
            rc = lib.frc_gemv_multi(q, m, wp, (ctypes.c_size_t * m)(*([raw.nbytes] * m)),
                                    (ctypes.c_int64 * m)(*([a.n] * m)), a.k, x_d.data_ptr(), a.batch,
                                    (ctypes.c_void_p * m)(*[t.data_ptr() for t in ys]),
                                    ctypes.c_void_p(stream.cuda_stream))
        _lib.check(rc, lib)
    torch.cuda.synchronize()
    print(f"ok {a.quant} n={a.n} k={a.k} batch={a.batch} launches={a.launches}")


if __name__ == "__main__":
    main()
