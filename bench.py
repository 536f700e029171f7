"""Benchmark of the fused GGUF dequant + matvec path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload layer_q4k|q8_0|head_q6k|down_q5k|...]

Default workload (the configuration the headline metric is quoted on): one
Qwen2-7B layer's projections at batch 1 in Q4_K -- q/o 3584x3584, k/v
512x3584, gate/up 18944x3584, down 3584x18944 (131,088,384 weight bytes).  A
step is one pass over the seven matvecs.  Eight distinct copies of the layer
(1.05 GB, well above the 126 MB L2) are rotated step by step, so every step
streams its weights from HBM.

value  = algorithmic bytes (weights + x + y) per step / device time per step,
         weights and activations resident in HBM; the K steps are one CUDA
         graph replay timed with CUDA events on the launching stream.
e2e    = the same metric through the public call a user makes,
         CudaBackend.matmul_q4k(x, weight, n, k) with x in pinned host memory:
         x host->device, kernel, y device->host and a synchronise per call.
roofline: achieved GB/s of the dominant kernel (the gemv_x1 launches of the
         3584-column projections: 6 of 7 launches, 71% of the bytes) from
         per-launch CUDA events inside the timed graph, against the measured
         copy bandwidth in MEASURED_PEAKS.json.
cpu_baseline: the reference's own native kernels (flatrun_native._C, built
         from its sources into oracle/_ref) on the same layer.

Multi-GPU (--gpus N under torchrun): each rank owns an n-row shard (the
config's shapes) of every projection of an N-times taller layer, whole quant
blocks per row, and the outputs are assembled by all-gathers in the
forwarder's dependency groups (qkv, o, gate+up, down).  Per-GPU work is fixed
("weak" scaling); value = bytes of all ranks / max-over-ranks time.  The
`layer_llama70b` workload (config 5) instead splits one whole Llama-3-70B
layer's rows over the ranks ("strong" scaling).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

from flatrun_b200 import synth  # noqa: E402

METRIC = "weight-stream HBM GB/s per quant matvec"
UNIT = "GB/s"

QWEN2_7B = [  # (name, quant, n, k, gather group)
    ("q", "Q4_K", 3584, 3584, "qkv"),
    ("k", "Q4_K", 512, 3584, "qkv"),
    ("v", "Q4_K", 512, 3584, "qkv"),
    ("o", "Q4_K", 3584, 3584, "o"),
    ("gate", "Q4_K", 18944, 3584, "gateup"),
    ("up", "Q4_K", 18944, 3584, "gateup"),
    ("down", "Q4_K", 3584, 18944, "down"),
]


LLAMA3_70B = [  # one Llama-3-70B layer: hidden 8192, 64 / 8 heads of 128, FFN 28672
    ("q", "Q4_K", 8192, 8192, "qkv"),
    ("k", "Q4_K", 1024, 8192, "qkv"),
    ("v", "Q4_K", 1024, 8192, "qkv"),
    ("o", "Q4_K", 8192, 8192, "o"),
    ("gate", "Q4_K", 28672, 8192, "gateup"),
    ("up", "Q4_K", 28672, 8192, "gateup"),
    ("down", "Q4_K", 8192, 28672, "down"),
]


def shard_rows(mats, world: int):
    """Strong scaling: rank-local shapes when every projection's n rows are
    split evenly over `world` ranks (whole quant blocks per row)."""
    if any(n % world for _, _, n, _, _ in mats):
        raise ValueError(f"row counts must divide by {world}")
    return [(nm, q, n // world, k, g) for nm, q, n, k, g in mats]


def qwen2_7b_decode_token():
    """Every projection of one Qwen2-7B decode token in the Q4_K_M mix: 28
    layers, Q4_K everywhere except v and down in half of the layers (Q6_K),
    plus the Q6_K lm_head: 4,369,225,728 bytes of weights."""
    mats = []
    for i in range(28):
        hi = "Q6_K" if i % 2 == 0 else "Q4_K"
        for name, q, n, k, grp in QWEN2_7B:
            if name in ("v", "down"):
                q = hi
            mats.append((f"L{i}.{name}", q, n, k, f"L{i}.{grp}"))
    mats.append(("lm_head", "Q6_K", 152064, 3584, "head"))
    return mats


WORKLOADS = {
    "layer_q4k": dict(mats=QWEN2_7B, batch=1,
                      desc="config 2: Qwen2-7B layer projections (q,k,v,o,gate,up,down) in Q4_K, batch 1"),
    "q8_0": dict(mats=[("w", "Q8_0", 4096, 4096, "w")], batch=1, desc="config 1: Q8_0 4096x4096, batch 1"),
    "head_q6k": dict(mats=[("lm_head", "Q6_K", 152064, 3584, "w")], batch=1,
                     desc="config 3: lm_head 152064x3584 Q6_K, batch 1"),
    "head_q6k_b4": dict(mats=[("lm_head", "Q6_K", 152064, 3584, "w")], batch=4,
                        desc="config 3: lm_head 152064x3584 Q6_K, batch 4"),
    "head_q6k_b16": dict(mats=[("lm_head", "Q6_K", 152064, 3584, "w")], batch=16,
                         desc="config 3: lm_head 152064x3584 Q6_K, batch 16"),
    "down_q5k": dict(mats=[("down", "Q5_K", 3584, 18944, "w")], batch=1,
                     desc="config 3: FFN down 3584x18944 Q5_K, batch 1"),
    "down_q5k_b4": dict(mats=[("down", "Q5_K", 3584, 18944, "w")], batch=4,
                        desc="config 3: FFN down 3584x18944 Q5_K, batch 4"),
    "down_q5k_b16": dict(mats=[("down", "Q5_K", 3584, 18944, "w")], batch=16,
                         desc="config 3: FFN down 3584x18944 Q5_K, batch 16"),
    "down_q6k": dict(mats=[("down", "Q6_K", 3584, 18944, "w")], batch=1,
                     desc="Q6_K down 3584x18944, batch 1"),
    "q1_0": dict(mats=[("w", "Q1_0", 4096, 4096, "w")], batch=1, desc="Q1_0 4096x4096, batch 1"),
    "gate_q4k": dict(mats=[("gate", "Q4_K", 18944, 3584, "w")], batch=1, desc="Q4_K gate 18944x3584, batch 1"),
    "layer_llama70b": dict(mats=LLAMA3_70B, batch=1, strong=True,
                           desc="config 5: one Llama-3-70B layer's projections (q,k,v,o,gate,up,down) in Q4_K, "
                                "batch 1; under --gpus N every projection's rows are split over the N ranks "
                                "(strong scaling)"),
    "decode_qwen2_7b": dict(mats=qwen2_7b_decode_token(), batch=1,
                            desc="config 4 projections: one Qwen2-7B decode token (28 layers, Q4_K_M mix, Q6_K "
                                 "lm_head), batch 1"),
    "prefill_gate_q4k": dict(mats=[("gate", "Q4_K", 18944, 3584, "w")], batch=512,
                             desc="config 3: batched prefill, 512 tokens x 3584 through gate 18944x3584 Q4_K"),
}


def algorithmic_bytes(mats, batch: int, fused: bool = True) -> int:
    """Weights + activations read + outputs written; projections sharing an
    x (same group tag) read it once when they are fused."""
    total, seen = 0, set()
    for _, q, n, k, g in mats:
        total += synth.weight_bytes(q, n, k) + batch * n * 4
        if not fused or (g, k) not in seen:
            total += batch * k * 4
            seen.add((g, k))
    return total


def peaks() -> tuple[float, str]:
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback 6.65 TB/s"


def tensor_peak() -> tuple[float, str]:
    """Dense 16-bit tensor-core peak for a kernel timed alone (fp16 and bf16
    run at the same rate on B200)."""
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback 1.59 PFLOP/s"


# Prefill batches: the reference's batched kernels re-read the whole weight
# per token (_C.cpp:154-283), so the CPU legs time a sample of this many
# tokens and scale linearly to the full batch.
CPU_SAMPLE_TOKENS = 16


def ncu_traffic(workload: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary, if one exists for this workload."""
    path = os.path.join(REPO, "profiles", "ncu_traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(workload)
    except (OSError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling in the background."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(device_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "power_w_max": max(power) if power else None, "reasons": sorted(reasons)}


# ---------------------------------------------------------------------------
# reference CPU arm / cpu_baseline
# ---------------------------------------------------------------------------

def _load_ref_native():
    import importlib.util
    d = os.path.join(REPO, "oracle", "_ref")
    if not os.path.isdir(d):
        return None
    for name in os.listdir(d):
        if name.startswith("_C") and name.endswith(".so"):
            spec = importlib.util.spec_from_file_location("_C", os.path.join(d, name))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            return mod
    return None


_REF_FN = {"Q4_K": "matmul_q4_k", "Q6_K": "matmul_q6_k", "Q8_0": "matmul_q8_0"}


def cpu_reference_step_fn(mats, batch, host_w, xs):
    """One step of the reference's CPU path: the native C++ kernels where the
    reference has one (scalar, single-threaded on x86: q4_k.h:38-41), else its
    NumPy decoders + BLAS (restated in oracle/)."""
    nat = _load_ref_native()
    from oracle import gguf_oracle as O

    calls = []
    kinds = set()
    for (name, q, n, k, _), w, x in zip(mats, host_w, xs):
        if nat is not None and q in _REF_FN:
            fn = getattr(nat, _REF_FN[q] + ("_batched" if batch > 1 else ""))
            calls.append(lambda fn=fn, x=x, w=w, n=n, k=k: fn(x, w, n, k))
            kinds.add("reference")
        else:
            calls.append(lambda q=q, x=x, w=w, n=n, k=k: O.matvec_fp32(q, w, x, n, k))
            kinds.add("port")
    return (lambda: [c() for c in calls]), ("reference" if kinds == {"reference"} else "port")


def run_cpu(mats, batch, steps, warmup, host_w, xs):
    """Median seconds of one reference step at `batch`; above
    CPU_SAMPLE_TOKENS tokens the step runs on the first CPU_SAMPLE_TOKENS rows
    of x and is scaled by batch / CPU_SAMPLE_TOKENS."""
    scale = 1.0
    if batch > CPU_SAMPLE_TOKENS:
        xs = [np.ascontiguousarray(x[:CPU_SAMPLE_TOKENS]) for x in xs]
        scale = batch / CPU_SAMPLE_TOKENS
        batch = CPU_SAMPLE_TOKENS
    step, kind = cpu_reference_step_fn(mats, batch, host_w, xs)
    for _ in range(warmup):
        step()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        times.append((time.perf_counter() - t0) * scale)
    return statistics.median(times), sum(times), kind


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def make_host_layer(mats, copy: int):
    return [synth.make_weight(q, n, k, seed=1000 * copy + i) for i, (_, q, n, k, _) in enumerate(mats)]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="layer_q4k")
    ap.add_argument("--copies", type=int, default=0, help="distinct weight copies rotated (0 = auto, > 3x L2)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--nccl-gather", action="store_true",
                    help="N > 1: assemble row shards with NCCL all-gathers instead of the gather fused into the GEMV")
    ap.add_argument("--unfused", action="store_true",
                    help="one launch per projection, each with its own x (no shared-x fusion)")
    ap.add_argument("--batch1-int16", action="store_true",
                    help="batch 1 on the 16-bit activation grid kernel (dp4a) instead of fp32 activations")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    wl = WORKLOADS[args.workload]
    mats, batch = wl["mats"], wl["batch"]
    step_bytes = algorithmic_bytes(mats, batch, fused=not getattr(args, "unfused", False))

    if args.impl == "reference":
        if rank != 0:
            return
        host_w = make_host_layer(mats, 0)
        xs = [synth.make_x(k, batch=None if batch == 1 else batch, seed=50 + i)
              for i, (_, _, _, k, _) in enumerate(mats)]
        # bounded: at most 20 timed and 3 warm-up steps of the host kernels
        steps = max(1, min(args.steps, 20))
        warm = min(args.warmup, 3)
        med, total, kind = run_cpu(mats, batch, steps, warm, host_w, xs)
        value = step_bytes / med / 1e9
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
            "steps": steps, "warmup": warm, "ms_per_step": round(med * 1e3, 3),
            "higher_is_better": True, "scaling": "strong" if wl.get("strong") else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": wl["desc"], "global_batch": batch},
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": 1, "kind": kind,
                             "sample": f"{steps} timed steps of the full workload (median), reference "
                                       "flatrun_native._C scalar kernels (single-threaded on x86)"
                                       + (f"; {CPU_SAMPLE_TOKENS} of the {batch} tokens per step, time scaled "
                                          f"by {batch / CPU_SAMPLE_TOKENS:g}" if batch > CPU_SAMPLE_TOKENS else "")},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "tokens_per_s": round(1.0 / med, 4) if args.workload.startswith("decode") else None,
        }), flush=True)
        return

    import ctypes

    import torch

    from flatrun_b200 import CudaBackend, _lib

    # strong scaling: the workload is one whole layer, each rank owns n / N
    # rows of every projection (whole quant blocks per row)
    if wl.get("strong") and world > 1:
        mats = shard_rows(mats, world)
        step_bytes = algorithmic_bytes(mats, batch, fused=not getattr(args, "unfused", False))
    scaling = "strong" if wl.get("strong") else "weak"

    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    else:
        torch.cuda.set_device(0)
    dev = torch.cuda.current_device()
    lib = _lib.load()
    if args.batch1_int16:
        _lib.set_option("batch1_int16", 1)
    be = CudaBackend(dev)
    if not be.available:
        raise RuntimeError(f"CUDA backend unavailable: {be._load_error}")

    props = torch.cuda.get_device_properties(dev)
    l2 = getattr(props, "L2_cache_size", 126 * 2**20)
    wbytes = sum(synth.weight_bytes(q, n, k) for _, q, n, k, _ in mats)
    copies = args.copies or (1 if wbytes >= 3 * l2 else max(2, min(16, int(np.ceil(3 * l2 / wbytes)) + 1)))

    # host weights: `copies` distinct layers (row-rolled copies of one random
    # layer), uploaded through the public backend (used by the e2e leg)
    base = make_host_layer(mats, rank)
    host_arrays = []  # the host bytes each cached DeviceWeight was uploaded from
    for c in range(copies):
        hosts = []
        for (name, q, n, k, _), raw in zip(mats, base):
            rb = synth.row_bytes(q, k)
            host = raw if c == 0 else np.ascontiguousarray(
                np.roll(raw.reshape(n, rb), c * 7919 % n, axis=0)).reshape(-1)
            be.weight(host, n, k, q)
            hosts.append(host)
        host_arrays.append(hosts)

    # device-resident pools for the timed graphs: per matrix, enough distinct
    # copies (>= 3x L2 of bytes) that no launch finds its weight in L2, even
    # when one projection is timed alone
    pools = []  # (buffer, stride, ncopies)
    for (name, q, n, k, _), raw in zip(mats, base):
        nb = max(int(raw.nbytes), 1)
        stride = (nb + 255) // 256 * 256
        # a step that streams >= 3x L2 of weights re-reads nothing from L2
        nc = 1 if wbytes >= 3 * l2 else int(min(1024, max(2, np.ceil(3 * l2 / nb))))
        buf = torch.empty(nc * stride, dtype=torch.uint8, device="cuda")
        src = torch.from_numpy(raw).cuda()
        for j in range(nc):
            buf[j * stride:j * stride + raw.nbytes].copy_(src)
        pools.append((buf, stride, nc))
    xs_host = [synth.make_x(k, batch=None if batch == 1 else batch, seed=50 + i)
               for i, (_, _, _, k, _) in enumerate(mats)]
    xs_dev = [torch.from_numpy(x).cuda() for x in xs_host]
    ys_dev = [torch.empty((batch, n), device="cuda") for (_, _, n, _, _) in mats]
    qid = [_lib.QUANT_IDS[q] for _, q, _, _, _ in mats]
    mbytes = [synth.weight_bytes(q, n, k) for _, q, n, k, _ in mats]

    # launch groups: projections that share x run as one fused launch
    # (frc_gemv_multi), the forwarder's dataflow (q/k/v, gate/up)
    lgroups = []
    for i, m in enumerate(mats):
        if not args.unfused and lgroups and mats[lgroups[-1][0]][4] == m[4] and mats[lgroups[-1][0]][1] == m[1] \
                and mats[lgroups[-1][0]][3] == m[3] and len(lgroups[-1]) < 4:
            lgroups[-1].append(i)
        else:
            lgroups.append([i])
    # the members of a group read the same x
    for g in lgroups:
        for i in g[1:]:
            xs_dev[i] = xs_dev[g[0]]
            xs_host[i] = xs_host[g[0]]

    # all-gather groups (N > 1)
    groups = []
    if world > 1:
        import torch.distributed as dist
        order = []
        for i, m in enumerate(mats):
            if not order or order[-1][0] != m[4]:
                order.append((m[4], []))
            order[-1][1].append(i)
        for gname, idx in order:
            local = sum(mats[i][2] for i in idx) * batch
            sendbuf = torch.empty(local, device="cuda")
            # the projections write their y shards straight into the send buffer
            off = 0
            for j in idx:
                sz = mats[j][2] * batch
                ys_dev[j] = sendbuf[off:off + sz].view(batch, mats[j][2])
                off += sz
            groups.append((idx[-1], sendbuf, torch.empty(local * world, device="cuda"), idx))

    stream = torch.cuda.Stream()

    def gemv(i: int, step: int) -> None:
        buf, stride, nc = pools[i]
        _, q, n, k, _ = mats[i]
        rc = lib.frc_gemv(qid[i], buf.data_ptr() + (step % nc) * stride, mbytes[i], n, k, xs_dev[i].data_ptr(),
                          batch, ys_dev[i].data_ptr(), ctypes.c_void_p(stream.cuda_stream))
        if rc:
            _lib.check(rc, lib)

    def gemv_group(g: list, step: int) -> None:
        if len(g) == 1:
            gemv(g[0], step)
            return
        cnt = len(g)
        wp = (ctypes.c_void_p * cnt)(*[pools[i][0].data_ptr() + (step % pools[i][2]) * pools[i][1] for i in g])
        wb = (ctypes.c_size_t * cnt)(*[mbytes[i] for i in g])
        nn = (ctypes.c_int64 * cnt)(*[mats[i][2] for i in g])
        yp = (ctypes.c_void_p * cnt)(*[ys_dev[i].data_ptr() for i in g])
        rc = lib.frc_gemv_multi(qid[g[0]], cnt, wp, wb, nn, mats[g[0]][3], xs_dev[g[0]].data_ptr(), batch, yp,
                                ctypes.c_void_p(stream.cuda_stream))
        if rc:
            _lib.check(rc, lib)

    # N > 1, batch 1: the all-gather fused into the GEMV (each rank's GEMV
    # stores its rows into every rank's gathered buffer over NVLink, then a
    # bounded wait), where the launch group is exactly one gather group
    fused = {}
    if world > 1 and batch == 1 and not args.nccl_gather:
        from flatrun_b200.shard import FusedGather
        for last, sendbuf, recvbuf, idx in groups:
            if idx in lgroups:
                fused[tuple(idx)] = (FusedGather(lib, world, rank, sendbuf.numel()), sendbuf)

    # each fused launch waits (before reading x) for the previous group's
    # gather, as the forwarder's next projection consumes it; the chain runs
    # across steps (q+k+v waits for the previous step's down)
    chain = {"prev": None}

    def fused_group(g: list, step: int) -> bool:
        fg, sendbuf = fused[tuple(g)]
        w = [pools[i][0].data_ptr() + (step % pools[i][2]) * pools[i][1] for i in g]
        rc = fg.gemv(qid[g[0]], w, [mbytes[i] for i in g], [mats[i][2] for i in g], mats[g[0]][3],
                     xs_dev[g[0]].data_ptr(), [ys_dev[i].data_ptr() for i in g], sendbuf.data_ptr(),
                     stream.cuda_stream, wait_for=chain["prev"])
        if rc == _lib.FRC_ERR_UNSUPPORTED:
            return False
        _lib.check(rc, lib)
        chain["prev"] = fg
        return True

    def launch(step: int, only=None) -> None:
        for g in lgroups:
            if only is not None and g[0] not in only:
                continue
            if only is None and tuple(g) in fused and fused_group(g, step):
                continue
            gemv_group(g, step)
            i = g[-1]
            for last, sendbuf, recvbuf, idx in groups:
                if only is None and last == i:
                    dist.all_gather_into_tensor(recvbuf, sendbuf)

    K = args.steps
    chunk = min(K, 256)

    def capture(only=None):
        graphs = []
        with torch.cuda.stream(stream):
            for g0 in range(0, K, chunk):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for s in range(g0, min(K, g0 + chunk)):
                        launch(s, only)
                graphs.append(g)
        return graphs

    def replay_ms(graphs) -> float:
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            start.record(stream)
            for g in graphs:
                g.replay()
            end.record(stream)
        end.synchronize()
        return start.elapsed_time(end)

    torch.cuda.synchronize()
    clocks = ClockSampler(dev if world == 1 else local_rank)
    with torch.cuda.stream(stream):
        for s in range(args.warmup):
            launch(s)
    torch.cuda.synchronize()
    graphs = capture()
    # soak: replay untimed for ~1 s so clocks settle and the sampler sees load;
    # every rank replays the same number of times (the graphs hold collective
    # steps), agreed on from the first replay
    n_soak = max(1, int(np.ceil(1000.0 / max(replay_ms(graphs), 1e-3))))
    if world > 1:
        t = torch.tensor([n_soak], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        n_soak = int(t.item())
    for _ in range(n_soak - 1):
        replay_ms(graphs)

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    elapsed_ms = replay_ms(graphs)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()

    if world > 1:
        t = torch.tensor([elapsed_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_step = elapsed_ms / K
    value = step_bytes * world / (ms_step / 1e3) / 1e9

    # per-launch time: K back-to-back launches of one group (a fused launch
    # or a single projection), one graph replay bracketed by CUDA events
    # launches of the same shapes (e.g. every layer's gate+up) are timed once,
    # rotating over those launches' weights so that none is re-read from L2
    sigs = {}
    for g in lgroups:
        sigs.setdefault(tuple((mats[i][1], mats[i][2], mats[i][3]) for i in g), []).append(g)
    per = {}
    for gs in sigs.values():
        g = gs[0]
        name = "+".join(mats[i][0] for i in g) + (f" (x{len(gs)})" if len(gs) > 1 else "")
        gi = []
        with torch.cuda.stream(stream):
            for g0 in range(0, K, chunk):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    for st_ in range(g0, min(K, g0 + chunk)):
                        gemv_group(gs[st_ % len(gs)], st_)
                gi.append(gr)
        replay_ms(gi)
        us = replay_ms(gi) * 1e3 / K
        b = sum(mbytes[i] + batch * (mats[i][3] + mats[i][2]) * 4 for i in g) - (len(g) - 1) * batch * mats[g[0]][3] * 4
        per[name] = {"us": round(us, 3), "gbs": round(b / (us / 1e6) / 1e9, 1), "bytes": b}
        del gi
    # dominant kernel: the launch carrying the most bytes
    dom_name = max(per, key=lambda nm: per[nm]["bytes"])
    achieved = per[dom_name]["bytes"] / (per[dom_name]["us"] / 1e6) / 1e9
    peak, peak_src = peaks()
    traffic = ncu_traffic(args.workload)

    # e2e through the public call, host buffers (pinned x), synchronous calls
    e2e = None
    if not args.no_e2e and world == 1:
        method = {"Q4_K": be.matmul_q4k, "Q6_K": be.matmul_q6k, "Q8_0": be.matmul_q8_0,
                  "Q5_K": be.matmul_q5k, "Q1_0": be.matmul_q1_0}
        pinned = []
        for x in xs_host:
            t = torch.empty(x.shape, dtype=torch.float32, pin_memory=True)
            t.numpy()[...] = x
            pinned.append(t.numpy())
        e2e_steps = min(K, 200)
        for s in range(3):
            for i, (_, q, n, k, _) in enumerate(mats):
                method[q](pinned[i], host_arrays[s % copies][i], n, k)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for s in range(e2e_steps):
            for i, (_, q, n, k, _) in enumerate(mats):
                method[q](pinned[i], host_arrays[s % copies][i], n, k)
        t_e2e = (time.perf_counter() - t0) / e2e_steps
        e2e = {"value": round(step_bytes / t_e2e / 1e9, 2), "unit": UNIT,
               "h2d_bytes_per_step": sum(batch * k * 4 for _, _, _, k, _ in mats),
               "d2h_bytes_per_step": sum(batch * n * 4 for _, _, n, _, _ in mats),
               "ms_per_step": round(t_e2e * 1e3, 4), "steps": e2e_steps,
               "tokens_per_s": round(1.0 / t_e2e, 2) if args.workload.startswith("decode") else None,
               "timer": "host wall clock over synchronous calls (each call copies x in, y out and synchronises)"}

    # CPU baseline: the reference's own native kernels on the same workload
    cpu = None
    if not args.no_cpu and rank == 0:
        med, total, kind = run_cpu(mats, batch, 3, 1, base, xs_host)
        cpu = {"value": round(step_bytes / med / 1e9, 4), "unit": UNIT, "cores": 1, "kind": kind,
               "sample": "3 timed passes over the full workload (median) after 1 warm-up, reference "
                         "flatrun_native._C built from its sources (scalar, single-threaded on x86)"
                         + (f"; {CPU_SAMPLE_TOKENS} of the {batch} tokens per pass, time scaled by "
                            f"{batch / CPU_SAMPLE_TOKENS:g}" if batch > CPU_SAMPLE_TOKENS else "")}

    if rank == 0:
        # the kernel family each call runs: batch 1 dp4a GEMV, 2..16 int8
        # tensor-core GEMV (pre-pass + main), more: tcgen05 GEMM (fp16 pre-pass
        # + main)
        if batch == 1:
            kname, dtype, calls_per_group = "gemv_b1 (fp32 activations)", "f32", lambda g: 1
        elif batch <= 16:
            kname, dtype, calls_per_group = "gemv_mma", "s8 x s8 -> s32 (mma.sync), fp32 scales", lambda g: 2 * len(g)
        else:
            kname, dtype, calls_per_group = "gemm_tc", "f16 x f16 -> f32 (tcgen05)", lambda g: 2 * len(g)
        if batch > 16:
            # tensor-bound: FLOPs of the dominant launch over its device time
            dom_group = next(g for g in lgroups if dom_name.startswith("+".join(mats[i][0] for i in g)))
            flops = sum(2.0 * mats[i][2] * mats[i][3] * batch for i in dom_group)
            tpk, tpk_src = tensor_peak()
            tflops = flops / (per[dom_name]["us"] / 1e6) / 1e12
            roof = {"bound": "tensor", "achieved": round(tflops, 1), "peak": tpk, "unit": "TFLOP/s",
                    "frac": round(tflops / tpk, 4), "traffic": traffic, "peak_source": tpk_src,
                    "flops_per_launch": flops}
        else:
            roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "traffic": traffic, "peak_source": peak_src}
        roof["kernel"] = f"{kname} <{mats[0][1]}> launch '{dom_name}' ({per[dom_name]['bytes'] / 1e6:.1f} MB per launch)"
        roof["timing"] = ("K back-to-back launches of the dominant launch, one CUDA graph replay bracketed by CUDA "
                          "events on the launching stream")
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None, "dtype": dtype, "data": "synthetic",
            "config": {"workload": wl["desc"], "global_batch": (batch if batch <= 16 else 1) * world,
                       "seq_len": 1 if batch <= 16 else batch,
                       "parallelism": f"row-shard x{world}" if world > 1 else "single GPU",
                       "gather": ("fused into the GEMV: stores to every rank over NVLink; the next GEMV waits for "
                                  "every rank's flag before reading x" if fused else "NCCL all_gather_into_tensor")
                                 if world > 1 else None,
                       "weight_bytes_per_step": wbytes, "algorithmic_bytes_per_step": step_bytes,
                       "weight_copies_rotated": [p[2] for p in pools],
                       "l2": f"inputs larger than L2: each projection rotates over distinct device copies "
                             f"totalling >= 3x L2 ({sum(p[2] * mbytes[i] for i, p in enumerate(pools)) / 1e9:.2f} GB);"
                             f" L2 {l2 / 2**20:.0f} MiB"},
            "frac_of_8tbs": round(value / world / 8000.0, 4),
            "tokens_per_s": round(1e3 / ms_step, 2) if args.workload.startswith("decode") else None,
            "roofline": roof,
            "per_launch": per,
            "launches_per_step": len(lgroups),
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clk,
            "gpu_launches": K * sum(calls_per_group(g) for g in lgroups),
        }
        print(json.dumps(out), flush=True)

    del graphs, pools
    if world > 1:
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier()
        for fg, _ in fused.values():
            fg.close()
        dist.barrier()
        dist.destroy_process_group()
    be.close()


if __name__ == "__main__":
    main()
