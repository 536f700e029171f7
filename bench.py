"""Benchmark of the fused GGUF dequant + matvec path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload layer_llama70b|layer_q4k|q8_0|head_q6k|...]

Default workload, at every N (config 5): one Llama-3-70B layer's projections
at batch 1 in Q4_K -- q/o 8192x8192, k/v 1024x8192, gate/up 28672x8192,
down 8192x28672 (481.8 MB of weights).  A step is one pass over the seven
matvecs in the forwarder's dataflow: q/k/v and gate/up each run as one fused
launch over matrices sharing x, so four launches.  Under torchrun (--gpus N)
every projection's rows are split over the N ranks (whole quant blocks per
row) and each launch assembles its outputs on every rank with the all-gather
fused into the GEMV (peer stores over NVLink): strong scaling, value = bytes
of the whole layer / max-over-ranks step time.  Per matrix, distinct device
copies totalling >= 3x L2 are rotated step by step, so every launch streams
its weights from HBM.  Other workloads: config 2 (`layer_q4k`, one Qwen2-7B
layer, weak scaling under N ranks), config 1 (`q8_0`), config 3 (`head_q6k*`,
`down_q5k*`, `prefill_gate_q4k`), config 4's projections (`decode_qwen2_7b`).

value  = algorithmic bytes (weights + x + y) per step / device time per step,
         weights and activations resident in HBM; the K steps are CUDA graph
         replays timed with CUDA events on the launching stream.
e2e    = the same metric through the public call a user makes,
         CudaBackend.matmul_q4k(x, weight, n, k) with x in pinned host memory:
         x host->device, kernel, y device->host and a synchronise per call
         (N > 1: each rank its own shard, the slowest rank's time).
kernels: batch-1 Q4_K and Q5_K on gemv_tc1 (x in fp32 as three exact fp16
         terms, weights as exact fp16 q*sc, products on the tensor cores,
         fp32 accumulation); rows whose activation fragments do not fit in
         shared memory (the k = 28672 down) run in parts of k on clusters of
         CTAs, one part each; the other formats on the fp32 CUDA-core
         gemv_b1; --cuda-core forces the latter for Q4_K too.
roofline: achieved GB/s of the dominant launch (the one carrying the most
         bytes: gate+up for the layer workloads) from K back-to-back launches
         timed with CUDA events, against the measured copy bandwidth in
         MEASURED_PEAKS.json.
cpu_baseline / cpu_baseline_numpy: the reference's native C++ kernels
         (flatrun_native._C built from its sources into oracle/_ref, one core)
         and its NumPy + BLAS path (restated in oracle/), each on a bounded
         row sample of the same workload (N = 1, rank 0).
assembly_share / gather_check (N > 1): the share of the step the output
         assembly adds to the GEMVs alone, and an in-run bit-exact check of
         the assembled outputs on every rank.
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
    "decode_qwen2_7b_device": dict(mats=qwen2_7b_decode_token(), batch=1, device_decode=True,
                                   desc="config 4: one Qwen2-7B decode token entirely on the GPU (28 layers, Q4_K_M "
                                        "mix, Q6_K lm_head, KV cache pre-filled with 4096 positions; embedding, "
                                        "norms, RoPE, attention, SwiGLU, head and argmax on the device, one CUDA "
                                        "graph per token), greedy, batch 1"),
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


def sample_rows(mats, host_w, frac: float):
    """The first ceil(frac * n) rows of every projection (whole rows, hence
    whole quant blocks): a bounded sample of the workload for the CPU legs."""
    out_m, out_w = [], []
    for (name, q, n, k, g), w in zip(mats, host_w):
        ns = max(1, min(n, int(np.ceil(frac * n))))
        out_m.append((name, q, ns, k, g))
        out_w.append(w[: ns * synth.row_bytes(q, k)])
    return out_m, out_w


def cpu_step_fn(mats, batch, host_w, xs, path: str):
    """One pass of a reference CPU path over the projections.

    path "native": the reference's own C++ kernels (flatrun_native._C, built
    from its sources into oracle/_ref; scalar and single-threaded on x86,
    kernels/q4_k.h:38-41, _C.cpp:190-194), and for the formats it has no
    kernel for (Q5_K, Q1_0) its NumPy decoders + BLAS, restated in oracle/.
    path "numpy": the reference's NumPy path for every format
    (PythonBackend.matmul_*, runtime/backend.py:164-213: dequantise to fp32,
    then a BLAS product), restated in oracle/.
    Returns (step, kind): kind "reference" when every call ran the
    reference's own compiled code, else "port"."""
    from oracle import gguf_oracle as O

    nat = _load_ref_native() if path == "native" else None
    calls, kinds = [], set()
    for (name, q, n, k, _), w, x in zip(mats, host_w, xs):
        if nat is not None and q in _REF_FN:
            fn = getattr(nat, _REF_FN[q] + ("_batched" if batch > 1 else ""))
            calls.append(lambda fn=fn, x=x, w=w, n=n, k=k: fn(x, w, n, k))
            kinds.add("reference")
        else:
            calls.append(lambda q=q, x=x, w=w, n=n, k=k: O.matvec_fp32(q, w, x, n, k))
            kinds.add("port")
    return (lambda: [c() for c in calls]), ("reference" if kinds == {"reference"} else "port")


def blas_threads() -> int:
    """Threads the BLAS library under NumPy runs with."""
    try:
        from threadpoolctl import threadpool_info
        n = [int(i.get("num_threads") or 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return max(n)
    except Exception:  # pragma: no cover - threadpoolctl absent
        pass
    return os.cpu_count() or 1


def cpu_leg(mats, batch, host_w, xs, path: str, steps: int, warmup: int, budget_s: float):
    """Time a reference CPU path on a bounded sample of the workload.

    Above CPU_SAMPLE_TOKENS tokens the passes use the first CPU_SAMPLE_TOKENS
    rows of x (the reference's batched kernels re-read the weight per token,
    so time scales linearly).  A 1 % row sample is timed once to size the
    sample: the largest row fraction whose warmup + steps passes fit in
    budget_s.  Returns (seconds per full-workload pass, as the median of
    `steps` sampled passes scaled by bytes and tokens; kind; description)."""
    tok_scale = 1.0
    if batch > CPU_SAMPLE_TOKENS:
        xs = [np.ascontiguousarray(x[:CPU_SAMPLE_TOKENS]) for x in xs]
        tok_scale = batch / CPU_SAMPLE_TOKENS
        batch = CPU_SAMPLE_TOKENS
    full_w = sum(synth.weight_bytes(q, n, k) for _, q, n, k, _ in mats)
    pm, pw = sample_rows(mats, host_w, 0.01)
    probe, _ = cpu_step_fn(pm, batch, pw, xs, path)
    t0 = time.perf_counter()
    probe()
    t_probe = max(time.perf_counter() - t0, 1e-6)
    probe_w = sum(synth.weight_bytes(q, n, k) for _, q, n, k, _ in pm)
    per_byte = t_probe / probe_w
    frac = min(1.0, budget_s / max(1, steps + warmup) / (per_byte * full_w))
    sm, sw = sample_rows(mats, host_w, frac)
    step, kind = cpu_step_fn(sm, batch, sw, xs, path)
    for _ in range(warmup):
        step()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    sample_w = sum(synth.weight_bytes(q, n, k) for _, q, n, k, _ in sm)
    t_full = statistics.median(times) * (full_w / sample_w) * tok_scale
    desc = (f"{steps} timed passes (median) after {warmup} warm-up over the first "
            f"{100.0 * sample_w / full_w:.3g} % of every projection's rows ({sample_w / 1e6:.1f} MB of weights), "
            f"scaled to the full workload by bytes")
    if tok_scale != 1.0:
        desc += f"; {CPU_SAMPLE_TOKENS} of the {int(batch * tok_scale)} tokens per pass, time scaled by {tok_scale:g}"
    return t_full, kind, desc


def cpu_baselines(mats, batch, host_w, xs, step_bytes: int, budget_s: float = 12.0) -> tuple[dict, dict]:
    """The reference's two CPU paths on the host cores: native C++ (1 core)
    and NumPy + BLAS (the BLAS library's threads), each on a bounded sample."""
    t_nat, kind, desc = cpu_leg(mats, batch, host_w, xs, "native", 3, 1, budget_s)
    native = {"value": round(step_bytes / t_nat / 1e9, 4), "unit": UNIT, "cores": 1, "kind": kind,
              "sample": desc + "; reference flatrun_native._C built from its sources (scalar, single-threaded "
                               "on x86: the x86 build has no threaded path)"}
    t_np, kind_np, desc_np = cpu_leg(mats, batch, host_w, xs, "numpy", 3, 1, budget_s)
    numpy_leg = {"value": round(step_bytes / t_np / 1e9, 4), "unit": UNIT, "cores": blas_threads(),
                 "kind": kind_np,
                 "sample": desc_np + "; the reference NumPy path (dequantise to fp32, then BLAS) restated in "
                                     "oracle/: NumPy decoding on one core, the BLAS product on the cores stated"}
    return native, numpy_leg


def config_of(wl: dict, mats, batch: int, world: int, scaling: str) -> dict:
    """The workload description both arms print (same keys and values)."""
    total = mats if scaling == "strong" or world == 1 else mats * world
    return {"workload": wl["desc"], "global_batch": (batch if batch <= 16 else 1),
            "seq_len": 1 if batch <= 16 else batch,
            "parallelism": f"row-shard x{world}" if world > 1 else "single GPU",
            "weight_bytes_per_step": sum(synth.weight_bytes(q, n, k) for _, q, n, k, _ in total),
            "algorithmic_bytes_per_step": algorithmic_bytes(mats, batch) * (world if scaling == "weak" else 1)}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def run_device_decode(args, wl: dict, config: dict, step_bytes: int) -> None:
    """The decode_qwen2_7b_device workload: K greedy tokens through
    flatrun_b200.decode.DecodeEngine (one CUDA graph replay per token) on a
    random-init Qwen2-7B in the Q4_K_M mix (centred Q4_K blocks, synthetic
    Q6_K blocks, fp32 embedding, norms 0.1, q/k/v biases) with a KV cache
    pre-filled with 4096 positions."""
    import ctypes

    import torch

    from flatrun_b200 import _lib
    from flatrun_b200.decode import DecodeEngine, DecoderConfig

    torch.cuda.set_device(0)
    H, F, V, L, NH, NKV, HD, PRE = 3584, 18944, 152064, 28, 28, 4, 128, 4096
    rng = np.random.default_rng(0)
    quant, w = {}, {}
    for i in range(L):
        p = f"model.layers.{i}"
        hi = "Q6_K" if i % 2 == 0 else "Q4_K"
        for j, (nm, n, k, q) in enumerate((("self_attn.q_proj", H, H, "Q4_K"), ("self_attn.k_proj", NKV * HD, H, "Q4_K"),
                                            ("self_attn.v_proj", NKV * HD, H, hi), ("self_attn.o_proj", H, H, "Q4_K"),
                                            ("mlp.gate_proj", F, H, "Q4_K"), ("mlp.up_proj", F, H, "Q4_K"),
                                            ("mlp.down_proj", H, F, hi))):
            name = f"{p}.{nm}.weight"
            quant[name] = (n, k, q)
            w[name] = synth.make_centered_q4_k(n, k, seed=100 * i + j) if q == "Q4_K" else \
                synth.make_weight(q, n, k, seed=100 * i + j)
        for nm in ("input_layernorm", "post_attention_layernorm"):
            w[f"{p}.{nm}.weight"] = np.full(H, 0.1, np.float32)
        for nm, n in (("q_proj", H), ("k_proj", NKV * HD), ("v_proj", NKV * HD)):
            w[f"{p}.self_attn.{nm}.bias"] = (rng.standard_normal(n) * 0.1).astype(np.float32)
    quant["lm_head.weight"] = (V, H, "Q6_K")
    w["lm_head.weight"] = synth.make_weight("Q6_K", V, H, seed=9999)
    w["model.norm.weight"] = np.full(H, 0.1, np.float32)
    w["model.embed_tokens.weight"] = rng.standard_normal((V, H), dtype=np.float32)
    kv = {i: (rng.standard_normal((PRE, NKV, HD), dtype=np.float32),
              rng.standard_normal((PRE, NKV, HD), dtype=np.float32)) for i in range(L)}
    K, W = args.steps, args.warmup
    e2e_steps = 0 if args.no_e2e else min(K, 200)
    cfg = DecoderConfig(hidden=H, ffn=F, vocab=V, layers=L, heads=NH, kv_heads=NKV, eps=1e-6, rope_theta=1e6,
                        max_pos=PRE + W + K + e2e_steps + 64)
    eng = DecodeEngine(cfg, w, quant.get, kv_prefill=kv)
    del w, kv
    eng.capture()
    st = eng.stream
    clocks = ClockSampler(0)
    eng.step(int(rng.integers(0, V)))
    for _ in range(W - 1):
        eng.step(None)
    st.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(st)
    for _ in range(K):
        eng.step(None)
    end.record(st)
    end.synchronize()
    clk = clocks.stop()
    ms_tok = start.elapsed_time(end) / K
    wbytes = config["weight_bytes_per_step"]
    value = step_bytes / (ms_tok / 1e3) / 1e9
    # the dominant launch: the lm_head GEMV (447 MB), timed alone K times
    lm = eng._w["lm_head.weight"]
    lib = eng.lib
    y = torch.empty(V, device="cuda")
    args_ = (lm[1], 1, (ctypes.c_void_p * 1)(lm[0].data_ptr()), (ctypes.c_size_t * 1)(lm[0].numel()),
             (ctypes.c_int64 * 1)(V), H, eng.h.data_ptr(), None, eng._norm["model.norm.weight"].data_ptr(), 1e-6, 0,
             (ctypes.c_void_p * 1)(y.data_ptr()), ctypes.c_void_p(st.cuda_stream))
    for _ in range(3):
        _lib.check(lib.frc_gemv_ex(*args_), lib)
    nl = min(K, 200)
    start.record(st)
    for _ in range(nl):
        _lib.check(lib.frc_gemv_ex(*args_), lib)
    end.record(st)
    end.synchronize()
    us = start.elapsed_time(end) * 1e3 / nl
    lm_bytes = synth.weight_bytes("Q6_K", V, H) + 4 * (H + V)
    peak, peak_src = peaks()
    achieved = lm_bytes / (us / 1e6) / 1e9
    # e2e through the engine's public calls: each token's greedy pick read
    # back to the host (a 4-byte copy and a synchronise per token)
    e2e = None
    if e2e_steps:
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            eng.step(None)
            eng.argmax_host()
        t_tok = (time.perf_counter() - t0) / e2e_steps
        e2e = {"value": round(step_bytes / t_tok / 1e9, 2), "unit": UNIT, "h2d_bytes_per_step": 0,
               "d2h_bytes_per_step": 4, "ms_per_step": round(t_tok * 1e3, 4), "tokens_per_s": round(1.0 / t_tok, 2),
               "timer": "host wall clock; each token: one graph replay, the argmax read back, a synchronise"}
    cpu = cpu_np = None
    if not args.no_cpu:
        mats = wl["mats"]
        host_w = make_host_layer(mats, 0)
        xs = [synth.make_x(k, seed=50 + i) for i, (_, _, _, k, _) in enumerate(mats)]
        cpu, cpu_np = cpu_baselines(mats, 1, host_w, xs, step_bytes)
        for leg in (cpu, cpu_np):
            leg["sample"] += "; the token's projections only (the reference's attention and norms not timed)"
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": 1, "steps": K, "warmup": W,
        "ms_per_step": round(ms_tok, 5), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic", "config": config,
        "tokens_per_s": round(1e3 / ms_tok, 2),
        "measurement": {"timer": "K graph replays (one token each) bracketed by CUDA events on the engine stream",
                        "weight_bytes_per_token": wbytes, "launches_per_token": eng.launches_per_token,
                        "l2": "inputs larger than L2: 4.37 GB of weights streamed per token"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": ncu_traffic("head_q6k"), "peak_source": peak_src,
                     "kernel": f"gemv_b1 (fp32 activations) <Q6_K> lm_head ({lm_bytes / 1e6:.1f} MB per launch)",
                     "timing": f"{nl} back-to-back launches bracketed by CUDA events on the engine stream"},
        "whole_token_frac": round(value / peak, 4),
        "cpu_baseline": cpu, "cpu_baseline_numpy": cpu_np, "e2e": e2e, "clocks": clk,
        "gpu_launches": K * eng.launches_per_token,
    }
    print(json.dumps(out), flush=True)
    eng.close()


def make_host_layer(mats, copy: int):
    return [synth.make_weight(q, n, k, seed=1000 * copy + i) for i, (_, q, n, k, _) in enumerate(mats)]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="layer_llama70b")
    ap.add_argument("--copies", type=int, default=0, help="distinct weight copies rotated (0 = auto, > 3x L2)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--nccl-gather", action="store_true",
                    help="N > 1: assemble row shards with NCCL all-gathers instead of the gather fused into the GEMV")
    ap.add_argument("--unfused", action="store_true",
                    help="one launch per projection, each with its own x (no shared-x fusion)")
    ap.add_argument("--batch1-int16", action="store_true",
                    help="batch 1 on the 16-bit activation grid kernel (dp4a) instead of fp32 activations")
    ap.add_argument("--cuda-core", action="store_true",
                    help="batch-1 Q4_K on the CUDA-core fp32 kernel instead of the tensor-core one (same arithmetic)")
    ap.add_argument("--tc-long-rows", action="store_true",
                    help="batch-1 Q4_K rows longer than one part of k on the tensor-core kernel too (FRC_OPT_BATCH1_TC=2)")
    ap.add_argument("--batched-fp32", action="store_true",
                    help="batch 2..16 on the fp32-activation CUDA-core kernel (gemv_xb) instead of the int8 tensor-core one")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    wl = WORKLOADS[args.workload]
    mats, batch = wl["mats"], wl["batch"]
    step_bytes = algorithmic_bytes(mats, batch, fused=not getattr(args, "unfused", False))

    scaling = "strong" if wl.get("strong") else "weak"
    config = config_of(wl, mats, batch, world, scaling)

    if args.impl == "reference":
        if rank != 0:
            return
        host_w = make_host_layer(mats, 0)
        xs = [synth.make_x(k, batch=None if batch == 1 else batch, seed=50 + i)
              for i, (_, _, _, k, _) in enumerate(mats)]
        # every one of the K timed and W warm-up steps runs; each step is a
        # row sample of the workload sized so that all of them take ~2 minutes
        t_full, kind, desc = cpu_leg(mats, batch, host_w, xs, "native", args.steps, args.warmup, budget_s=120.0)
        full_bytes = config["algorithmic_bytes_per_step"]
        value = full_bytes / t_full / 1e9
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t_full * 1e3, 3),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
            "dtype": "f32", "data": "synthetic", "config": config,
            "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": 1, "kind": kind,
                             "sample": desc + "; reference flatrun_native._C built from its sources (scalar, "
                                              "single-threaded on x86: the x86 build has no threaded path)"},
            "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "tokens_per_s": round(1.0 / t_full, 4) if args.workload.startswith("decode") else None,
        }), flush=True)
        return

    if wl.get("device_decode"):
        if world > 1:
            raise SystemExit("the device decode workload runs on one GPU")
        run_device_decode(args, wl, config, step_bytes)
        return

    import ctypes

    import torch

    from flatrun_b200 import CudaBackend, _lib

    # strong scaling: the workload is one whole layer, each rank owns n / N
    # rows of every projection (whole quant blocks per row)
    if wl.get("strong") and world > 1:
        mats = shard_rows(mats, world)
        step_bytes = algorithmic_bytes(mats, batch, fused=not getattr(args, "unfused", False))

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
    if args.batched_fp32:
        _lib.set_option("batched_fp32", 1)
    if args.cuda_core:
        _lib.set_option("batch1_tc", 0)
    elif args.tc_long_rows:
        _lib.set_option("batch1_tc", 2)
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
    sig_bytes = {}  # weight bytes of all matrices of one shape (timed together per launch)
    for _, q, n, k, _ in mats:
        sig_bytes[(q, n, k)] = sig_bytes.get((q, n, k), 0) + synth.weight_bytes(q, n, k)
    for (name, q, n, k, _), raw in zip(mats, base):
        nb = max(int(raw.nbytes), 1)
        stride = (nb + 255) // 256 * 256
        # the launches of one shape, timed back to back, stream >= 3x L2 of
        # distinct weights: they re-read nothing from L2 (nor does a step)
        nc = 1 if sig_bytes[(q, n, k)] >= 3 * l2 else int(min(1024, max(2, np.ceil(3 * l2 / nb))))
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
    launch_us = {}  # per launch group: its plain GEMV time (no assembly)
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
        for g_ in gs:
            launch_us[tuple(g_)] = us
        del gi
    gemv_us_step = sum(launch_us[tuple(g)] for g in lgroups)
    if world > 1:
        t = torch.tensor([gemv_us_step], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        gemv_us_step = float(t.item())
    # the share of the step that the output assembly (stores to peers, the
    # flag publication and waits, the skew between ranks) adds to the GEMVs
    assembly_share = max(0.0, 1.0 - gemv_us_step / (ms_step * 1e3)) if world > 1 else None

    # in-run correctness of the assembly (N > 1, every rank): one more step
    # run eagerly; each fused group's gathered buffer must equal, bit for bit,
    # the NCCL all-gather of the ranks' own outputs, and each rank's own
    # outputs must equal a plain per-matrix GEMV of its rows
    gather_check = None
    if world > 1 and fused:
        with torch.cuda.stream(stream):
            launch(K)
            for fg, _ in fused.values():
                fg.wait(stream.cuda_stream)
        stream.synchronize()
        ok = True
        for idx, (fg, sendbuf) in fused.items():
            ref = torch.empty(world * sendbuf.numel(), device="cuda")
            dist.all_gather_into_tensor(ref, sendbuf)
            ok = ok and torch.equal(fg.gathered(), ref)
            local = sendbuf.clone()
            with torch.cuda.stream(stream):
                for i in idx:
                    gemv(i, K)
            stream.synchronize()
            ok = ok and torch.equal(local, sendbuf)
        t = torch.tensor([0 if ok else 1], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        gather_check = "bit-exact on every rank" if int(t.item()) == 0 else "MISMATCH"
    # dominant kernel: the launch carrying the most bytes
    dom_name = max(per, key=lambda nm: per[nm]["bytes"])
    achieved = per[dom_name]["bytes"] / (per[dom_name]["us"] / 1e6) / 1e9
    peak, peak_src = peaks()
    traffic = ncu_traffic(args.workload)

    # e2e through the public call, host buffers (pinned x), synchronous calls;
    # under --gpus N every rank runs its own shard's calls (the same number
    # of steps on every rank) and the slowest rank's time counts
    e2e = None
    if not args.no_e2e:
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
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for s in range(e2e_steps):
            for i, (_, q, n, k, _) in enumerate(mats):
                method[q](pinned[i], host_arrays[s % copies][i], n, k)
        t_e2e = (time.perf_counter() - t0) / e2e_steps
        if world > 1:
            t = torch.tensor([t_e2e], dtype=torch.float64, device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_e2e = float(t.item())
        e2e = {"value": round(step_bytes * world / t_e2e / 1e9, 2), "unit": UNIT,
               "h2d_bytes_per_step": world * sum(batch * k * 4 for _, _, _, k, _ in mats),
               "d2h_bytes_per_step": world * sum(batch * n * 4 for _, _, n, _, _ in mats),
               "ms_per_step": round(t_e2e * 1e3, 4), "steps": e2e_steps,
               "tokens_per_s": round(1.0 / t_e2e, 2) if args.workload.startswith("decode") else None,
               "timer": ("host wall clock over synchronous calls (each call copies x in, y out and synchronises)"
                         + ("; each rank its own row shard, the slowest rank's time; y shards stay on their ranks"
                            if world > 1 else ""))}

    # CPU baselines (rank 0 at N = 1 only): the reference's native C++ path
    # and its NumPy path, each on a bounded sample of the same workload
    cpu = cpu_np = None
    if not args.no_cpu and world == 1:
        cpu, cpu_np = cpu_baselines(mats, batch, base, xs_host, step_bytes)

    if rank == 0:
        # the kernel family each call runs: batch 1 dp4a GEMV, 2..16 int8
        # tensor-core GEMV (pre-pass + main), more: tcgen05 GEMM (fp16 pre-pass
        # + main)
        if batch == 1:
            dom_q, dom_k = next((mats[i][1], mats[i][3]) for g in lgroups for i in g
                                if dom_name.startswith("+".join(mats[j][0] for j in g)))
            if _lib.batch1_kernel(dom_q, dom_k) == "tensor_fp32":
                kname = ("gemv_tc1 (fp32 activations: x as three exact fp16 terms, weights as exact fp16 "
                         "q*sc, products on the tensor cores (mma.sync), fp32 accumulation)")
            else:
                kname = "gemv_b1 (fp32 activations, fp32 FMAs)"
            dtype, calls_per_group = "f32", lambda g: 1
        elif batch <= 16 and args.batched_fp32:
            kname, dtype, calls_per_group = "gemv_xb (fp32 activations, fp32 FMAs)", "f32", lambda g: len(g)
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
            "config": config,
            "measurement": {
                "gather": ("fused into the GEMV: stores to every rank over NVLink; the next GEMV waits for every "
                           "rank's flag before reading x" if fused else "NCCL all_gather_into_tensor")
                          if world > 1 else None,
                "rank_bytes_per_step": step_bytes,
                "weight_copies_rotated": [p[2] for p in pools],
                "l2": f"inputs larger than L2: each projection rotates over distinct device copies totalling "
                      f">= 3x L2 ({sum(p[2] * mbytes[i] for i, p in enumerate(pools)) / 1e9:.2f} GB); "
                      f"L2 {l2 / 2**20:.0f} MiB"},
            "frac_of_8tbs": round(value / world / 8000.0, 4),
            "tokens_per_s": round(1e3 / ms_step, 2) if args.workload.startswith("decode") else None,
            "roofline": roof,
            "per_launch": per,
            "launches_per_step": len(lgroups),
            "assembly_share": round(assembly_share, 4) if assembly_share is not None else None,
            "gemv_us_per_step": round(gemv_us_step, 3),
            "gather_check": gather_check,
            "cpu_baseline": cpu,
            "cpu_baseline_numpy": cpu_np,
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
