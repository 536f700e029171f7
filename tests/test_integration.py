"""Registration in the reference's backend slot (CPU; skipped when the
reference source tree is not importable, e.g. on the GPU box).

The forwarder routing is exercised with the real reference forwarder on a
tiny in-memory model: a planted checker replaces the C-ABI call so the test
sees which projections reach the backend and with what arguments (the numbers
themselves are checked on the GPU by test_gpu_parity)."""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# the reference checkout: FLATRUN_REFERENCE, else "reference" beside this repository
REF = os.environ.get("FLATRUN_REFERENCE") or os.path.join(os.path.dirname(REPO), "reference")
REF_SRC = os.path.join(REF, "src")


@pytest.fixture(scope="module")
def rb():
    if not os.path.isdir(os.path.join(REF_SRC, "flatrun")):
        pytest.skip("reference source tree not available")
    if REF_SRC not in sys.path:
        sys.path.insert(0, REF_SRC)
    from flatrun.runtime import backend
    return backend


def test_register_adds_cuda_backends(rb):
    from flatrun_b200 import integration
    slot, adapter = integration.register(rb)
    b = rb.get_backend("cuda")
    assert isinstance(b, slot) and b.name == "cuda"
    a = rb.get_backend("native-cuda")
    assert isinstance(a, adapter) and a.name == "native"
    assert isinstance(b, rb.BackendBase)
    # get_backend is case-insensitive in the reference (backend.py:309)
    assert isinstance(rb.get_backend("CUDA"), slot)


def test_no_gpu_means_unavailable_and_raises(rb):
    from flatrun_b200 import integration
    integration.register(rb)
    b = rb.get_backend("cuda")
    if b.available:
        pytest.skip("a GPU is present")
    assert b.supported_quants == set()
    with pytest.raises(RuntimeError):
        b.matmul_q4k(np.zeros(256, np.float32), np.zeros(144, np.uint8), 1, 256)


def test_dispatch_routes_by_quant_tag(rb):
    from flatrun_b200 import integration
    slot, _ = integration.register(rb)
    b = slot()
    calls = []
    for m in ("matmul_q4k", "matmul_q6k", "matmul_q8_0", "matmul_q5k", "matmul_q1_0"):
        setattr(b._cuda, m, (lambda name: lambda x, w, n, k: calls.append(name) or np.zeros(n, np.float32))(m))
    for tag in ("Q4_K", "Q6_K", "Q8_0", "Q5_K", "Q1_0"):
        b.dispatch(np.zeros(4, np.float32), None, 2, 4, tag)
    assert calls == ["matmul_q4k", "matmul_q6k", "matmul_q8_0", "matmul_q5k", "matmul_q1_0"]
    w = np.eye(3, dtype=np.float32)
    np.testing.assert_array_equal(b.dispatch(np.ones(3, np.float32), w, 3, 3, None), np.ones(3))


def test_forwarder_method_table_extension(rb):
    from flatrun.model import qwen2
    from flatrun_b200 import integration
    before = dict(qwen2._NATIVE_METHOD)
    try:
        integration.extend_forwarder_method_table(qwen2)
        assert qwen2._NATIVE_METHOD["Q5_K"] == "matmul_q5k"
        assert qwen2._NATIVE_METHOD["Q1_0"] == "matmul_q1_0"
        assert qwen2._NATIVE_METHOD["Q4_K"] == before["Q4_K"]
    finally:
        qwen2._NATIVE_METHOD.clear()
        qwen2._NATIVE_METHOD.update(before)


# ---- the unchanged reference forwarder routed through the adapter -----------

def _handle(name, shape, raw, quant, rb_types):
    TensorMetadata, TensorKey, BufferTensorHandle = rb_types
    if quant is None:
        arr = np.ascontiguousarray(raw, dtype=np.float32)
        meta = TensorMetadata(key=TensorKey(file="syn", name=name, backend=""), shape=tuple(arr.shape),
                              dtype="float32", byte_size=arr.nbytes, offset=0)
        return BufferTensorHandle(meta, arr.tobytes())
    meta = TensorMetadata(key=TensorKey(file="syn", name=name, backend="gguf"), shape=tuple(shape), dtype="uint8",
                          byte_size=int(raw.nbytes), offset=0, quantization=quant)
    return BufferTensorHandle(meta, raw.tobytes())


def test_reference_forwarder_routes_projections_to_adapter(rb):
    """Layers with all-Q4_K/Q6_K projections and a Q6_K head go through the
    adapter's matmul_* (the GPU compute is replaced by the oracle here, on
    CPU); logits equal the reference python backend's within 1e-3."""
    from flatrun.core.tensor import BufferTensorHandle
    from flatrun.model.qwen2 import Qwen2Config, make_qwen2_forwarder
    from flatrun.runtime.kv_cache import KVCache
    from flatrun.runtime.scheduler import LayerHandles
    from flatrun.utils.types import LayerDescriptor, TensorKey, TensorMetadata

    from flatrun_b200 import integration, synth
    from oracle import gguf_oracle as O

    types = (TensorMetadata, TensorKey, BufferTensorHandle)
    H, F, V, L, NH, NKV = 256, 512, 320, 2, 4, 2
    KVD = NKV * (H // NH)
    cfg = Qwen2Config(hidden_size=H, intermediate_size=F, num_hidden_layers=L, num_attention_heads=NH,
                      num_key_value_heads=NKV, vocab_size=V, rms_norm_eps=1e-6, rope_theta=1e6,
                      max_position_embeddings=256, tie_word_embeddings=False, model_arch="qwen2")
    rng = np.random.default_rng(5)

    def build():
        h = {}
        h["model.embed_tokens.weight"] = _handle("e", None, rng.standard_normal((V, H)).astype(np.float32), None, types)
        h["model.norm.weight"] = _handle("n", None, np.ones(H, np.float32), None, types)
        h["lm_head.weight"] = _handle("lm", (V, H), synth.make_weight("Q6_K", V, H, seed=1), "Q6_K", types)
        for i in range(L):
            p = f"model.layers.{i}"
            h[f"{p}.input_layernorm.weight"] = _handle("a", None, np.ones(H, np.float32), None, types)
            h[f"{p}.post_attention_layernorm.weight"] = _handle("b", None, np.ones(H, np.float32), None, types)
            for nm, (n, k, q) in {"self_attn.q_proj": (H, H, "Q4_K"), "self_attn.k_proj": (KVD, H, "Q4_K"),
                                  "self_attn.v_proj": (KVD, H, "Q6_K"), "self_attn.o_proj": (H, H, "Q4_K"),
                                  "mlp.gate_proj": (F, H, "Q4_K"), "mlp.up_proj": (F, H, "Q4_K"),
                                  "mlp.down_proj": (H, F, "Q6_K")}.items():
                h[f"{p}.{nm}.weight"] = _handle(nm, (n, k), synth.make_weight(q, n, k, seed=10 * i + len(nm)), q,
                                                types)
        return h

    handles = build()
    names_l = ("input_layernorm", "self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
               "post_attention_layernorm", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")
    tokens = rng.integers(0, V, size=6).tolist()

    def drive(fwd, kv, toks):
        out = None
        for i in range(L):
            names = tuple(f"model.layers.{i}.{n}.weight" for n in names_l)
            if i == 0:
                names = ("model.embed_tokens.weight",) + names
            if i == L - 1:
                names = names + ("model.norm.weight", "lm_head.weight")
            lh = LayerHandles({n: handles[n] for n in names}, names)
            lh.is_first, lh.is_last, lh.tokens, lh.layer_index = i == 0, i == L - 1, list(toks), i
            out = fwd(LayerDescriptor(index=i, tensor_names=names), lh, kv)
        return out

    ref = make_qwen2_forwarder(cfg, enable_dequant_cache=False, backend=rb.get_backend("python"))
    kv = KVCache(capacity=64)
    y_ref = drive(ref, kv, tokens)
    y_ref2 = drive(ref, kv, tokens[-1:])

    _, adapter = integration.register(rb)
    a = adapter()
    calls = []

    class Checker:
        """Stands in for the GPU on this CPU-only test: records each call and
        answers with the oracle."""
        available = True
        supported_quants = {"Q4_K", "Q6_K"}

    for meth, q in (("matmul_q4k", "Q4_K"), ("matmul_q6k", "Q6_K")):
        def checker(x, w, n, k, q=q, meth=meth):
            calls.append((meth, np.asarray(x).shape, n, k))
            return O.matvec_fp32(q, np.asarray(w).view(np.uint8).reshape(-1), np.asarray(x, np.float32), n, k)
        setattr(Checker, meth, staticmethod(checker))
    a._cuda = Checker()
    fwd = make_qwen2_forwarder(cfg, enable_dequant_cache=False, backend=a)
    kv2 = KVCache(capacity=64)
    y = drive(fwd, kv2, tokens)
    y2 = drive(fwd, kv2, tokens[-1:])
    assert O.rel_err(y, y_ref) < 1e-3 and O.rel_err(y2, y_ref2) < 1e-3
    seen = {(m, n, k) for m, _, n, k in calls}
    assert ("matmul_q4k", H, H) in seen and ("matmul_q4k", F, H) in seen and ("matmul_q6k", H, F) in seen
    assert ("matmul_q6k", V, H) in seen  # LM head
    assert ("matmul_q6k", KVD, H) in seen and ("matmul_q4k", KVD, H) in seen
    # prefill calls carry the whole (seq, k) activation, decode calls one row
    assert any(shape == (6, H) for _, shape, _, _ in calls) and any(shape == (1, H) for _, shape, _, _ in calls)


def test_cli_launcher_accepts_backend_cuda(rb):
    """`python -m flatrun_b200.cli run ... --backend cuda` reaches the
    reference CLI with the choice accepted (its --help lists it), and
    get_backend("cuda") then builds the adapter the forwarder dispatches to."""
    import subprocess

    env = dict(os.environ, PYTHONPATH=os.pathsep.join([REF_SRC, REPO, os.environ.get("PYTHONPATH", "")]))
    for sub in ("run", "chat", "serve"):
        r = subprocess.run([sys.executable, "-m", "flatrun_b200.cli", sub, "--help"], capture_output=True, text=True,
                           env=env, timeout=120)
        assert r.returncode == 0, r.stderr[-1000:]
        assert "cuda" in r.stdout.split("--backend", 1)[1][:80]
    from flatrun_b200 import cli, integration
    adapter = cli.install(rb)
    b = rb.get_backend("cuda")
    assert isinstance(b, adapter) and b.name == "native"
    integration.register(rb)  # restore the plain registry entry for the other tests


def test_cli_choice_patch_is_scoped():
    import argparse

    from flatrun_b200.cli import backend_choice_added
    with backend_choice_added("cuda"):
        p = argparse.ArgumentParser()
        p.add_argument("--backend", choices=["python", "native"])
        assert p.parse_args(["--backend", "cuda"]).backend == "cuda"
    p = argparse.ArgumentParser()
    p.add_argument("--backend", choices=["python", "native"])
    with pytest.raises(SystemExit):
        p.parse_args(["--backend", "cuda"])
