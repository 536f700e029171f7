"""Generate the greedy-decode golden files: a random-init Qwen2 model
(``tests/qwen2_restated.py``) decoded greedily by the reference itself.

    python tests/golden/make_decode_golden.py [--model tiny|qwen2-7b] [--ref <reference checkout>]

The unchanged reference forwarder (``flatrun.model.qwen2.make_qwen2_forwarder``
with the ``python`` backend: dequantise to fp32, then ``x @ W.T``) prefills
the prompt and decodes greedily through its KV cache
(``flatrun.runtime.kv_cache.KVCache``), layer by layer as its scheduler does
(``LayerHandles`` with ``is_first`` / ``is_last``), as in the reference's
incremental-decode test (``src/flatrun/tests/test_qwen2.py:241-263``).

* ``tiny`` -> ``decode_tiny_qwen2.npz``: an 8-token prompt, 12 greedy
  tokens and the last-position logits after the prompt and after each token
  (13 x 320 fp32).
* ``qwen2-7b`` -> ``decode_qwen2_7b.npz`` (config 4): the KV cache is first
  filled with the model's 4096 pre-filled positions per layer, then a
  32-token prompt of uniform random ids and 64 greedy tokens.  The full
  logits (65 x 152064) are too large to commit, so each step keeps its top
  16 (ids and values), the values at 1024 fixed random vocabulary ids and
  max |logit|; plus the hidden states after layers 0 and 1 for the prompt
  (pins a two-layer CPU run of the restatement).  The weights are not
  stored: they are regenerated from their seeds.  Needs ~45 GB of RAM and
  ~10 minutes (the reference dequantises every weight to fp32 once).
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.dirname(HERE))

import qwen2_restated as Q  # noqa: E402

RUNS = {
    # spec, prompt length, greedy steps, prompt seed, output file
    "tiny": (Q.TINY, 8, 12, 11, "decode_tiny_qwen2.npz"),
    "qwen2-7b": (Q.QWEN2_7B, 32, 64, 23, "decode_qwen2_7b.npz"),
}
TOPK, NSAMPLE, SAMPLE_SEED = 16, 1024, 29


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", choices=sorted(RUNS), default="tiny")
    ap.add_argument("--ref", default=os.environ.get("FLATRUN_REFERENCE") or os.path.join(os.path.dirname(REPO), "reference"))
    a = ap.parse_args()
    spec, plen, steps, pseed, fname = RUNS[a.model]
    sys.path.insert(0, os.path.join(a.ref, "src"))
    from flatrun.core.tensor import BufferTensorHandle
    from flatrun.model.qwen2 import Qwen2Config, make_qwen2_forwarder
    from flatrun.runtime import backend as rb
    from flatrun.runtime.kv_cache import KVCache
    from flatrun.runtime.scheduler import LayerHandles
    from flatrun.utils.types import LayerDescriptor, TensorKey, TensorMetadata

    cfg = Qwen2Config(hidden_size=spec.H, intermediate_size=spec.F, num_hidden_layers=spec.L,
                      num_attention_heads=spec.NH, num_key_value_heads=spec.NKV, vocab_size=spec.V,
                      rms_norm_eps=spec.EPS, rope_theta=spec.THETA, max_position_embeddings=spec.MAX_POS,
                      tie_word_embeddings=False, model_arch="qwen2")
    w = Q.build(spec)
    handles = {}
    for name in list(w):
        arr = w.pop(name)
        q = Q.quant_of(spec, name)
        if q is None:
            meta = TensorMetadata(key=TensorKey(file=spec.name, name=name, backend=""), shape=tuple(arr.shape),
                                  dtype="float32", byte_size=arr.nbytes, offset=0)
        else:
            n, k, quant = q
            meta = TensorMetadata(key=TensorKey(file=spec.name, name=name, backend="gguf"), shape=(n, k),
                                  dtype="uint8", byte_size=int(arr.nbytes), offset=0, quantization=quant)
        handles[name] = BufferTensorHandle(meta, arr.tobytes())
        del arr
    names_l = ("input_layernorm", "self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
               "post_attention_layernorm", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")

    fwd = make_qwen2_forwarder(cfg, enable_dequant_cache=spec.kv_prefill > 0, backend=rb.get_backend("python"))
    kv = KVCache(capacity=max(64, 2 * (spec.kv_prefill + plen + steps)))
    for i in range(spec.L if spec.kv_prefill else 0):
        kp, vp = Q.kv_prefill(spec, i)
        for t in range(spec.kv_prefill):
            kv.append(i, kp[t], vp[t])
    hidden_after = {}

    def run(toks, record=False):
        out = None
        for i in range(spec.L):
            names = tuple(f"model.layers.{i}.{n}.weight" for n in names_l)
            names += tuple(f"model.layers.{i}.self_attn.{p}.bias" for p in ("q_proj", "k_proj", "v_proj")
                           if f"model.layers.{i}.self_attn.{p}.bias" in handles)
            if i == 0:
                names = ("model.embed_tokens.weight",) + names
            if i == spec.L - 1:
                names = names + ("model.norm.weight", "lm_head.weight")
            lh = LayerHandles({n: handles[n] for n in names}, names)
            lh.is_first, lh.is_last, lh.tokens, lh.layer_index = i == 0, i == spec.L - 1, list(toks), i
            out = fwd(LayerDescriptor(index=i, tensor_names=names), lh, kv)
            if record and i < 2:
                hidden_after[i] = np.array(out, np.float32, copy=True)
        return np.asarray(out, np.float32)

    prompt = np.random.default_rng(pseed).integers(0, spec.V, size=plen)
    logits = [run(prompt.tolist(), record=True)[-1]]
    tokens = []
    for s in range(steps):
        t = int(np.argmax(logits[-1]))
        tokens.append(t)
        logits.append(run([t])[-1])
        print("step", s, "token", t, flush=True)
    lg = np.stack(logits).astype(np.float32)
    out = os.path.join(HERE, fname)
    if spec.name == "tiny":
        np.savez_compressed(out, prompt=prompt.astype(np.int64), tokens=np.asarray(tokens, np.int64), logits=lg)
    else:
        top = np.argsort(-lg, axis=1)[:, :TOPK]
        sample = np.sort(np.random.default_rng(SAMPLE_SEED).choice(spec.V, NSAMPLE, replace=False))
        np.savez_compressed(out, prompt=prompt.astype(np.int64), tokens=np.asarray(tokens, np.int64),
                            top_ids=top.astype(np.int64), top_vals=np.take_along_axis(lg, top, axis=1),
                            sample_ids=sample.astype(np.int64), sample_vals=lg[:, sample],
                            max_abs=np.max(np.abs(lg), axis=1), hidden_l0=hidden_after[0], hidden_l1=hidden_after[1])
    print(out, "tokens", tokens)


if __name__ == "__main__":
    main()
