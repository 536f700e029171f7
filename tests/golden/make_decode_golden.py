"""Generate ``decode_tiny_qwen2.npz``: a greedy decode of the tiny random-init
Qwen2 model (``tests/tiny_qwen2.py``) run by the reference itself.

    python tests/golden/make_decode_golden.py --ref <reference checkout>

The unchanged reference forwarder (``flatrun.model.qwen2.make_qwen2_forwarder``
with the ``python`` backend: dequantise to fp32, then ``x @ W.T``) prefills an
8-token prompt and decodes 12 tokens greedily through its KV cache
(``flatrun.runtime.kv_cache.KVCache``), layer by layer as its scheduler does
(``LayerHandles`` with ``is_first`` / ``is_last``).  Stored: the prompt, the
12 greedy tokens, and the last-position logits after the prompt and after
each token (13 x 320 fp32).
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

import tiny_qwen2 as T  # noqa: E402

PROMPT_LEN, STEPS, PROMPT_SEED = 8, 12, 11


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("FLATRUN_REFERENCE") or os.path.join(os.path.dirname(REPO), "reference"))
    a = ap.parse_args()
    sys.path.insert(0, os.path.join(a.ref, "src"))
    from flatrun.core.tensor import BufferTensorHandle
    from flatrun.model.qwen2 import Qwen2Config, make_qwen2_forwarder
    from flatrun.runtime import backend as rb
    from flatrun.runtime.kv_cache import KVCache
    from flatrun.runtime.scheduler import LayerHandles
    from flatrun.utils.types import LayerDescriptor, TensorKey, TensorMetadata

    cfg = Qwen2Config(hidden_size=T.H, intermediate_size=T.F, num_hidden_layers=T.L, num_attention_heads=T.NH,
                      num_key_value_heads=T.NKV, vocab_size=T.V, rms_norm_eps=T.EPS, rope_theta=T.THETA,
                      max_position_embeddings=T.MAX_POS, tie_word_embeddings=False, model_arch="qwen2")
    w = T.build()
    handles = {}
    for name, arr in w.items():
        spec = T.quant_of(name)
        if spec is None:
            meta = TensorMetadata(key=TensorKey(file="tiny", name=name, backend=""), shape=tuple(arr.shape),
                                  dtype="float32", byte_size=arr.nbytes, offset=0)
        else:
            n, k, q = spec
            meta = TensorMetadata(key=TensorKey(file="tiny", name=name, backend="gguf"), shape=(n, k),
                                  dtype="uint8", byte_size=int(arr.nbytes), offset=0, quantization=q)
        handles[name] = BufferTensorHandle(meta, arr.tobytes())
    names_l = ("input_layernorm", "self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
               "post_attention_layernorm", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")

    fwd = make_qwen2_forwarder(cfg, enable_dequant_cache=False, backend=rb.get_backend("python"))
    kv = KVCache(capacity=64)

    def run(toks):
        out = None
        for i in range(T.L):
            names = tuple(f"model.layers.{i}.{n}.weight" for n in names_l)
            if i == 0:
                names = ("model.embed_tokens.weight",) + names
            if i == T.L - 1:
                names = names + ("model.norm.weight", "lm_head.weight")
            lh = LayerHandles({n: handles[n] for n in names}, names)
            lh.is_first, lh.is_last, lh.tokens, lh.layer_index = i == 0, i == T.L - 1, list(toks), i
            out = fwd(LayerDescriptor(index=i, tensor_names=names), lh, kv)
        return np.asarray(out, np.float32)

    prompt = np.random.default_rng(PROMPT_SEED).integers(0, T.V, size=PROMPT_LEN)
    logits = [run(prompt.tolist())[-1]]
    tokens = []
    for _ in range(STEPS):
        t = int(np.argmax(logits[-1]))
        tokens.append(t)
        logits.append(run([t])[-1])
    out = os.path.join(HERE, "decode_tiny_qwen2.npz")
    np.savez_compressed(out, prompt=prompt.astype(np.int64), tokens=np.asarray(tokens, np.int64),
                        logits=np.stack(logits).astype(np.float32))
    print(out, "tokens", tokens)


if __name__ == "__main__":
    main()
