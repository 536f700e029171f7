"""Random-init Qwen2 decoders and a NumPy restatement of the reference's
forward pass, for greedy-decode parity tests (test infrastructure only).

Two models share one restated forward:

* ``TINY``: the Qwen2-7B layout at toy size (2 layers, hidden 256, FFN 512,
  4 query / 2 KV heads of 64, vocab 320) in the config-4 quant mix: Q4_K
  q/k/o/gate/up, Q6_K v/down and a Q6_K lm_head; norms are ones, the
  embedding table is fp32, no biases, an empty KV cache.
* ``QWEN2_7B``: config 4 of the benchmark: 28 layers, hidden 3584, 28 query /
  4 KV heads of 128, FFN 18944, vocab 152064, RMSNorm eps 1e-6, RoPE theta
  1e6, q/k/v biases, the Q4_K_M mix (Q4_K everywhere except v and down in
  the even layers, Q6_K, and the Q6_K lm_head), and a KV cache pre-filled
  with 4096 positions of N(0, 1) keys and values.  Q6_K blocks follow the
  benchmark's synthetic distribution (``flatrun_b200.synth``, zero-mean
  weights); Q4_K blocks are centred (``synth.make_centered_q4_k``); norm weights 0.1,
  biases N(0, 0.1^2), embedding rows N(0, 1), so activations stay O(1).  Every tensor is generated from its own seed, so a
  test can build any subset (one layer, a few embedding rows) without the
  rest, and the golden generator (which runs the reference forwarder) and
  the tests see identical bytes.

`forward()` restates `flatrun.model.qwen2.make_qwen2_forwarder` for this
architecture (no q/k norms, rotate-half RoPE, full causal attention over the
cached positions, untied head):
  embedding lookup                     qwen2.py:2153-2159
  RMSNorm in fp32                      qwen2.py:365-378
  RoPE tables, rotate-half layout      qwen2.py:398-476
  q/k/v (+ bias), RoPE at absolute
  positions, KV append, GQA repeat,
  scaled scores + causal mask,
  softmax, AV                          qwen2.py:1510-1625, :480-509
  o_proj + residual                    qwen2.py:1617-1646
  RMSNorm, gate/up, silu(gate) * up,
  down + residual                      qwen2.py:1648-1750
  final RMSNorm + lm_head (all rows)   qwen2.py:2238-2290
Projections go through `backend.matmul_q4k / matmul_q6k(x, raw, n, k)` with
x of shape (seq, k), the reference's native method signature.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from flatrun_b200 import synth


@dataclass(frozen=True)
class Spec:
    name: str
    H: int      # hidden size
    F: int      # FFN size
    V: int      # vocabulary
    L: int      # layers
    NH: int     # query heads
    NKV: int    # key/value heads
    EPS: float
    THETA: float
    MAX_POS: int
    bias: bool       # q/k/v biases
    kv_prefill: int  # cached positions before the prompt
    seed: int

    @property
    def HD(self) -> int:
        return self.H // self.NH

    @property
    def KVD(self) -> int:
        return self.NKV * self.HD

    def proj(self, layer: int) -> dict:
        """projection -> (rows n, columns k, quant) of one layer."""
        hi = "Q6_K" if (self.name == "tiny" or layer % 2 == 0) else "Q4_K"
        return {
            "self_attn.q_proj": (self.H, self.H, "Q4_K"),
            "self_attn.k_proj": (self.KVD, self.H, "Q4_K"),
            "self_attn.v_proj": (self.KVD, self.H, hi),
            "self_attn.o_proj": (self.H, self.H, "Q4_K"),
            "mlp.gate_proj": (self.F, self.H, "Q4_K"),
            "mlp.up_proj": (self.F, self.H, "Q4_K"),
            "mlp.down_proj": (self.H, self.F, hi),
        }

    @property
    def head(self) -> tuple[int, int, str]:
        return (self.V, self.H, "Q6_K")


TINY = Spec("tiny", H=256, F=512, V=320, L=2, NH=4, NKV=2, EPS=1e-6, THETA=1e6, MAX_POS=256, bias=False,
            kv_prefill=0, seed=5)
QWEN2_7B = Spec("qwen2-7b", H=3584, F=18944, V=152064, L=28, NH=28, NKV=4, EPS=1e-6, THETA=1e6, MAX_POS=32768,
                bias=True, kv_prefill=4096, seed=17)

NORM_WEIGHT = 0.1  # QWEN2_7B RMSNorm gains
BIAS_STD = 0.1


def _weight(spec: Spec, q: str, n: int, k: int, seed: int) -> np.ndarray:
    if spec.name != "tiny" and q == "Q4_K":
        return synth.make_centered_q4_k(n, k, seed)
    return synth.make_weight(q, n, k, seed=seed)


def quant_of(spec: Spec, name: str) -> tuple[int, int, str] | None:
    """(n, k, quant) of a quantised tensor name, None for fp32 tensors."""
    if name == "lm_head.weight":
        return spec.head
    if name.startswith("model.layers.") and name.endswith(".weight"):
        layer = int(name.split(".")[2])
        for proj, s in spec.proj(layer).items():
            if name.endswith(f".{proj}.weight"):
                return s
    return None


def _proj_seed(spec: Spec, layer: int, j: int) -> int:
    return spec.seed * 1000 + 10 * layer + j


def layer_tensors(spec: Spec, layer: int) -> dict:
    """Every tensor of one decoder layer by name."""
    p = f"model.layers.{layer}"
    norm = np.ones(spec.H, np.float32) if spec.name == "tiny" else np.full(spec.H, NORM_WEIGHT, np.float32)
    w = {f"{p}.input_layernorm.weight": norm, f"{p}.post_attention_layernorm.weight": norm.copy()}
    for j, (name, (n, k, q)) in enumerate(spec.proj(layer).items()):
        w[f"{p}.{name}.weight"] = _weight(spec, q, n, k, _proj_seed(spec, layer, j))
    if spec.bias:
        rng = np.random.default_rng([spec.seed, 3, layer])
        for name, n in (("q_proj", spec.H), ("k_proj", spec.KVD), ("v_proj", spec.KVD)):
            w[f"{p}.self_attn.{name}.bias"] = (rng.standard_normal(n) * BIAS_STD).astype(np.float32)
    return w


def embedding_rows(spec: Spec, ids) -> np.ndarray:
    """Rows `ids` of the fp32 embedding table (QWEN2_7B: row r from its own
    seed, so any subset is cheap to build)."""
    ids = np.asarray(ids, np.int64)
    if spec.name == "tiny":
        return build(spec)["model.embed_tokens.weight"][ids]
    return np.stack([np.random.default_rng([spec.seed, 1, int(r)]).standard_normal(spec.H).astype(np.float32)
                     for r in ids]) if ids.size else np.zeros((0, spec.H), np.float32)


def kv_prefill(spec: Spec, layer: int) -> tuple[np.ndarray, np.ndarray]:
    """The pre-filled cache of one layer: (kv_prefill, NKV, HD) keys and values ~ N(0, 1)."""
    rng = np.random.default_rng([spec.seed, 2, layer])
    shape = (spec.kv_prefill, spec.NKV, spec.HD)
    return rng.standard_normal(shape).astype(np.float32), rng.standard_normal(shape).astype(np.float32)


def build(spec: Spec = TINY, layers=None, embedding: bool = True, head: bool = True) -> dict:
    """Weights by tensor name: fp32 arrays for the embedding, norms and
    biases, raw GGUF block bytes (uint8) for the projections and the head.
    `layers` (default all) and the flags select a subset."""
    if spec.name == "tiny":
        # the tiny model's original single-stream generator (its golden file
        # was made from these bytes)
        rng = np.random.default_rng(spec.seed)
        w = {"model.embed_tokens.weight": rng.standard_normal((spec.V, spec.H)).astype(np.float32),
             "model.norm.weight": np.ones(spec.H, np.float32),
             "lm_head.weight": synth.make_weight("Q6_K", spec.V, spec.H, seed=spec.seed + 1)}
    else:
        w = {"model.norm.weight": np.full(spec.H, NORM_WEIGHT, np.float32)}
        if embedding:
            w["model.embed_tokens.weight"] = embedding_rows(spec, np.arange(spec.V))
        if head:
            w["lm_head.weight"] = synth.make_weight("Q6_K", spec.V, spec.H, seed=spec.seed * 1000 + 999)
    for i in range(spec.L) if layers is None else layers:
        w.update(layer_tensors(spec, i))
    return w


def _rms_norm(spec: Spec, x: np.ndarray, w: np.ndarray) -> np.ndarray:
    x32 = x.astype(np.float32, copy=False)
    var = np.mean(x32 * x32, axis=-1, keepdims=True)
    inv = 1.0 / np.sqrt(var + spec.EPS)
    return x32 * inv * w.astype(np.float32, copy=False)


_ROPE: dict = {}


def _rope_tables(spec: Spec) -> tuple[np.ndarray, np.ndarray]:
    if spec.name not in _ROPE:
        inv_freq = 1.0 / (spec.THETA ** (np.arange(0, spec.HD, 2, dtype=np.float32) / spec.HD))
        freqs = np.outer(np.arange(spec.MAX_POS, dtype=np.float32), inv_freq)
        _ROPE[spec.name] = (np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32))
    return _ROPE[spec.name]


def _rope(spec: Spec, x: np.ndarray, positions: np.ndarray) -> np.ndarray:
    cos, sin = _rope_tables(spec)
    half = spec.HD // 2
    x32 = x.astype(np.float32, copy=False)
    c = cos[positions][:, None, :]
    s = sin[positions][:, None, :]
    a, b = x32[..., :half], x32[..., half:]
    return np.concatenate([a * c - b * s, b * c + a * s], axis=-1)


def _softmax(x: np.ndarray) -> np.ndarray:
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def _proj(spec: Spec, backend, w: dict, name: str, x: np.ndarray) -> np.ndarray:
    n, k, q = quant_of(spec, name)
    method = {"Q4_K": backend.matmul_q4k, "Q6_K": backend.matmul_q6k}[q]
    y = np.asarray(method(np.ascontiguousarray(x, np.float32), w[name], n, k), np.float32).reshape(x.shape[0], n)
    bias = w.get(name[: -len("weight")] + "bias")
    return y if bias is None else y + bias


class KV:
    """Per-layer key/value history of one sequence (rows: positions),
    pre-filled as the spec says for the layers in `layers`."""

    def __init__(self, spec: Spec, layers=None):
        self.spec = spec
        self.k, self.v = {}, {}
        for i in range(spec.L) if layers is None else layers:
            if spec.kv_prefill:
                self.k[i], self.v[i] = kv_prefill(spec, i)
            else:
                self.k[i] = np.zeros((0, spec.NKV, spec.HD), np.float32)
                self.v[i] = np.zeros((0, spec.NKV, spec.HD), np.float32)

    def length(self, layer: int) -> int:
        return int(self.k[layer].shape[0])


def layer_forward(spec: Spec, backend, w: dict, i: int, hidden: np.ndarray, kv: KV) -> np.ndarray:
    """One decoder layer on `hidden` (seq, H) appended after layer i's cache."""
    seq = hidden.shape[0]
    past = kv.length(i)
    positions = np.arange(past, past + seq)
    group = spec.NH // spec.NKV
    p = f"model.layers.{i}"
    residual = hidden
    x = _rms_norm(spec, hidden, w[f"{p}.input_layernorm.weight"])
    q = _proj(spec, backend, w, f"{p}.self_attn.q_proj.weight", x).reshape(seq, spec.NH, spec.HD)
    k = _proj(spec, backend, w, f"{p}.self_attn.k_proj.weight", x).reshape(seq, spec.NKV, spec.HD)
    v = _proj(spec, backend, w, f"{p}.self_attn.v_proj.weight", x).reshape(seq, spec.NKV, spec.HD)
    q = _rope(spec, q, positions)
    k = _rope(spec, k, positions)
    kv.k[i] = np.concatenate([kv.k[i], k.astype(np.float32)], axis=0)
    kv.v[i] = np.concatenate([kv.v[i], v.astype(np.float32)], axis=0)
    # GQA: query head h reads KV head h // group (the reference repeats the
    # KV heads, np.repeat(k, group, axis=1); grouping the query heads instead
    # is the same product without the copy)
    scale = np.float32(1.0 / np.sqrt(spec.HD))
    qg = q.reshape(seq, spec.NKV, group, spec.HD)
    att = np.einsum("tkgd,Tkd->kgtT", qg, kv.k[i]).reshape(spec.NH, seq, -1) * scale
    total = past + seq
    mask = np.zeros((seq, total), np.float32)
    mask[np.arange(total)[None, :] > (np.arange(seq)[:, None] + past)] = -np.inf
    att = _softmax(att + mask).reshape(spec.NKV, group, seq, total)
    ctx = np.einsum("kgtT,Tkd->tkgd", att, kv.v[i]).reshape(seq, spec.H)
    hidden = residual + _proj(spec, backend, w, f"{p}.self_attn.o_proj.weight", ctx)
    residual = hidden
    x = _rms_norm(spec, hidden, w[f"{p}.post_attention_layernorm.weight"])
    gate = _proj(spec, backend, w, f"{p}.mlp.gate_proj.weight", x)
    up = _proj(spec, backend, w, f"{p}.mlp.up_proj.weight", x)
    with np.errstate(over="ignore"):
        s = 1.0 / (1.0 + np.exp(-gate))
    return residual + _proj(spec, backend, w, f"{p}.mlp.down_proj.weight", s * gate * up)


def forward(spec: Spec, backend, w: dict, tokens, kv: KV) -> np.ndarray:
    """Logits (seq, V) of `tokens` appended after the cached positions."""
    tokens = np.asarray(tokens, np.int64)
    if "model.embed_tokens.weight" in w:
        hidden = w["model.embed_tokens.weight"][tokens].astype(np.float32)
    else:
        hidden = embedding_rows(spec, tokens)
    for i in range(spec.L):
        hidden = layer_forward(spec, backend, w, i, hidden, kv)
    hidden = _rms_norm(spec, hidden, w["model.norm.weight"])
    return _proj(spec, backend, w, "lm_head.weight", hidden)


def teacher_forced_logits(spec: Spec, backend, w: dict, prompt, tokens, prompt_chunk: int = 0) -> np.ndarray:
    """Last-position logits after the prompt and after each of `tokens`
    (fed regardless of what this backend would pick): shape
    (len(tokens) + 1, V).  prompt_chunk > 0 feeds the prompt in chunks of
    that many tokens (the cache makes this the same computation)."""
    kv = KV(spec)
    prompt = np.asarray(prompt, np.int64)
    step = prompt_chunk or prompt.size
    for c0 in range(0, prompt.size, step):
        last = forward(spec, backend, w, prompt[c0:c0 + step], kv)[-1]
    out = [last]
    for t in tokens:
        out.append(forward(spec, backend, w, [int(t)], kv)[-1])
    return np.stack(out)
