"""A tiny random-init Qwen2 decoder and a NumPy restatement of the reference's
forward pass, for greedy-decode parity tests (test infrastructure only).

The model has the Qwen2-7B layout at toy size (2 layers, hidden 256, FFN
512, 4 query / 2 KV heads of 64, vocab 320) and the config-4 quant mix: Q4_K
q/k/o/gate/up, Q6_K v/down and a Q6_K lm_head; norms are ones and the
embedding table is fp32.  `build()` is deterministic, so the golden generator
(which runs the reference forwarder on these weights) and the tests (which run
`forward()` below with the CUDA backend or the oracle) see identical bytes.

`forward()` restates `flatrun.model.qwen2.make_qwen2_forwarder` for this
architecture (no biases, no q/k norms, rotate-half RoPE, full causal
attention, untied head):
  embedding lookup                     qwen2.py:2153-2159
  RMSNorm in fp32                      qwen2.py:365-378
  RoPE tables, rotate-half layout      qwen2.py:398-476
  q/k/v, RoPE at absolute positions,
  KV append, GQA repeat, scaled
  scores + causal mask, softmax, AV    qwen2.py:1510-1625, :480-509
  o_proj + residual                    qwen2.py:1617-1646
  RMSNorm, gate/up, silu(gate) * up,
  down + residual                      qwen2.py:1648-1750
  final RMSNorm + lm_head (all rows)   qwen2.py:2238-2290
Projections go through `backend.matmul_q4k / matmul_q6k(x, raw, n, k)` with
x of shape (seq, k), the reference's native method signature.
"""

from __future__ import annotations

import numpy as np

from flatrun_b200 import synth

H, F, V, L, NH, NKV = 256, 512, 320, 2, 4, 2
HD = H // NH
KVD = NKV * HD
EPS = 1e-6
THETA = 1e6
MAX_POS = 256

# projection -> (rows n, columns k, quant)
PROJ = {
    "self_attn.q_proj": (H, H, "Q4_K"),
    "self_attn.k_proj": (KVD, H, "Q4_K"),
    "self_attn.v_proj": (KVD, H, "Q6_K"),
    "self_attn.o_proj": (H, H, "Q4_K"),
    "mlp.gate_proj": (F, H, "Q4_K"),
    "mlp.up_proj": (F, H, "Q4_K"),
    "mlp.down_proj": (H, F, "Q6_K"),
}
HEAD = (V, H, "Q6_K")


def build(seed: int = 5) -> dict:
    """Weights by tensor name: fp32 arrays for the embedding and norms, raw
    GGUF block bytes (uint8) for the projections and the head."""
    rng = np.random.default_rng(seed)
    w = {
        "model.embed_tokens.weight": rng.standard_normal((V, H)).astype(np.float32),
        "model.norm.weight": np.ones(H, np.float32),
        "lm_head.weight": synth.make_weight(HEAD[2], HEAD[0], HEAD[1], seed=seed + 1),
    }
    for i in range(L):
        p = f"model.layers.{i}"
        w[f"{p}.input_layernorm.weight"] = np.ones(H, np.float32)
        w[f"{p}.post_attention_layernorm.weight"] = np.ones(H, np.float32)
        for j, (name, (n, k, q)) in enumerate(PROJ.items()):
            w[f"{p}.{name}.weight"] = synth.make_weight(q, n, k, seed=seed * 1000 + 10 * i + j)
    return w


def quant_of(name: str) -> tuple[int, int, str] | None:
    """(n, k, quant) of a quantised tensor name, None for fp32 tensors."""
    if name == "lm_head.weight":
        return HEAD
    for proj, spec in PROJ.items():
        if name.endswith(f".{proj}.weight"):
            return spec
    return None


def _rms_norm(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    x32 = x.astype(np.float32, copy=False)
    var = np.mean(x32 * x32, axis=-1, keepdims=True)
    inv = 1.0 / np.sqrt(var + EPS)
    return x32 * inv * w.astype(np.float32, copy=False)


def _rope_tables() -> tuple[np.ndarray, np.ndarray]:
    inv_freq = 1.0 / (THETA ** (np.arange(0, HD, 2, dtype=np.float32) / HD))
    freqs = np.outer(np.arange(MAX_POS, dtype=np.float32), inv_freq)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


_COS, _SIN = _rope_tables()


def _rope(x: np.ndarray, positions: np.ndarray) -> np.ndarray:
    half = HD // 2
    x32 = x.astype(np.float32, copy=False)
    c = _COS[positions][:, None, :]
    s = _SIN[positions][:, None, :]
    a, b = x32[..., :half], x32[..., half:]
    return np.concatenate([a * c - b * s, b * c + a * s], axis=-1)


def _softmax(x: np.ndarray) -> np.ndarray:
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def _proj(backend, w: dict, name: str, x: np.ndarray) -> np.ndarray:
    n, k, q = quant_of(name)
    method = {"Q4_K": backend.matmul_q4k, "Q6_K": backend.matmul_q6k}[q]
    return np.asarray(method(np.ascontiguousarray(x, np.float32), w[name], n, k), np.float32).reshape(x.shape[0], n)


class KV:
    """Per-layer key/value history of one sequence (rows: positions)."""

    def __init__(self):
        self.k = [np.zeros((0, NKV, HD), np.float32) for _ in range(L)]
        self.v = [np.zeros((0, NKV, HD), np.float32) for _ in range(L)]

    @property
    def length(self) -> int:
        return int(self.k[0].shape[0])


def forward(backend, w: dict, tokens, kv: KV) -> np.ndarray:
    """Logits (seq, V) of `tokens` appended after the cached positions."""
    tokens = np.asarray(tokens, np.int64)
    seq = int(tokens.size)
    past = kv.length
    positions = np.arange(past, past + seq)
    hidden = w["model.embed_tokens.weight"][tokens].astype(np.float32)
    group = NH // NKV
    for i in range(L):
        p = f"model.layers.{i}"
        residual = hidden
        x = _rms_norm(hidden, w[f"{p}.input_layernorm.weight"])
        q = _proj(backend, w, f"{p}.self_attn.q_proj.weight", x).reshape(seq, NH, HD)
        k = _proj(backend, w, f"{p}.self_attn.k_proj.weight", x).reshape(seq, NKV, HD)
        v = _proj(backend, w, f"{p}.self_attn.v_proj.weight", x).reshape(seq, NKV, HD)
        q = _rope(q, positions)
        k = _rope(k, positions)
        kv.k[i] = np.concatenate([kv.k[i], k.astype(np.float32)], axis=0)
        kv.v[i] = np.concatenate([kv.v[i], v.astype(np.float32)], axis=0)
        k_full = np.repeat(kv.k[i], group, axis=1)
        v_full = np.repeat(kv.v[i], group, axis=1)
        scale = np.float32(1.0 / np.sqrt(HD))
        att = np.einsum("thd,Thd->htT", q, k_full) * scale
        total = past + seq
        mask = np.zeros((seq, total), np.float32)
        mask[np.arange(total)[None, :] > (np.arange(seq)[:, None] + past)] = -np.inf
        att = _softmax(att + mask)
        ctx = np.einsum("htT,Thd->thd", att, v_full).reshape(seq, H)
        hidden = residual + _proj(backend, w, f"{p}.self_attn.o_proj.weight", ctx)
        residual = hidden
        x = _rms_norm(hidden, w[f"{p}.post_attention_layernorm.weight"])
        gate = _proj(backend, w, f"{p}.mlp.gate_proj.weight", x)
        up = _proj(backend, w, f"{p}.mlp.up_proj.weight", x)
        with np.errstate(over="ignore"):
            s = 1.0 / (1.0 + np.exp(-gate))
        hidden = residual + _proj(backend, w, f"{p}.mlp.down_proj.weight", s * gate * up)
    hidden = _rms_norm(hidden, w["model.norm.weight"])
    return _proj(backend, w, "lm_head.weight", hidden)


def teacher_forced_logits(backend, w: dict, prompt, tokens) -> np.ndarray:
    """Last-position logits after the prompt and after each of `tokens`
    (fed regardless of what this backend would pick): shape
    (len(tokens) + 1, V)."""
    kv = KV()
    out = [forward(backend, w, prompt, kv)[-1]]
    for t in tokens:
        out.append(forward(backend, w, [int(t)], kv)[-1])
    return np.stack(out)
