"""Device-resident greedy decode of a Qwen2/Llama-architecture model.

Every operator of a decode token runs on the GPU, stream-ordered, with no
host round trip between layers, and the whole token is captured in one CUDA
graph that replays for every token (the token's position and id live in
device memory):

  embedding row                       frc_embed_row
  per layer:
    RMSNorm + q, k, v projections     frc_gemv_ex (norm inside the launch;
                                      one launch per quant group)
    bias + RoPE + KV append           frc_rope_append
    GQA attention over the cache      frc_attention_decode (split positions)
    o projection + residual           frc_gemv_ex, FRC_GEMV_ACCUMULATE
    RMSNorm + gate, up projections    frc_gemv_ex (one fused launch)
    SwiGLU + down + residual          frc_gemv_ex: x = silu(gate) * up, accumulate
  final RMSNorm + lm_head, argmax     frc_gemv_ex, frc_argmax

This is the reference forwarder's decode step (flatrun/model/qwen2.py
``make_qwen2_forwarder``: :1510-1646 attention, :1648-1751 MLP, :2238-2297
head) with the NumPy work moved onto the device; the projections are the
same B200 kernels the ``cuda`` backend slot calls.  PyTorch is used only to
allocate device memory and for the stream and graph plumbing.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib

_PROJ = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
         "mlp.up_proj", "mlp.down_proj")


@dataclass(frozen=True)
class DecoderConfig:
    hidden: int
    ffn: int
    vocab: int
    layers: int
    heads: int
    kv_heads: int
    eps: float
    rope_theta: float
    max_pos: int

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


def rope_tables(head_dim: int, theta: float, max_pos: int) -> tuple[np.ndarray, np.ndarray]:
    """cos/sin tables [max_pos][head_dim / 2] in fp32, computed as the
    reference does (qwen2.py:398-476): inv_freq = 1 / theta^(2i / d),
    angles = positions x inv_freq."""
    inv_freq = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))
    freqs = np.outer(np.arange(max_pos, dtype=np.float32), inv_freq)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


class DecodeEngine:
    """Greedy decode of one sequence with every weight and the KV cache in HBM.

    `weights` maps the reference's tensor names to host arrays or device
    tensors: raw GGUF block bytes (uint8, with `quant_of(name)` -> (n, k,
    quant)) for the projections and the head, fp32 arrays for norms, biases
    and an fp32 embedding table (or raw bytes with its quant).  `kv_prefill` optionally
    maps a layer to (keys, values) of shape (positions, kv_heads, head_dim)
    already in the cache before the first token.
    """

    def __init__(self, cfg: DecoderConfig, weights: dict, quant_of, device: int = 0, kv_prefill=None,
                 attn_splits: int = 0):
        import torch

        self.torch = torch
        self.cfg = cfg
        self.lib = _lib.load()
        self.device = device
        self._dev = torch.device("cuda", device)
        self.stream = torch.cuda.Stream(device=self._dev)
        c = cfg
        hd, kvd = c.head_dim, c.kv_heads * c.head_dim
        f32 = torch.float32

        def up(a, dtype):
            # host arrays are copied in; device tensors (a streamed GGUF
            # file, gguf_stream.load_decoder) are used where they are
            if isinstance(a, torch.Tensor):
                return a.to(self._dev).reshape(-1).view(torch.uint8) if dtype is np.uint8 \
                    else a.to(self._dev, torch.float32)
            a = np.asarray(a, dtype)
            return torch.from_numpy(np.ascontiguousarray(a.reshape(-1) if dtype is np.uint8 else a)).to(self._dev)

        self._w = {}  # name -> (device tensor, quant id, n, k)
        for name, arr in weights.items():
            q = quant_of(name)
            if q is not None:
                n, k, quant = q
                self._w[name] = (up(arr, np.uint8), _lib.QUANT_IDS[quant], n, k)
        self._norm = {name: up(a, np.float32) for name, a in weights.items() if name.endswith("norm.weight")}
        self._bias = {}
        for i in range(c.layers):
            p = f"model.layers.{i}.self_attn"
            if f"{p}.q_proj.bias" in weights:
                self._bias[i] = torch.cat([up(weights[f"{p}.{n}.bias"], np.float32).reshape(-1)
                                           for n in ("q_proj", "k_proj", "v_proj")])
        emb = weights["model.embed_tokens.weight"]
        eq = quant_of("model.embed_tokens.weight")
        self._emb_quant = 0 if eq is None else _lib.QUANT_IDS[eq[2]]
        self._emb = up(emb, np.float32 if eq is None else np.uint8)
        cos, sin = rope_tables(hd, c.rope_theta, c.max_pos)
        self._cos, self._sin = up(cos, np.float32), up(sin, np.float32)
        self.k_cache = [torch.zeros((c.max_pos, c.kv_heads, hd), dtype=f32, device=self._dev) for _ in range(c.layers)]
        self.v_cache = [torch.zeros((c.max_pos, c.kv_heads, hd), dtype=f32, device=self._dev) for _ in range(c.layers)]
        start = 0
        for i, (kp, vp) in (kv_prefill or {}).items():
            t = kp.shape[0]
            self.k_cache[i][:t] = up(kp, np.float32).reshape(kp.shape)
            self.v_cache[i][:t] = up(vp, np.float32).reshape(vp.shape)
            start = t
        self.pos = torch.tensor([start], dtype=torch.int32, device=self._dev)
        self.tok_in = torch.zeros(1, dtype=torch.int32, device=self._dev)
        self.tok_out = torch.zeros(1, dtype=torch.int32, device=self._dev)
        self.h = torch.zeros(c.hidden, dtype=f32, device=self._dev)
        self.x = torch.zeros(c.hidden, dtype=f32, device=self._dev)
        self.qkv = torch.zeros(c.hidden + 2 * kvd, dtype=f32, device=self._dev)
        self.ctx = torch.zeros(c.hidden, dtype=f32, device=self._dev)
        self.gate = torch.zeros(c.ffn, dtype=f32, device=self._dev)
        self.upb = torch.zeros(c.ffn, dtype=f32, device=self._dev)
        self.logits = torch.zeros(c.vocab, dtype=f32, device=self._dev)
        # one attention CTA per SM and KV head: each of its eight warps keeps
        # eight K (or V) rows in flight
        sm = torch.cuda.get_device_properties(self._dev).multi_processor_count
        self.splits = attn_splits or max(1, sm // c.kv_heads)
        ws = ctypes.c_size_t()
        _lib.check(self.lib.frc_attention_workspace(c.heads, hd, self.splits, ctypes.byref(ws)), self.lib)
        self.part = torch.zeros(int(ws.value), dtype=f32, device=self._dev)
        _lib.check(self.lib.frc_argmax_workspace(c.vocab, ctypes.byref(ws)), self.lib)
        self.argmax_ws = torch.zeros(int(ws.value), dtype=torch.uint8, device=self._dev)
        self._graph = None
        self.launches_per_token = 0

    # ---- launches ------------------------------------------------------------
    def _gemv(self, names, x, ys, x_mul=None, norm=None, accumulate=False):
        ws = [self._w[nm] for nm in names]
        cnt = len(ws)
        rc = self.lib.frc_gemv_ex(ws[0][1], cnt, (ctypes.c_void_p * cnt)(*[w[0].data_ptr() for w in ws]),
                                  (ctypes.c_size_t * cnt)(*[w[0].numel() for w in ws]),
                                  (ctypes.c_int64 * cnt)(*[w[2] for w in ws]), ws[0][3], x.data_ptr(),
                                  x_mul.data_ptr() if x_mul is not None else None,
                                  norm.data_ptr() if norm is not None else None, self.cfg.eps,
                                  _lib.FRC_GEMV_ACCUMULATE if accumulate else 0,
                                  (ctypes.c_void_p * cnt)(*[y.data_ptr() for y in ys]), self._st)
        _lib.check(rc, self.lib)
        self.launches_per_token += 1

    def _groups(self, names):
        """Consecutive names grouped by quant (one fused launch per group)."""
        out = []
        for nm in names:
            if out and self._w[out[-1][0]][1] == self._w[nm][1] and len(out[-1]) < 4:
                out[-1].append(nm)
            else:
                out.append([nm])
        return out

    def _token(self) -> None:
        """Enqueue one decode token (the graph body)."""
        c, lib, st = self.cfg, self.lib, self._st
        hd, kvd = c.head_dim, c.kv_heads * c.head_dim
        self.launches_per_token = 0

        def chk(rc: int, kernels: int = 1) -> None:
            _lib.check(rc, lib)
            self.launches_per_token += kernels

        chk(lib.frc_embed_row(self._emb_quant, self._emb.data_ptr(), c.hidden, self.tok_in.data_ptr(),
                              self.h.data_ptr(), st))
        q_out = self.qkv[:c.hidden]
        k_out = self.qkv[c.hidden:c.hidden + kvd]
        v_out = self.qkv[c.hidden + kvd:]
        outs = {"self_attn.q_proj": q_out, "self_attn.k_proj": k_out, "self_attn.v_proj": v_out}
        scale = float(np.float32(1.0 / np.sqrt(hd)))
        for i in range(c.layers):
            p = f"model.layers.{i}"
            ln1 = self._norm[f"{p}.input_layernorm.weight"]
            for grp in self._groups([f"{p}.{nm}.weight" for nm in _PROJ[:3]]):
                self._gemv(grp, self.h, [outs[g[len(p) + 1:-len(".weight")]] for g in grp], norm=ln1)
            bias = self._bias.get(i)
            chk(lib.frc_rope_append(self.qkv.data_ptr(), bias.data_ptr() if bias is not None else None, c.heads,
                                    c.kv_heads, hd, self._cos.data_ptr(), self._sin.data_ptr(), self.pos.data_ptr(),
                                    self.k_cache[i].data_ptr(), self.v_cache[i].data_ptr(), st))
            chk(lib.frc_attention_decode(q_out.data_ptr(), self.k_cache[i].data_ptr(), self.v_cache[i].data_ptr(),
                                         self.pos.data_ptr(), c.heads, c.kv_heads, hd, scale, self.splits,
                                         self.part.data_ptr(), self.ctx.data_ptr(), st), kernels=2)
            self._gemv([f"{p}.self_attn.o_proj.weight"], self.ctx, [self.h], accumulate=True)
            ln2 = self._norm[f"{p}.post_attention_layernorm.weight"]
            gu = [f"{p}.mlp.gate_proj.weight", f"{p}.mlp.up_proj.weight"]
            for grp in self._groups(gu):
                self._gemv(grp, self.h, [self.gate if g.endswith("gate_proj.weight") else self.upb for g in grp],
                           norm=ln2)
            self._gemv([f"{p}.mlp.down_proj.weight"], self.gate, [self.h], x_mul=self.upb, accumulate=True)
        self._gemv(["lm_head.weight"], self.h, [self.logits], norm=self._norm["model.norm.weight"])
        chk(lib.frc_argmax(self.logits.data_ptr(), c.vocab, self.tok_out.data_ptr(), self.argmax_ws.data_ptr(), st))
        chk(lib.frc_pos_advance(self.pos.data_ptr(), st))
        # the greedy pick is the next token's input unless step() overrides it
        self.tok_in.copy_(self.tok_out)
        self.launches_per_token += 1

    @property
    def _st(self):
        return ctypes.c_void_p(self.stream.cuda_stream)

    def capture(self) -> None:
        """Record one token as a CUDA graph (replayed by step())."""
        torch = self.torch
        with torch.cuda.stream(self.stream):
            # one eager token first: lazy module loading and launch
            # configuration happen outside the capture; then undo its effects
            pos0, tok0 = self.pos.clone(), self.tok_in.clone()
            self._token()
            self.stream.synchronize()
            self.pos.copy_(pos0)
            self.tok_in.copy_(tok0)
            self._graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self._graph, stream=self.stream):
                self._token()
        self.stream.synchronize()

    def step(self, token: int | None = None) -> None:
        """One token: feed `token` (None: the previous step's argmax) and
        advance the position.  Asynchronous on the engine's stream."""
        torch = self.torch
        with torch.cuda.stream(self.stream):
            if token is not None:
                self.tok_in.fill_(int(token))
            if self._graph is None:
                self._token()
            else:
                self._graph.replay()

    def logits_host(self) -> np.ndarray:
        self.stream.synchronize()
        return self.logits.cpu().numpy()

    def argmax_host(self) -> int:
        self.stream.synchronize()
        return int(self.tok_out.item())

    def close(self) -> None:
        self._graph = None
        self.stream.synchronize()


__all__ = ["DecoderConfig", "DecodeEngine", "rope_tables"]
