"""Greedy-decode parity (the third correctness gate): random-init Qwen2
models in the config-4 quant mix decode against the reference.

The golden files hold what the unchanged reference forwarder computed on
these weights (``tests/golden/make_decode_golden.py``):

* ``decode_tiny_qwen2.npz``: the tiny model, an 8-token prompt, 12 greedy
  tokens and the full last-position logits after each step;
* ``decode_qwen2_7b.npz``: config 4, the Qwen2-7B architecture (28 layers,
  KV cache pre-filled with 4096 positions), a 32-token prompt and 64 greedy
  tokens; per step the top 16 logits, the logits at 1024 fixed vocabulary
  ids and max |logit|; plus the hidden states after layers 0 and 1 for the
  prompt.

The forward pass is restated in ``qwen2_restated.py`` (the reference tree is
not on the GPU box).  On CPU the restatement with the fp32 oracle doing the
projections is pinned to the golden data (tiny: every logit; Qwen2-7B: the
first two layers' hidden states, which is what fits a CPU run).  On the GPU
the same restatement runs with every projection on the B200 kernels (prompt
rows through the batched kernels, decode rows through the batch-1 kernel)
and, with the golden tokens fed back (teacher forcing), the logits must stay
within 1e-3 of the reference's and the argmax must match at every step whose
top-2 logit gap exceeds that tolerance; a free-running greedy decode must
then pick the reference's tokens.
"""

from __future__ import annotations

import os

import numpy as np
import pytest

import qwen2_restated as Q
from oracle import gguf_oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "decode_tiny_qwen2.npz")
GOLDEN_7B = os.path.join(HERE, "golden", "decode_qwen2_7b.npz")
TOL = 1e-3  # max|logit - reference| / max|reference logit|, per step


class OracleBackend:
    """The reference fp32 projections (dequantise, then a BLAS product)."""

    @staticmethod
    def matmul_q4k(x, w, n, k):
        return O.matvec_fp32("Q4_K", w, x, n, k)

    @staticmethod
    def matmul_q6k(x, w, n, k):
        return O.matvec_fp32("Q6_K", w, x, n, k)


def _golden():
    g = np.load(GOLDEN)
    return g["prompt"], g["tokens"], g["logits"]


def _check(logits, ref, tokens, tol):
    assert logits.shape == ref.shape
    for s in range(ref.shape[0]):
        err = O.rel_err(logits[s], ref[s])
        assert err < tol, (s, err)
        top2 = np.sort(ref[s])[-2:]
        if top2[1] - top2[0] > tol * np.max(np.abs(ref[s])):
            assert int(np.argmax(logits[s])) == int(np.argmax(ref[s])), s
    # the golden tokens are the reference's own greedy picks
    assert [int(np.argmax(r)) for r in ref[:-1]] == [int(t) for t in tokens]


def test_golden_tokens_are_greedy_and_confident():
    prompt, tokens, ref = _golden()
    assert prompt.shape == (8,) and tokens.shape == (12,) and ref.shape == (13, Q.TINY.V)
    gaps = [np.diff(np.sort(r)[-2:])[0] / np.max(np.abs(r)) for r in ref]
    assert sum(g > TOL for g in gaps) >= 10  # most steps are decisive


def test_restated_forward_matches_reference_on_cpu():
    """The NumPy restatement with the oracle's projections reproduces the
    reference forwarder's logits (to fp32 summation-order noise)."""
    prompt, tokens, ref = _golden()
    logits = Q.teacher_forced_logits(Q.TINY, OracleBackend, Q.build(Q.TINY), prompt, tokens)
    _check(logits, ref, tokens, 1e-5)


@pytest.mark.gpu
def test_greedy_decode_on_gpu_matches_reference(cuda_backend):
    prompt, tokens, ref = _golden()
    w = Q.build(Q.TINY)
    logits = Q.teacher_forced_logits(Q.TINY, cuda_backend, w, prompt, tokens)
    _check(logits, ref, tokens, TOL)
    # free-running greedy decode picks the reference's tokens
    kv = Q.KV(Q.TINY)
    last = Q.forward(Q.TINY, cuda_backend, w, prompt, kv)[-1]
    picked = []
    for _ in range(len(tokens)):
        picked.append(int(np.argmax(last)))
        last = Q.forward(Q.TINY, cuda_backend, w, [picked[-1]], kv)[-1]
    assert picked == [int(t) for t in tokens]


# ---- config 4: Qwen2-7B architecture ---------------------------------------

def _golden_7b():
    if not os.path.exists(GOLDEN_7B):
        pytest.fail(f"{GOLDEN_7B} missing: run tests/golden/make_decode_golden.py --model qwen2-7b")
    return np.load(GOLDEN_7B)


def _decisive(g) -> np.ndarray:
    """Steps whose reference top-2 logit gap exceeds the tolerance."""
    return (g["top_vals"][:, 0] - g["top_vals"][:, 1]) > TOL * g["max_abs"]


def test_qwen2_7b_golden_is_greedy_and_decisive():
    g = _golden_7b()
    assert g["prompt"].shape == (32,) and g["tokens"].shape == (64,)
    assert g["top_ids"].shape == (65, 16) and g["sample_vals"].shape == (65, 1024)
    # the golden tokens are the reference's own greedy picks
    assert list(g["top_ids"][:-1, 0]) == list(g["tokens"])
    assert _decisive(g).sum() >= 60
    assert _free_run_steps(_decisive(g), 64) >= 16


def test_qwen2_7b_restated_layers_match_reference_on_cpu():
    """The restatement's first two Qwen2-7B layers (biases, the pre-filled
    cache, RoPE at positions 4096.., GQA over 4 KV heads) with the oracle's
    projections reproduce the reference's hidden states for the prompt."""
    g = _golden_7b()
    spec = Q.QWEN2_7B
    w = Q.build(spec, layers=[0, 1], embedding=False, head=False)
    kv = Q.KV(spec, layers=[0, 1])
    hidden = Q.embedding_rows(spec, g["prompt"])
    for i, ref in ((0, g["hidden_l0"]), (1, g["hidden_l1"])):
        hidden = Q.layer_forward(spec, OracleBackend, w, i, hidden, kv)
        assert O.rel_err(hidden, ref) < 1e-5, i


@pytest.mark.gpu
def test_qwen2_7b_greedy_decode_on_gpu_matches_reference(cuda_backend):
    """Config 4 end to end on the B200 kernels: every q/k/v/o, gate/up/down
    and lm_head projection of the 28 layers (4.37 GB of Q4_K / Q6_K blocks)
    for a 32-token prompt (two 16-token chunks) and 64 decode tokens."""
    g = _golden_7b()
    spec = Q.QWEN2_7B
    w = Q.build(spec, embedding=False)
    prompt, tokens = g["prompt"], g["tokens"]
    logits = Q.teacher_forced_logits(spec, cuda_backend, w, prompt, tokens, prompt_chunk=16)
    decisive = _decisive(g)
    for s in range(logits.shape[0]):
        scale = float(g["max_abs"][s])
        err = max(np.max(np.abs(logits[s, g["sample_ids"]] - g["sample_vals"][s])),
                  np.max(np.abs(logits[s, g["top_ids"][s]] - g["top_vals"][s]))) / scale
        assert err < TOL, (s, err)
        if decisive[s]:
            assert int(np.argmax(logits[s])) == int(g["top_ids"][s, 0]), s
    # free-running greedy decode picks the reference's tokens up to the first
    # step whose top-2 gap is within the tolerance (after it the two runs
    # may legitimately part)
    m = _free_run_steps(decisive, len(tokens))
    kv = Q.KV(spec)
    for c0 in range(0, prompt.size, 16):
        last = Q.forward(spec, cuda_backend, w, prompt[c0:c0 + 16], kv)[-1]
    picked = []
    for _ in range(m):
        picked.append(int(np.argmax(last)))
        last = Q.forward(spec, cuda_backend, w, [picked[-1]], kv)[-1]
    assert picked == [int(t) for t in tokens[:m]]
    cuda_backend.close()


def _free_run_steps(decisive: np.ndarray, n: int) -> int:
    """Greedy tokens a free-running decode must reproduce: those before the
    first step that is not decisive (that step's pick may differ)."""
    nd = np.flatnonzero(~decisive)
    return n if nd.size == 0 else min(n, int(nd[0]))


# ---- the device-resident decode engine (every operator on the GPU) ---------

def _engine(spec, w, kv_prefill=None, max_pos=None):
    from flatrun_b200.decode import DecodeEngine, DecoderConfig
    cfg = DecoderConfig(hidden=spec.H, ffn=spec.F, vocab=spec.V, layers=spec.L, heads=spec.NH, kv_heads=spec.NKV,
                        eps=spec.EPS, rope_theta=spec.THETA, max_pos=max_pos or spec.MAX_POS)
    eng = DecodeEngine(cfg, w, lambda name: Q.quant_of(spec, name), kv_prefill=kv_prefill)
    eng.capture()
    return eng


def _engine_teacher_forced(eng, prompt, tokens):
    for t in prompt:
        eng.step(int(t))
    out = [eng.logits_host()]
    for t in tokens:
        eng.step(int(t))
        out.append(eng.logits_host())
    return np.stack(out)


@pytest.mark.gpu
def test_device_decode_engine_tiny(cuda_backend):
    """The whole token on the GPU (embedding, norms, RoPE, KV cache,
    attention, SwiGLU, head, argmax) in one CUDA graph per token: logits
    within 1e-3 of the reference at every step, and a free-running greedy
    decode that picks the reference's tokens."""
    prompt, tokens, ref = _golden()
    eng = _engine(Q.TINY, Q.build(Q.TINY))
    _check(_engine_teacher_forced(eng, prompt, tokens), ref, tokens, TOL)
    eng2 = _engine(Q.TINY, Q.build(Q.TINY))
    for t in prompt:
        eng2.step(int(t))
    picked = [eng2.argmax_host()]
    for _ in range(len(tokens) - 1):
        eng2.step(None)
        picked.append(eng2.argmax_host())
    assert picked == [int(t) for t in tokens]


@pytest.mark.gpu
def test_device_decode_engine_qwen2_7b(cuda_backend):
    """Config 4 on the device-resident engine: the 4096-position pre-filled
    cache, the 32-token prompt fed one token at a time, then the golden
    tokens (teacher forcing) and a free-running greedy decode."""
    g = _golden_7b()
    spec = Q.QWEN2_7B
    w = Q.build(spec)
    kv = {i: Q.kv_prefill(spec, i) for i in range(spec.L)}
    max_pos = spec.kv_prefill + 32 + 64 + 8
    eng = _engine(spec, w, kv_prefill=kv, max_pos=max_pos)
    logits = _engine_teacher_forced(eng, g["prompt"], g["tokens"])
    decisive = _decisive(g)
    for s in range(logits.shape[0]):
        scale = float(g["max_abs"][s])
        err = max(np.max(np.abs(logits[s, g["sample_ids"]] - g["sample_vals"][s])),
                  np.max(np.abs(logits[s, g["top_ids"][s]] - g["top_vals"][s]))) / scale
        assert err < TOL, (s, err)
        if decisive[s]:
            assert int(np.argmax(logits[s])) == int(g["top_ids"][s, 0]), s
    eng.close()
    del eng
    m = _free_run_steps(decisive, len(g["tokens"]))
    assert m >= 16  # the golden run is decisive long enough to be a real check
    eng = _engine(spec, w, kv_prefill=kv, max_pos=max_pos)
    for t in g["prompt"]:
        eng.step(int(t))
    picked = [eng.argmax_host()]
    for _ in range(m - 1):
        eng.step(None)
        picked.append(eng.argmax_host())
    assert picked == [int(t) for t in g["tokens"][:m]]
    eng.close()
