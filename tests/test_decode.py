"""Greedy-decode parity (the third correctness gate): a tiny random-init
Qwen2 model in the config-4 quant mix decodes against the reference.

``tests/golden/decode_tiny_qwen2.npz`` holds what the reference forwarder
computed on these weights (an 8-token prompt, 12 greedy tokens and the
last-position logits after each step; ``make_decode_golden.py``).  The
forward pass itself is restated in ``tiny_qwen2.py`` (the reference tree is
not on the GPU box); the CPU test pins that restatement to the golden logits
with the fp32 oracle doing the projections, and the GPU test runs the same
restatement with every projection on the B200 kernels (prefill rows through
the batched kernel, decode rows through the batch-1 kernel) and checks, with
the golden tokens fed back (teacher forcing), that the logits stay within
1e-3 of the reference's and that the argmax matches at every step whose
top-2 logit gap exceeds that tolerance.
"""

from __future__ import annotations

import os

import numpy as np
import pytest

import tiny_qwen2 as T
from oracle import gguf_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "decode_tiny_qwen2.npz")
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
    assert prompt.shape == (8,) and tokens.shape == (12,) and ref.shape == (13, T.V)
    gaps = [np.diff(np.sort(r)[-2:])[0] / np.max(np.abs(r)) for r in ref]
    assert sum(g > TOL for g in gaps) >= 10  # most steps are decisive


def test_restated_forward_matches_reference_on_cpu():
    """The NumPy restatement with the oracle's projections reproduces the
    reference forwarder's logits (to fp32 summation-order noise)."""
    prompt, tokens, ref = _golden()
    logits = T.teacher_forced_logits(OracleBackend, T.build(), prompt, tokens)
    _check(logits, ref, tokens, 1e-5)


@pytest.mark.gpu
def test_greedy_decode_on_gpu_matches_reference(cuda_backend):
    prompt, tokens, ref = _golden()
    logits = T.teacher_forced_logits(cuda_backend, T.build(), prompt, tokens)
    _check(logits, ref, tokens, TOL)
    # free-running greedy decode picks the reference's tokens
    kv = T.KV()
    w = T.build()
    last = T.forward(cuda_backend, w, prompt, kv)[-1]
    picked = []
    for _ in range(len(tokens)):
        picked.append(int(np.argmax(last)))
        last = T.forward(cuda_backend, w, [picked[-1]], kv)[-1]
    assert picked == [int(t) for t in tokens]
