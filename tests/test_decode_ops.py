"""The device-resident decoder-step operators against NumPy restatements of
the reference forwarder's steps (GPU, through the C ABI)."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from flatrun_b200 import _lib, synth
from oracle import gguf_oracle as O

pytestmark = pytest.mark.gpu


def _t(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _st():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _np(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def _rms(x, w, eps):
    x = x.astype(np.float32)
    return x * (1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps)) * w


def test_rmsnorm_matches_reference_expression(cuda_backend):
    lib = _lib.load()
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, 3584)).astype(np.float32) * 40
    w = rng.standard_normal(3584).astype(np.float32)
    xd, wd = _t(x), _t(w)
    out = _t(np.zeros_like(x))
    _lib.check(lib.frc_rmsnorm(xd.data_ptr(), wd.data_ptr(), 3, 3584, 1e-6, out.data_ptr(), _st()), lib)
    np.testing.assert_allclose(_np(out), _rms(x, w, 1e-6), rtol=2e-6, atol=1e-6)


def _rope_ref(x, pos, cos, sin):
    half = x.shape[-1] // 2
    a, b = x[..., :half], x[..., half:]
    c, s = cos[pos], sin[pos]
    return np.concatenate([a * c - b * s, b * c + a * s], axis=-1)


@pytest.mark.parametrize("hd,past,splits", [(128, 777, 37), (128, 777, 1), (64, 300, 5), (128, 40, 64)])
def test_rope_append_and_attention_match_numpy(cuda_backend, hd, past, splits):
    """Bias + rotate-half RoPE at the device position, the cache append, and
    GQA decode attention (28 query / 4 KV heads) against the reference's
    NumPy steps (qwen2.py:1527-1614): 778 positions over 37 ranges, over
    one range (four passes of positions), head dim 64, and more ranges than
    positions (empty ranges)."""
    from flatrun_b200.decode import rope_tables
    lib = _lib.load()
    nh, nkv = 28, 4
    rng = np.random.default_rng(2 + hd + past + splits)
    cos, sin = rope_tables(hd, 1e6, 1024)
    kc = np.zeros((1024, nkv, hd), np.float32)
    vc = np.zeros((1024, nkv, hd), np.float32)
    kc[:past] = rng.standard_normal((past, nkv, hd))
    vc[:past] = rng.standard_normal((past, nkv, hd))
    qkv = rng.standard_normal(nh * hd + 2 * nkv * hd).astype(np.float32)
    bias = rng.standard_normal(qkv.size).astype(np.float32) * 0.1
    qkv_d, bias_d, cos_d, sin_d = _t(qkv), _t(bias), _t(cos), _t(sin)
    kc_d, vc_d = _t(kc), _t(vc)
    pos = _t(np.array([past], np.int32))
    _lib.check(lib.frc_rope_append(qkv_d.data_ptr(), bias_d.data_ptr(), nh, nkv, hd, cos_d.data_ptr(),
                                   sin_d.data_ptr(), pos.data_ptr(), kc_d.data_ptr(), vc_d.data_ptr(), _st()), lib)
    b = qkv + bias
    q = _rope_ref(b[:nh * hd].reshape(nh, hd), past, cos, sin)
    k = _rope_ref(b[nh * hd:nh * hd + nkv * hd].reshape(nkv, hd), past, cos, sin)
    v = b[nh * hd + nkv * hd:].reshape(nkv, hd)
    np.testing.assert_allclose(_np(qkv_d)[:nh * hd].reshape(nh, hd), q, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(_np(kc_d)[past], k, rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(_np(vc_d)[past], v)
    ws = ctypes.c_size_t()
    _lib.check(lib.frc_attention_workspace(nh, hd, splits, ctypes.byref(ws)), lib)
    import torch
    part = torch.zeros(ws.value, device="cuda")
    out = torch.zeros(nh * hd, device="cuda")
    scale = float(np.float32(1.0 / np.sqrt(hd)))
    _lib.check(lib.frc_attention_decode(qkv_d.data_ptr(), kc_d.data_ptr(), vc_d.data_ptr(), pos.data_ptr(), nh, nkv,
                                        hd, scale, splits, part.data_ptr(), out.data_ptr(), _st()), lib)
    kh, vh = _np(kc_d)[:past + 1], _np(vc_d)[:past + 1]
    qd = _np(qkv_d)[:nh * hd].reshape(nh, hd)
    kf, vf = np.repeat(kh, nh // nkv, axis=1), np.repeat(vh, nh // nkv, axis=1)
    att = np.einsum("hd,Thd->hT", qd, kf) * np.float32(scale)
    att = np.exp(att - att.max(axis=-1, keepdims=True))
    att /= att.sum(axis=-1, keepdims=True)
    ref = np.einsum("hT,Thd->hd", att, vf)
    np.testing.assert_allclose(_np(out).reshape(nh, hd), ref, rtol=2e-5, atol=2e-6)


@pytest.mark.parametrize("n", [1, 7, 152064, 300001])
def test_argmax_lowest_index_of_ties_and_replays(cuda_backend, n):
    import torch
    lib = _lib.load()
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    if n > 10:
        x[n // 3] = x[n - 2] = x.max() + 1.0  # a tie: the lower index wins
    xd = _t(x)
    ws = ctypes.c_size_t()
    _lib.check(lib.frc_argmax_workspace(n, ctypes.byref(ws)), lib)
    wsd = torch.zeros(ws.value, dtype=torch.uint8, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(3):  # the ticket resets itself
        _lib.check(lib.frc_argmax(xd.data_ptr(), n, out.data_ptr(), wsd.data_ptr(), _st()), lib)
        assert int(_np(out)[0]) == int(np.argmax(x))


@pytest.mark.parametrize("fmt", [None, "Q4_K", "Q6_K", "Q8_0"])
def test_embed_row(cuda_backend, fmt):
    lib = _lib.load()
    vocab, n = 50, 512
    if fmt is None:
        table = np.random.default_rng(3).standard_normal((vocab, n)).astype(np.float32)
        ref = table
        qid = 0
    else:
        table = synth.make_weight(fmt, vocab, n, seed=4)
        ref = O.dequant(fmt, table, vocab, n)
        qid = _lib.QUANT_IDS[fmt]
    td = _t(table)
    import torch
    out = torch.zeros(n, device="cuda")
    for tok in (0, 17, vocab - 1):
        tk = _t(np.array([tok], np.int32))
        _lib.check(lib.frc_embed_row(qid, td.data_ptr(), n, tk.data_ptr(), out.data_ptr(), _st()), lib)
        assert O.same_bits(_np(out), ref[tok])


@pytest.mark.parametrize("fmt,k", [("Q4_K", 3584), ("Q6_K", 3584), ("Q4_K", 18944), ("Q5_K", 4096), ("Q8_0", 4096)])
def test_gemv_ex_norm_swiglu_accumulate(cuda_backend, fmt, k):
    """frc_gemv_ex: RMSNorm applied inside the launch, SwiGLU activations and
    y += W x, each against the reference expression with the fp64 oracle."""
    import torch
    lib = _lib.load()
    n = 700
    raw = synth.make_weight(fmt, n, k, seed=5)
    rng = np.random.default_rng(6)
    x = (rng.standard_normal(k) * 30).astype(np.float32)
    u = rng.standard_normal(k).astype(np.float32)
    w = rng.standard_normal(k).astype(np.float32)
    y0 = rng.standard_normal(n).astype(np.float32)
    wd, xd, ud, gd = _t(raw), _t(x), _t(u), _t(w)
    qid = _lib.QUANT_IDS[fmt]

    def run(x_mul=None, norm=None, acc=False, y_init=None):
        y = _t(y_init if y_init is not None else np.zeros(n, np.float32))
        _lib.check(lib.frc_gemv_ex(qid, 1, (ctypes.c_void_p * 1)(wd.data_ptr()), (ctypes.c_size_t * 1)(raw.nbytes),
                                   (ctypes.c_int64 * 1)(n), k, xd.data_ptr(),
                                   x_mul.data_ptr() if x_mul is not None else None,
                                   norm.data_ptr() if norm is not None else None, 1e-6,
                                   _lib.FRC_GEMV_ACCUMULATE if acc else 0, (ctypes.c_void_p * 1)(y.data_ptr()),
                                   _st()), lib)
        return _np(y)

    xn = _rms(x, w, 1e-6)
    ref = O.matvec_fp64(fmt, raw, xn, n, k)
    assert O.rel_err(run(norm=gd), ref) < 2e-5
    s = 1.0 / (1.0 + np.exp(-x.astype(np.float32)))
    xs = (s * x) * u
    ref = O.matvec_fp64(fmt, raw, xs, n, k)
    assert O.rel_err(run(x_mul=ud), ref) < 2e-5
    ref = O.matvec_fp64(fmt, raw, x, n, k) + y0
    assert O.rel_err(run(acc=True, y_init=y0), ref) < 2e-5
    torch.cuda.synchronize()
