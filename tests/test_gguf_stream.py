"""GGUF -> HBM streaming loader: the GGUF reader against files written per the
format (and against the reference's own reader where the reference tree is
present), and the streamed upload and a decoder built from a GGUF file on the
GPU."""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

import gguf_writer as W
import qwen2_restated as Q
from flatrun_b200 import gguf_stream as G
from flatrun_b200 import synth

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFERENCE = os.environ.get("FLATRUN_REFERENCE", os.path.join(os.path.dirname(REPO), "reference"))


def _tiny_gguf(path: str, spec=Q.TINY) -> dict:
    """The tiny Qwen2 model (qwen2_restated.build) written as GGUF with
    llama.cpp tensor names; returns the weights by the reference's names."""
    w = Q.build(spec)
    inv = {v: k for k, v in G._TO_HF.items()}
    tensors = []
    for name, arr in w.items():
        q = Q.quant_of(spec, name)
        parts = name.split(".")
        if name.startswith("model.layers."):
            gname = f"blk.{parts[2]}.{inv['.'.join(parts[3:-1])]}.{parts[-1]}"
        else:
            gname = f"{inv['.'.join(parts[:-1])]}.{parts[-1]}"
        if q is None:
            a = np.asarray(arr, np.float32)
            tensors.append((gname, 0, a.shape, a))
        else:
            n, k, quant = q
            tensors.append((gname, G.GGML_IDS[quant], (n, k), np.asarray(arr, np.uint8)))
    md = {
        "general.architecture": (W.STR, "qwen2"), "general.alignment": (W.U32, 64),
        "qwen2.block_count": (W.U32, spec.L), "qwen2.embedding_length": (W.U32, spec.H),
        "qwen2.feed_forward_length": (W.U32, spec.F), "qwen2.attention.head_count": (W.U32, spec.NH),
        "qwen2.attention.head_count_kv": (W.U32, spec.NKV),
        "qwen2.attention.layer_norm_rms_epsilon": (W.F32, spec.EPS), "qwen2.rope.freq_base": (W.F32, spec.THETA),
        "qwen2.context_length": (W.U32, spec.MAX_POS),
        "tokenizer.ggml.tokens": (W.ARR, W.STR, [f"t{i}" for i in range(8)]),
    }
    W.write_gguf(path, md, tensors, alignment=64)
    return w


def test_reader_round_trip(tmp_path):
    path = str(tmp_path / "tiny.gguf")
    w = _tiny_gguf(path)
    with G.GGUFReader(path) as r:
        assert r.version == 3
        assert r.metadata["qwen2.block_count"] == Q.TINY.L
        assert r.metadata["tokenizer.ggml.tokens"][3] == "t3"
        assert abs(r.metadata["qwen2.rope.freq_base"] - Q.TINY.THETA) < 1
        assert r.data_offset % 64 == 0
        assert set(r.tensors) == set(w)
        for name, arr in w.items():
            t = r.tensors[name]
            assert t.offset % 64 == 0
            q = Q.quant_of(Q.TINY, name)
            if q is None:
                assert t.quant == "F32" and t.shape == np.asarray(arr).shape
                assert np.array_equal(r.array(name), arr)
            else:
                assert (t.quant, t.shape) == (q[2], (q[0], q[1]))
                assert t.nbytes == synth.weight_bytes(q[2], q[0], q[1])
                assert np.array_equal(r.raw(name), arr)
        cfg = G.decoder_config(r)
        assert (cfg.hidden, cfg.ffn, cfg.vocab, cfg.layers, cfg.heads, cfg.kv_heads) == \
            (Q.TINY.H, Q.TINY.F, Q.TINY.V, Q.TINY.L, Q.TINY.NH, Q.TINY.NKV)


def test_reader_rejects_bad_files(tmp_path):
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGML" + b"\0" * 40)
    with pytest.raises(ValueError):
        G.GGUFReader(str(bad))
    path = str(tmp_path / "short.gguf")
    W.write_gguf(path, {}, [("blk.0.attn_q.weight", 12, (16, 256), np.zeros(16 * 144, np.uint8))])
    data = open(path, "rb").read()
    open(path, "wb").write(data[:-100])  # the tensor runs past the end
    with pytest.raises(ValueError):
        G.GGUFReader(path)


def test_names_follow_the_reference_translation():
    assert G.hf_name("blk.3.attn_q.weight") == "model.layers.3.self_attn.q_proj.weight"
    assert G.hf_name("blk.0.ffn_down.weight") == "model.layers.0.mlp.down_proj.weight"
    assert G.hf_name("token_embd.weight") == "model.embed_tokens.weight"
    assert G.hf_name("output.weight") == "lm_head.weight"
    assert G.hf_name("output_norm.weight") == "model.norm.weight"


def test_reader_matches_reference_reader(tmp_path):
    """The reference's GGUFBackend (backend/gguf.py:270, :422) on the same
    file: names, shapes, byte sizes, offsets and quant tags agree."""
    src = os.path.join(REFERENCE, "src")
    if not os.path.isdir(os.path.join(src, "flatrun")):
        pytest.skip("reference tree not present")
    sys.path.insert(0, src)
    try:
        from flatrun.backend.gguf import GGUFBackend
    finally:
        sys.path.remove(src)
    path = str(tmp_path / "tiny.gguf")
    _tiny_gguf(path)
    ref = GGUFBackend(path)
    ref.open()
    try:
        with G.GGUFReader(path) as r:
            assert {k.name for k in ref.list_tensors()} == set(r.tensors)
            for name, t in r.tensors.items():
                m = ref.get_metadata(name)
                assert tuple(m.shape) == t.shape and m.byte_size == t.nbytes and m.offset == t.offset
                assert (m.quantization or "F32") == t.quant
                h = ref.open_handle(name)
                assert bytes(np.asarray(h.as_numpy()).view(np.uint8).reshape(-1)) == bytes(r.raw(name))
    finally:
        ref.close()


@pytest.mark.gpu
def test_streamer_uploads_bytes_exactly():
    import torch
    rng = np.random.default_rng(1)
    arrays = {f"t{i}": rng.integers(0, 256, size, dtype=np.uint8) for i, size in
              enumerate([1, 4096, 65536, 65537, 300001, 1 << 20])}
    st = G.HBMStreamer(0, chunk_bytes=65536, buffers=2, workers=3)
    for name, a in arrays.items():
        st.submit(name, a)
    for name, a in arrays.items():
        d = st.get(name)
        torch.cuda.synchronize()
        assert np.array_equal(d.cpu().numpy(), a), name
    assert st.bytes_streamed == sum(a.nbytes for a in arrays.values())
    st.close()


@pytest.mark.gpu
def test_decoder_from_streamed_gguf_matches_host_arrays(tmp_path, cuda_backend):
    """The tiny model streamed from a GGUF file into HBM decodes exactly as
    the same weights uploaded from host arrays: identical logits, bit for
    bit, over a prompt and greedy steps."""
    from flatrun_b200.decode import DecodeEngine, DecoderConfig
    path = str(tmp_path / "tiny.gguf")
    w = _tiny_gguf(path)
    st = G.HBMStreamer(0, chunk_bytes=1 << 16, buffers=2)
    eng = G.load_decoder(path, streamer=st)
    st.close()
    s = Q.TINY
    # GGUF stores eps and theta as float32: the same values the kernels take
    cfg = DecoderConfig(hidden=s.H, ffn=s.F, vocab=s.V, layers=s.L, heads=s.NH, kv_heads=s.NKV,
                        eps=float(np.float32(s.EPS)), rope_theta=float(np.float32(s.THETA)), max_pos=s.MAX_POS)
    assert eng.cfg == cfg
    ref = DecodeEngine(cfg, w, lambda name: Q.quant_of(s, name))
    for e in (eng, ref):
        e.capture()
    for t in [3, 17, 250, 9, 41]:
        eng.step(t)
        ref.step(t)
        assert np.array_equal(eng.logits_host(), ref.logits_host())
    for _ in range(6):
        eng.step(None)
        ref.step(None)
        assert eng.argmax_host() == ref.argmax_host()
        assert np.array_equal(eng.logits_host(), ref.logits_host())
