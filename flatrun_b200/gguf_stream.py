"""GGUF -> HBM streaming loader.

The reference reads GGUF files in ``backend/gguf.py`` (``GGUFBackend.open``
:270 parses the header and maps the file, ``open_handle`` :422 returns
zero-copy mmap handles) and its layer scheduler (``runtime/scheduler.py:222``)
hands those handles to the NumPy forwarder; nothing is uploaded anywhere.
This module puts the same bytes in HBM:

* ``GGUFReader`` parses a GGUF v2/v3 file (magic, version, tensor and
  key/value counts, typed key/value pairs, the tensor table, the data section
  at ``general.alignment``) and exposes every tensor as a read-only view of
  one memory map.  Shapes are reported in NumPy order (GGUF stores the fastest
  axis first; the reference reverses them the same way, gguf.py:542-551) and
  names are translated to the reference's HuggingFace Qwen2 names
  (gguf.py:185-215).
* ``HBMStreamer`` uploads tensors through a ring of pinned staging buffers on
  a dedicated copy stream: a host thread copies the next chunk from the map
  into a free pinned buffer while the DMA of the previous one runs, and every
  tensor completes an event.  Compute on other streams waits only for the
  tensors it uses, so layer L + 1 streams in while layer L runs, and decoding
  can start as soon as the first layers are resident.
* ``load_decoder`` builds a ``DecodeEngine``'s configuration and weights from a
  Qwen2 GGUF file through the streamer (the embedding stays in its GGUF quant
  and is gathered a row at a time on the device, instead of the forwarder's
  full-table dequantisation, qwen2.py:1367-1386).
"""

from __future__ import annotations

import mmap
import os
import struct
import threading
from dataclasses import dataclass
from typing import Any

import numpy as np

GGUF_MAGIC = b"GGUF"

# ggml tensor types: id -> (name, bytes per block, elements per block); the
# ids and block geometries of the GGUF format (the reference's table,
# gguf.py:59-86, holds the same values)
GGML_TYPES: dict[int, tuple[str, int, int]] = {
    0: ("F32", 4, 1), 1: ("F16", 2, 1), 2: ("Q4_0", 18, 32), 3: ("Q4_1", 20, 32), 6: ("Q5_0", 22, 32),
    7: ("Q5_1", 24, 32), 8: ("Q8_0", 34, 32), 9: ("Q8_1", 36, 32), 10: ("Q2_K", 84, 256),
    11: ("Q3_K", 110, 256), 12: ("Q4_K", 144, 256), 13: ("Q5_K", 176, 256), 14: ("Q6_K", 210, 256),
    15: ("Q8_K", 292, 256), 30: ("BF16", 2, 1), 41: ("Q1_0", 18, 128),
}
GGML_IDS = {v[0]: k for k, v in GGML_TYPES.items()}

# GGUF metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_SCALAR = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f", _BOOL: "<?",
           _U64: "<Q", _I64: "<q", _F64: "<d"}

# llama.cpp tensor names -> the reference's HuggingFace Qwen2 names
_TO_HF = {
    "token_embd": "model.embed_tokens", "output_norm": "model.norm", "output": "lm_head",
    "attn_norm": "input_layernorm", "attn_q": "self_attn.q_proj", "attn_k": "self_attn.k_proj",
    "attn_v": "self_attn.v_proj", "attn_output": "self_attn.o_proj", "ffn_norm": "post_attention_layernorm",
    "ffn_gate": "mlp.gate_proj", "ffn_up": "mlp.up_proj", "ffn_down": "mlp.down_proj",
}


def hf_name(name: str) -> str:
    """``blk.3.attn_q.weight`` -> ``model.layers.3.self_attn.q_proj.weight``;
    names outside the table are returned unchanged."""
    stem, dot, suffix = name.rpartition(".")
    if not dot:
        return name
    if stem.startswith("blk."):
        _, idx, base = stem.split(".", 2)
        return f"model.layers.{idx}.{_TO_HF.get(base, base)}.{suffix}"
    return f"{_TO_HF.get(stem, stem)}.{suffix}"


def tensor_bytes(ggml_type: int, numel: int) -> int:
    name, bsize, qk = GGML_TYPES[ggml_type]
    return (numel + qk - 1) // qk * bsize


@dataclass(frozen=True)
class GGUFTensor:
    name: str          # the reference's (HuggingFace) name
    gguf_name: str
    shape: tuple       # NumPy order (rows, cols) for a matrix
    ggml_type: int
    offset: int        # absolute file offset
    nbytes: int

    @property
    def quant(self) -> str:
        return GGML_TYPES[self.ggml_type][0]


class GGUFReader:
    """Header, metadata and tensor table of a GGUF v2/v3 file; tensor bytes
    as views of one read-only memory map."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self._map = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        buf = self._map
        if len(buf) < 24 or buf[:4] != GGUF_MAGIC:
            raise ValueError(f"{path}: not a GGUF file")
        self.version, n_tensors, n_kv = struct.unpack_from("<IQQ", buf, 4)
        if self.version not in (2, 3):
            raise ValueError(f"{path}: GGUF version {self.version} is not supported (2 or 3)")
        pos = 24
        self.metadata: dict[str, Any] = {}
        for _ in range(n_kv):
            key, pos = self._string(pos)
            (vt,) = struct.unpack_from("<I", buf, pos)
            value, pos = self._value(vt, pos + 4)
            self.metadata[key] = value
        infos = []
        for _ in range(n_tensors):
            name, pos = self._string(pos)
            (nd,) = struct.unpack_from("<I", buf, pos)
            dims = struct.unpack_from(f"<{nd}Q", buf, pos + 4)
            pos += 4 + 8 * nd
            gtype, rel = struct.unpack_from("<IQ", buf, pos)
            pos += 12
            infos.append((name, tuple(int(d) for d in dims), int(gtype), int(rel)))
        align = int(self.metadata.get("general.alignment", 32))
        self.data_offset = (pos + align - 1) // align * align
        self.tensors: dict[str, GGUFTensor] = {}
        for name, dims, gtype, rel in infos:
            if gtype not in GGML_TYPES:
                raise ValueError(f"{path}: tensor {name} has unknown ggml type {gtype}")
            numel = int(np.prod(dims)) if dims else 1
            t = GGUFTensor(hf_name(name), name, tuple(reversed(dims)), gtype, self.data_offset + rel,
                           tensor_bytes(gtype, numel))
            if t.offset + t.nbytes > len(buf):
                raise ValueError(f"{path}: tensor {name} runs past the end of the file")
            self.tensors[t.name] = t

    def _string(self, pos: int) -> tuple[str, int]:
        (n,) = struct.unpack_from("<Q", self._map, pos)
        return bytes(self._map[pos + 8:pos + 8 + n]).decode("utf-8"), pos + 8 + n

    def _value(self, vt: int, pos: int):
        if vt in _SCALAR:
            fmt = _SCALAR[vt]
            (v,) = struct.unpack_from(fmt, self._map, pos)
            return v, pos + struct.calcsize(fmt)
        if vt == _STR:
            return self._string(pos)
        if vt == _ARR:
            et, n = struct.unpack_from("<IQ", self._map, pos)
            pos += 12
            out = []
            for _ in range(n):
                v, pos = self._value(et, pos)
                out.append(v)
            return out, pos
        raise ValueError(f"{self.path}: unknown metadata value type {vt}")

    def raw(self, name: str) -> np.ndarray:
        """The tensor's bytes (uint8, a view of the map)."""
        t = self.tensors[name]
        return np.frombuffer(self._map, dtype=np.uint8, count=t.nbytes, offset=t.offset)

    def array(self, name: str) -> np.ndarray:
        """F32/F16 tensors as float arrays in NumPy shape; quantised tensors as
        their raw bytes."""
        t = self.tensors[name]
        if t.ggml_type == 0:
            return self.raw(name).view(np.float32).reshape(t.shape)
        if t.ggml_type == 1:
            return self.raw(name).view(np.float16).reshape(t.shape)
        return self.raw(name)

    def close(self) -> None:
        try:
            self._map.close()
        except BufferError:
            pass  # views of the map are still alive; it closes when they go
        self._f.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


class HBMStreamer:
    """Host arrays -> device tensors through pinned staging on copy streams.

    ``submit(name, array)`` returns at once.  Each of ``workers`` host threads
    owns a ring of ``buffers`` pinned buffers of ``chunk_bytes`` and a copy
    stream; it takes the next submitted tensor, copies it chunk by chunk from
    the (mapped) host array into its next free pinned buffer while the DMA of
    the previous chunk runs, and records the tensor's event after its last
    chunk.  Tensors are taken in submission order, several at a time (one per
    worker), so the host copies, which bound a single stream, run in parallel.
    ``get(name, stream)`` makes `stream` wait for that event and returns the
    device tensor (uint8 bytes, reshaped and typed by the caller)."""

    def __init__(self, device: int = 0, chunk_bytes: int = 16 << 20, buffers: int = 2, workers: int = 4):
        import torch

        self.torch = torch
        self.device = torch.device("cuda", device)
        self.chunk = int(chunk_bytes)
        self._queue: list = []
        self._cv = threading.Condition()
        self._done: dict[str, Any] = {}    # name -> (device tensor, event)
        self._error: BaseException | None = None
        self._closed = False
        self.bytes_streamed = 0
        self._threads = [threading.Thread(target=self._run, args=(buffers,), name=f"hbm-streamer-{i}", daemon=True)
                         for i in range(workers)]
        for t in self._threads:
            t.start()

    def submit(self, name: str, array: np.ndarray) -> None:
        src = np.ascontiguousarray(array).reshape(-1).view(np.uint8)
        dev = self.torch.empty(src.nbytes, dtype=self.torch.uint8, device=self.device)
        with self._cv:
            self._queue.append((name, src, dev))
            self._cv.notify()

    def _run(self, nbuf: int) -> None:
        torch = self.torch
        try:
            with torch.cuda.device(self.device):
                stream = torch.cuda.Stream(device=self.device)
                bufs = [torch.empty(self.chunk, dtype=torch.uint8, pin_memory=True) for _ in range(nbuf)]
                views = [b.numpy() for b in bufs]
                last = [None] * nbuf  # event of the last DMA out of each buffer
                nxt = 0
                while True:
                    with self._cv:
                        while not self._queue and not self._closed:
                            self._cv.wait()
                        if not self._queue:
                            stream.synchronize()
                            return
                        name, src, dev = self._queue.pop(0)
                    for off in range(0, src.nbytes, self.chunk):
                        n = min(self.chunk, src.nbytes - off)
                        b = nxt
                        nxt = (b + 1) % nbuf
                        if last[b] is not None:
                            last[b].synchronize()  # the buffer's previous DMA has read it
                        np.copyto(views[b][:n], src[off:off + n])
                        with torch.cuda.stream(stream):
                            dev[off:off + n].copy_(bufs[b][:n], non_blocking=True)
                            ev = torch.cuda.Event()
                            ev.record(stream)
                        last[b] = ev
                    ev = torch.cuda.Event()
                    ev.record(stream)
                    nbytes = src.nbytes
                    del src  # no view of the caller's (mapped) array outlives its upload
                    with self._cv:
                        self._done[name] = (dev, ev)
                        self.bytes_streamed += nbytes
                        self._cv.notify_all()
        except BaseException as exc:  # surfaced by get()
            with self._cv:
                self._error = exc
                self._cv.notify_all()

    def ready(self, name: str) -> bool:
        with self._cv:
            return name in self._done and self._done[name][1].query()

    def get(self, name: str, stream=None):
        """The device bytes of `name`; `stream` (default: the current one)
        waits for their upload."""
        with self._cv:
            while name not in self._done:
                if self._error is not None:
                    raise RuntimeError(f"HBM streamer failed: {self._error!r}") from self._error
                self._cv.wait()
            dev, ev = self._done[name]
        (stream or self.torch.cuda.current_stream(self.device)).wait_event(ev)
        return dev

    def close(self) -> None:
        with self._cv:
            self._closed = True
            self._cv.notify_all()
        for t in self._threads:
            t.join()


def decoder_config(reader: GGUFReader, max_pos: int | None = None):
    """The decoder configuration of a Qwen2 GGUF file (its ``qwen2.*``
    metadata, the vocabulary from the embedding's rows)."""
    from .decode import DecoderConfig

    md = reader.metadata
    arch = md.get("general.architecture", "qwen2")
    g = lambda key, default=None: md.get(f"{arch}.{key}", default)  # noqa: E731
    vocab = reader.tensors["model.embed_tokens.weight"].shape[0]
    return DecoderConfig(hidden=int(g("embedding_length")), ffn=int(g("feed_forward_length")), vocab=int(vocab),
                         layers=int(g("block_count")), heads=int(g("attention.head_count")),
                         kv_heads=int(g("attention.head_count_kv")),
                         eps=float(g("attention.layer_norm_rms_epsilon", 1e-6)),
                         rope_theta=float(g("rope.freq_base", 1e6)),
                         max_pos=int(max_pos or g("context_length", 4096)))


def load_decoder(path: str, device: int = 0, max_pos: int | None = None, streamer: HBMStreamer | None = None,
                 **engine_kwargs):
    """A ``DecodeEngine`` whose weights stream from a Qwen2 GGUF file into
    HBM: every tensor is submitted in layer order at once, and the engine's
    construction takes each one as it lands (layer 0 first)."""
    import torch

    from . import _lib
    from .decode import DecodeEngine

    reader = GGUFReader(path)
    cfg = decoder_config(reader, max_pos)
    own = streamer is None
    st = streamer or HBMStreamer(device)
    order = sorted(reader.tensors, key=_layer_order)
    for name in order:
        st.submit(name, reader.raw(name))
    quant = {}
    weights = {}
    for name in order:
        t = reader.tensors[name]
        dev = st.get(name)
        if t.quant in _lib.QUANT_IDS:
            weights[name] = dev
            quant[name] = (t.shape[0], t.shape[1], t.quant)
        elif t.quant == "F32":
            weights[name] = dev.view(torch.float32)
        elif t.quant == "F16":
            weights[name] = dev.view(torch.float16).float()
        else:
            raise ValueError(f"{path}: tensor {name} has type {t.quant}, which the decoder does not take")
    if "lm_head.weight" not in weights:  # tied embeddings
        weights["lm_head.weight"] = weights["model.embed_tokens.weight"]
        if "model.embed_tokens.weight" in quant:
            quant["lm_head.weight"] = quant["model.embed_tokens.weight"]
    torch.cuda.current_stream(torch.device("cuda", device)).synchronize()
    if own:
        st.close()
    reader.close()
    return DecodeEngine(cfg, weights, lambda name: quant.get(name), device=device, **engine_kwargs)


def _layer_order(name: str):
    """Embedding first, then layers in order, then the final norm and head."""
    if name.startswith("model.embed_tokens"):
        return (0, 0, name)
    if name.startswith("model.layers."):
        return (1, int(name.split(".")[2]), name)
    return (2, 0, name)


def _measure(gib: float, path: str) -> dict:
    """Write a synthetic GGUF of `gib` GiB (Q4_K matrices of 18944 x 3584) to
    `path`, then time file -> HBM through the streamer and through one
    pageable copy per tensor (the file is in the page cache after writing)."""
    import json
    import time

    import torch

    rows, cols = 18944, 3584
    nb = rows * (cols // 256) * 144
    count = max(1, int(gib * (1 << 30) // nb))
    rng = np.random.default_rng(0)
    block = rng.integers(0, 256, nb, dtype=np.uint8)
    with open(path, "wb") as f:  # GGUF v3: no metadata, `count` tensors, 32-byte alignment
        head = GGUF_MAGIC + struct.pack("<IQQ", 3, count, 0)
        for i in range(count):
            name = f"blk.{i}.ffn_up.weight".encode()
            head += struct.pack("<Q", len(name)) + name + struct.pack("<I2Q", 2, cols, rows)
            head += struct.pack("<IQ", 12, i * nb)
        head += b"\0" * ((-len(head)) % 32)
        f.write(head)
        for _ in range(count):
            f.write(block.tobytes())
    reader = GGUFReader(path)
    names = list(reader.tensors)
    total = sum(reader.tensors[n].nbytes for n in names)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    st = HBMStreamer(0)
    for n in names:
        st.submit(n, reader.raw(n))
    for n in names:
        st.get(n)
    torch.cuda.synchronize()
    t_stream = time.perf_counter() - t0
    st.close()
    t0 = time.perf_counter()
    devs = [torch.from_numpy(reader.raw(n)).cuda() for n in names]
    torch.cuda.synchronize()
    t_plain = time.perf_counter() - t0
    del devs
    reader.close()
    os.remove(path)
    out = {"bytes": total, "tensors": count, "stream_gbs": round(total / t_stream / 1e9, 2),
           "pageable_copy_gbs": round(total / t_plain / 1e9, 2)}
    print(json.dumps(out))
    return out


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description="file -> HBM throughput of the GGUF streamer")
    ap.add_argument("--measure", type=float, default=4.0, help="GiB of synthetic Q4_K tensors")
    ap.add_argument("--path", default="/tmp/frc_stream_probe.gguf")
    a = ap.parse_args()
    _measure(a.measure, a.path)
