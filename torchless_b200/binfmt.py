"""The torchless model binary: reader, writer and int8 quantiser.

Layout (export_mistral.py:33-46, 143-180 of the reference):

    [u64 little-endian H] [H bytes: UTF-8 JSON header, zero padded so that
    8 + H is a multiple of 64] [payload]

The JSON header has ``metadata`` (model hyper-parameters as strings,
export_mistral.py:70-88), ``tensors`` (name -> dtype, shape, offset and, for
int8, scale_offset / scale_size, export_mistral.py:107-135) and
``tokenizer`` (vocab + merges, export_mistral.py:90-98).  Offsets are
relative to the payload start and every tensor and scale block starts on a
64-byte boundary (pad_to_64, export_mistral.py:100-105).

Quantisation (export_mistral.py:53-68): per group of 64 consecutive elements
of a ``*_proj`` tensor, ``scale = 127 / max|x|`` and
``q = round_half_even(x * scale)`` as int8; the scale is stored, and the
engine dequantises with ``q / scale`` (src/common/tensor.cpp:101-104).
``int_max / tensor`` in torch evaluates as ``reciprocal(tensor) * int_max``
(two fp32 roundings, not one division), and that is what is restated here.

This module writes byte-identical files to the reference exporter for the
same fp32 inputs and tensor order (checked by tests/golden/make_golden.py
against export_mistral.py itself).

fp8 (format extension; the reference's roadmap item "Support fp8 with a cast
``tensor.to(torch.float8_e5m2)`` during model export", README.md:160): with
``quant = "fp8"`` every ``*_proj`` tensor is that cast, one byte per element
(the e5m2 bit pattern: sign, 5 exponent bits with bias 15, 2 mantissa bits),
dtype ``"fp8"`` in the header, no scales, each block padded to 64.  The
engine's weight is the e5m2 value itself.
"""
from __future__ import annotations

import json
import struct
from dataclasses import dataclass, field
from typing import Dict, Iterable, List, Optional, Tuple

import numpy as np

GROUP_SIZE = 64  # export_mistral.py:194
QUANTS = ("f32", "int8", "fp8")  # export_mistral.py:187 accepts f32 and int8; fp8 is the extension


def pad_to_64(offset: int) -> int:
    """Bytes needed to bring ``offset`` to a multiple of 64 (export_mistral.py:100-105)."""
    r = offset % 64
    return 0 if r == 0 else 64 - r


def quantize_i8(x: np.ndarray, group: int = GROUP_SIZE) -> Tuple[np.ndarray, np.ndarray]:
    """Per-group symmetric int8 quantisation with fp32 arithmetic.

    Restates export_mistral.py:53-68 (torch CPU) in numpy: fp32 absmax,
    ``fl(fl(1 / absmax) * 127)`` (torch's reverse true-divide by a tensor),
    fp32 product, round-half-to-even, cast to int8.
    Returns ``(q, scales)`` with ``q`` shaped like ``x`` and ``scales`` of
    length ``x.size // group``.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.size % group:
        raise ValueError(f"numel {x.size} is not a multiple of the group size {group}")
    g = x.reshape(-1, group)
    amax = np.abs(g).max(axis=1)
    with np.errstate(divide="ignore"):
        scales = ((np.float32(1.0) / amax).astype(np.float32) * np.float32(127.0)).astype(np.float32)
    q = np.rint(g * scales[:, None]).astype(np.int8)
    return q.reshape(x.shape), scales


def quantize_fp8(x: np.ndarray) -> np.ndarray:
    """The fp8 export: ``x.to(torch.float8_e5m2)`` (round to nearest even; values
    beyond the e5m2 range become infinities), returned as the uint8 bit
    patterns, shaped like ``x``."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    return t.to(torch.float8_e5m2).view(torch.uint8).numpy().copy()


def fp8_to_f32(b: np.ndarray) -> np.ndarray:
    """e5m2 bit patterns to fp32, exactly: an e5m2 byte is the high byte of the
    IEEE half with the same value (same sign, exponent width and bias)."""
    return (np.asarray(b, dtype=np.uint8).astype(np.uint16) << 8).view(np.float16).astype(np.float32)


@dataclass
class TensorInfo:
    name: str
    dtype: str            # "f32", "int8" or "fp8"
    shape: List[int]
    offset: int
    scale_offset: Optional[int] = None
    scale_size: Optional[int] = None

    @property
    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n


@dataclass
class Config:
    """Parameters::load_config (src/loader/parameters.cpp:32-47)."""
    hidden_size: int
    intermediate_size: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    vocab_size: int
    sliding_window: int
    rope_theta: float
    norm_eps: float
    max_position_embeddings: int
    quant: str
    head_dim: int = field(init=False)

    def __post_init__(self):
        self.head_dim = self.hidden_size // self.n_heads  # parameters.cpp:45

    @classmethod
    def from_metadata(cls, m: dict) -> "Config":
        # std::stoi / std::stof of the metadata strings.
        return cls(
            hidden_size=int(m["hidden_size"]),
            intermediate_size=int(m["intermediate_size"]),
            n_layers=int(m["n_layers"]),
            n_heads=int(m["n_heads"]),
            n_kv_heads=int(m["n_kv_heads"]),
            vocab_size=int(m["vocab_size"]),
            sliding_window=int(m["sliding_window"]),
            rope_theta=float(np.float32(float(m["rope_theta"]))),
            norm_eps=float(np.float32(float(m["norm_eps"]))),
            max_position_embeddings=int(m["max_position_embeddings"]),
            quant=str(m["quant"]),
        )


class ModelFile:
    """A parsed model binary held in memory (bytes, bytearray, numpy or mmap).

    ``tensor(name)`` returns numpy views into the payload, like the
    reference's Tensor views into its mmap (parameters.cpp:49-68).
    """

    def __init__(self, buf):
        self.buf = np.frombuffer(buf, dtype=np.uint8) if not isinstance(buf, np.ndarray) else buf
        if self.buf.size < 8:
            raise ValueError("model binary shorter than its 8-byte header length")
        (hsize,) = struct.unpack("<Q", self.buf[:8].tobytes())
        if 8 + hsize > self.buf.size:
            raise ValueError("model binary header length exceeds the file")
        raw = self.buf[8:8 + hsize].tobytes().rstrip(b"\x00")
        self.header = json.loads(raw.decode("utf-8"))
        self.header_size = hsize
        self.payload_offset = 8 + hsize
        self.config = Config.from_metadata(self.header["metadata"])
        self.tensors: Dict[str, TensorInfo] = {}
        for name, v in self.header["tensors"].items():
            self.tensors[name] = TensorInfo(name, v["dtype"], list(v["shape"]), int(v["offset"]),
                                            v.get("scale_offset"), v.get("scale_size"))

    @classmethod
    def open(cls, path: str) -> "ModelFile":
        return cls(np.memmap(path, dtype=np.uint8, mode="r"))

    def _slice(self, offset: int, nbytes: int) -> np.ndarray:
        start = self.payload_offset + offset
        if start + nbytes > self.buf.size:
            raise ValueError("tensor extends past the end of the model binary")
        return self.buf[start:start + nbytes]

    def tensor(self, name: str):
        """(data, scales-or-None) as numpy views; data shaped like the tensor:
        float32 (f32), int8 with fp32 scales (int8), or uint8 e5m2 bit
        patterns without scales (fp8)."""
        t = self.tensors[name]
        if t.dtype == "f32":
            return self._slice(t.offset, 4 * t.numel).view(np.float32).reshape(t.shape), None
        if t.dtype == "int8":
            q = self._slice(t.offset, t.numel).view(np.int8).reshape(t.shape)
            s = self._slice(t.scale_offset, 4 * t.scale_size).view(np.float32)
            return q, s
        if t.dtype == "fp8":
            return self._slice(t.offset, t.numel).reshape(t.shape), None
        raise ValueError(f"unknown dtype {t.dtype!r} for {name}")

    def layer_tensor(self, layer: int, name: str):
        return self.tensor(f"model.layers.{layer}.{name}")


LM_HEAD = "lm_head.weight"


def build_header(metadata: dict, tensors: Iterable[Tuple[str, Tuple[int, ...]]], quant: str,
                 tokenizer: dict, quant_lm_head: bool = False) -> Tuple[dict, int]:
    """The header dict and payload size for tensors in the given order.

    Offsets follow load_tensor_map (export_mistral.py:107-135): int8 only for
    names containing "_proj" when quant != "f32", each block padded to 64.
    quant_lm_head (a format extension; the reference exporter keeps the
    lm_head fp32, export_mistral.py:119) also stores ``lm_head.weight`` in the
    ``_proj`` tensors' format (int8 + per-64-group scales, or fp8): its dtype
    entry in the header is what tells a loader.  quant "fp8" stores one e5m2
    byte per element and no scales.
    """
    if quant not in QUANTS:
        raise ValueError(f"quant {quant!r} not in {QUANTS}")
    header = {"metadata": dict(metadata), "tensors": {}}
    start = 0
    for name, shape in tensors:
        numel = int(np.prod(shape))
        if quant != "f32" and ("_proj" in name or (quant_lm_head and name == LM_HEAD)):
            entry = {"dtype": quant, "shape": list(shape)[:4], "offset": start}
            start += numel
            start += pad_to_64(start)
            if quant == "int8":
                entry["scale_offset"] = start
                entry["scale_size"] = numel // GROUP_SIZE
                start += numel // GROUP_SIZE * 4
                start += pad_to_64(start)
        else:
            entry = {"dtype": "f32", "shape": list(shape)[:4], "offset": start}
            start += numel * 4
            start += pad_to_64(start)
        header["tensors"][name] = entry
    header["tokenizer"] = tokenizer
    return header, start


def metadata_from_hf(cfg: dict, quant: str) -> dict:
    """load_config (export_mistral.py:70-88): HF config.json -> string metadata."""
    return {
        "hidden_size": str(cfg["hidden_size"]),
        "intermediate_size": str(cfg["intermediate_size"]),
        "n_layers": str(cfg["num_hidden_layers"]),
        "n_heads": str(cfg["num_attention_heads"]),
        "n_kv_heads": str(cfg["num_key_value_heads"]),
        "vocab_size": str(cfg["vocab_size"]),
        "max_position_embeddings": str(cfg["max_position_embeddings"]),
        "sliding_window": str(cfg["sliding_window"]),
        "rope_theta": str(cfg["rope_theta"]),
        "norm_eps": str(cfg["rms_norm_eps"]),
        "act_type": cfg["hidden_act"],
        "quant": str(quant),
    }


class BinWriter:
    """Assembles a model binary in one contiguous host buffer.

    ``put(name, data, scales)`` copies already-converted bytes (fp32, or int8
    plus fp32 scales) to the offsets ``build_header`` assigned, so producers
    may quantise anywhere (numpy here, or the CUDA quantiser) and only hand
    over the bytes.  Gaps stay zero, like the seeks in write_binary
    (export_mistral.py:143-180).
    """

    def __init__(self, metadata: dict, tensors: List[Tuple[str, Tuple[int, ...]]], quant: str,
                 tokenizer: dict, buffer: Optional[np.ndarray] = None, quant_lm_head: bool = False):
        self.header, payload = build_header(metadata, tensors, quant, tokenizer, quant_lm_head)
        hb = json.dumps(self.header).encode("utf-8")
        pad = pad_to_64(8 + len(hb))
        self.header_size = len(hb) + pad
        self.payload_offset = 8 + self.header_size
        self.size = self.payload_offset + payload
        if buffer is None:
            buffer = np.zeros(self.size, dtype=np.uint8)
        elif buffer.size < self.size:
            raise ValueError("buffer too small")
        self.buf = buffer[: self.size]
        self.buf[:8] = np.frombuffer(struct.pack("<Q", self.header_size), dtype=np.uint8)
        self.buf[8:8 + len(hb)] = np.frombuffer(hb, dtype=np.uint8)
        self.buf[8 + len(hb):self.payload_offset] = 0

    def view(self, name: str):
        """Writable numpy views (data, scales-or-None) for tensor ``name``, typed
        as ModelFile.tensor returns them."""
        e = self.header["tensors"][name]
        numel = int(np.prod(e["shape"]))
        o = self.payload_offset + e["offset"]
        if e["dtype"] == "f32":
            return self.buf[o:o + 4 * numel].view(np.float32).reshape(e["shape"]), None
        if e["dtype"] == "fp8":
            return self.buf[o:o + numel].reshape(e["shape"]), None
        q = self.buf[o:o + numel].view(np.int8).reshape(e["shape"])
        so = self.payload_offset + e["scale_offset"]
        s = self.buf[so:so + 4 * e["scale_size"]].view(np.float32)
        return q, s

    def put_fp32(self, name: str, x: np.ndarray) -> None:
        """Store an fp32 source tensor, quantising it when the header says int8
        or casting it when it says fp8."""
        d, s = self.view(name)
        if d.dtype == np.uint8:
            d[...] = quantize_fp8(np.asarray(x, dtype=np.float32).reshape(d.shape))
        elif s is None:
            d[...] = np.asarray(x, dtype=np.float32).reshape(d.shape)
        else:
            q, sc = quantize_i8(np.asarray(x, dtype=np.float32).reshape(d.shape))
            d[...] = q
            s[...] = sc

    def tobytes(self) -> bytes:
        return self.buf.tobytes()

    def save(self, path: str) -> None:
        with open(path, "wb") as f:
            f.write(memoryview(self.buf))
