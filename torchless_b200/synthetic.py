"""Seeded random-init Mistral-architecture models in the torchless binary format.

Stands in for the Hugging Face checkpoint that export_mistral.py consumes:
every ``*_proj`` matrix, the embedding and the lm_head are drawn from
N(0, std) (std 0.02 by default) with a fixed seed; norm weights are 1.0
(``norm="ones"``) or 1 + N(0, 0.1) (``norm="random"``, used by the parity
tests so the norm gain is exercised).  Tensor names and shapes follow the HF
Mistral checkpoint that the reference loads (src/model/mistral/modules.h:77-116).

Three generators produce the same layout:
  * ``numpy`` (one PCG64 stream): small models, and the HF directory that
    tests/golden/make_golden.py feeds to the reference's own exporter;
  * ``seeded`` (PCG64 streams per row block, host threads): the Mistral-7B
    workload model of the benchmarks and of the full-depth parity fixture,
    identical bytes on every host (about 20 s on 8 cores);
  * ``torch`` on a device (CUDA when present): Mistral-7B sized models in a few
    seconds, quantised on the device by the library's own quantiser.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Iterator, List, Optional, Tuple

import numpy as np

from .binfmt import BinWriter, metadata_from_hf, quantize_fp8, quantize_i8

# Mistral-7B-v0.1 architecture (the reference's target model).
MISTRAL_7B = dict(
    hidden_size=4096, intermediate_size=14336, num_hidden_layers=32, num_attention_heads=32,
    num_key_value_heads=8, vocab_size=32000, max_position_embeddings=32768, sliding_window=4096,
    rope_theta=10000.0, rms_norm_eps=1e-05, hidden_act="silu",
)

# Small models with the same structure for parity tests that the CPU oracle
# finishes in well under a second per token.  The reference hard-codes the
# GQA ratio n_heads / n_kv_heads = 4 (modules.cpp:70), so every config keeps it.
SMALL = dict(
    hidden_size=1024, intermediate_size=2048, num_hidden_layers=2, num_attention_heads=8,
    num_key_value_heads=2, vocab_size=1000, max_position_embeddings=4096, sliding_window=4096,
    rope_theta=10000.0, rms_norm_eps=1e-05, hidden_act="silu",
)
TINY = dict(
    hidden_size=512, intermediate_size=1536, num_hidden_layers=2, num_attention_heads=4,
    num_key_value_heads=1, vocab_size=777, max_position_embeddings=4096, sliding_window=4096,
    rope_theta=10000.0, rms_norm_eps=1e-05, hidden_act="silu",
)

PLACEHOLDER_TOKENIZER = {"vocab": {"<unk>": 0, "<s>": 1, "</s>": 2}, "merges": []}


def tensor_list(cfg: dict) -> List[Tuple[str, Tuple[int, ...]]]:
    """HF Mistral tensor names and shapes, in the order written to the binary."""
    D, F = cfg["hidden_size"], cfg["intermediate_size"]
    H, KV = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    hd = D // H
    out = [("model.embed_tokens.weight", (cfg["vocab_size"], D))]
    for l in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{l}."
        out += [
            (p + "input_layernorm.weight", (D,)),
            (p + "self_attn.q_proj.weight", (H * hd, D)),
            (p + "self_attn.k_proj.weight", (KV * hd, D)),
            (p + "self_attn.v_proj.weight", (KV * hd, D)),
            (p + "self_attn.o_proj.weight", (D, H * hd)),
            (p + "post_attention_layernorm.weight", (D,)),
            (p + "mlp.gate_proj.weight", (F, D)),
            (p + "mlp.up_proj.weight", (F, D)),
            (p + "mlp.down_proj.weight", (D, F)),
        ]
    out += [("model.norm.weight", (D,)), ("lm_head.weight", (cfg["vocab_size"], D))]
    return out


def _is_norm(name: str) -> bool:
    return name.endswith("norm.weight")


def numpy_tensors(cfg: dict, seed: int, std: float = 0.02,
                  norm: str = "ones") -> Iterator[Tuple[str, np.ndarray]]:
    """fp32 source tensors from one PCG64 stream, in ``tensor_list`` order."""
    rng = np.random.Generator(np.random.PCG64(seed))
    for name, shape in tensor_list(cfg):
        if _is_norm(name):
            if norm == "ones":
                x = np.ones(shape, dtype=np.float32)
            else:
                x = (1.0 + 0.1 * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32)
        else:
            x = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
        yield name, x


META = "\u2581"  # the Metaspace marker of Mistral's pre-tokeniser

# A short text for training the synthetic BPE tokenizer (plain prose written
# for this purpose, with a few accented, CJK and emoji characters so that the
# UTF-8 and byte-fallback paths are exercised).
TOKENIZER_CORPUS = (
    "the model reads its weights once from the binary file and keeps them resident in memory. "
    "every decode step reads the weights again, so the speed of a step is set by memory bandwidth. "
    "a prompt is split into pieces by the tokenizer, and each piece becomes one id in the vocabulary. "
    "the pieces are merged pair by pair, the lowest ranked pair first, until no pair can be merged. "
    "caf\u00e9 na\u00efve r\u00e9sum\u00e9 \u4e2d\u6587 \u6587\u5b57 \U0001F600 tokens and the tokenizer again. "
)


def make_bpe_tokenizer(corpus: str = TOKENIZER_CORPUS, n_merges: int = 200) -> dict:
    """A small Mistral-style BPE tokenizer object {vocab, merges}: <unk>, <s>,
    </s>, the 256 byte pieces <0xXX>, the corpus's characters after Metaspace
    pre-tokenisation, then `n_merges` merges of the most frequent adjacent
    pair (ties: the pair seen first), trained over the whole text the way
    tokenizer.cpp applies them."""
    vocab = {"<unk>": 0, "<s>": 1, "</s>": 2}
    for b in range(256):
        vocab[f"<0x{b:02X}>"] = len(vocab)
    text = META + corpus.replace(" ", META)
    seq = list(text)
    for ch in seq:
        if ch not in vocab:
            vocab[ch] = len(vocab)
    merges = []
    for _ in range(n_merges):
        counts, first = {}, {}
        for i in range(len(seq) - 1):
            p = (seq[i], seq[i + 1])
            counts[p] = counts.get(p, 0) + 1
            first.setdefault(p, i)
        if not counts:
            break
        best = max(counts, key=lambda p: (counts[p], -first[p]))
        if counts[best] < 2:
            break
        a, b = best
        merges.append(f"{a} {b}")
        if a + b not in vocab:
            vocab[a + b] = len(vocab)
        out, i = [], 0
        while i < len(seq):
            if i + 1 < len(seq) and seq[i] == a and seq[i + 1] == b:
                out.append(a + b)
                i += 2
            else:
                out.append(seq[i])
                i += 1
        seq = out
    return {"vocab": vocab, "merges": merges}


def make_numpy_model(cfg: dict, seed: int, quant: str = "int8", std: float = 0.02,
                     norm: str = "ones", quant_lm_head: bool = False, tokenizer: Optional[dict] = None) -> BinWriter:
    """A complete model binary built on the CPU (small configs).  quant: "int8",
    "fp8" (the e5m2 cast) or "f32"; quant_lm_head: the lm_head stored in the
    projections' format too (format extension, see binfmt.build_header);
    tokenizer: the header's tokenizer object (default: a 3-piece placeholder)."""
    w = BinWriter(metadata_from_hf(cfg, quant), tensor_list(cfg), quant, tokenizer or PLACEHOLDER_TOKENIZER,
                  quant_lm_head=quant_lm_head)
    for name, x in numpy_tensors(cfg, seed, std, norm):
        w.put_fp32(name, x)
    return w


# Seeded chunks: the unit of the parallel generator below.  Tensor t of
# ``tensor_list`` is cut into blocks of whole rows of about CHUNK_ELEMS
# elements; block c of tensor t draws from its own PCG64 stream keyed by
# SeedSequence([seed, t, c]).  The blocks are fixed by the shapes alone, so
# the bytes do not depend on the thread count or the machine (numpy's PCG64
# and ziggurat normal sampler are platform-independent).  Quantisation
# groups (64 along a row) never straddle a block.
CHUNK_ELEMS = 1 << 22


def _chunks(cfg: dict):
    for t, (name, shape) in enumerate(tensor_list(cfg)):
        if _is_norm(name):
            yield t, 0, name, shape, 0, shape[0]
            continue
        rows, cols = shape
        per = max(1, CHUNK_ELEMS // cols)
        for c, r0 in enumerate(range(0, rows, per)):
            yield t, c, name, shape, r0, min(rows, r0 + per)


def make_seeded_model(cfg: dict, seed: int, quant: str = "int8", std: float = 0.02,
                      quant_lm_head: bool = False, threads: Optional[int] = None,
                      buffer: Optional[np.ndarray] = None) -> BinWriter:
    """A complete model binary built on the host CPU, in parallel, from seeded
    row blocks (CHUNK_ELEMS above): every ``*_proj`` matrix, the embedding and
    the lm_head ~ N(0, std), norm weights 1.0; quantised by ``quantize_i8``
    (the export_mistral.py arithmetic) or cast to e5m2 for quant "fp8".

    This is the workload model of the Mistral-7B benchmarks and of the
    full-depth parity fixture: the same seed gives the same bytes on any
    host, so the CPU checkers and the GPU load the identical binary."""
    from concurrent.futures import ThreadPoolExecutor

    w = BinWriter(metadata_from_hf(cfg, quant), tensor_list(cfg), quant, PLACEHOLDER_TOKENIZER,
                  buffer=buffer, quant_lm_head=quant_lm_head)

    def job(item):
        t, c, name, shape, r0, r1 = item
        d, s = w.view(name)
        if _is_norm(name):
            d[...] = 1.0
            return
        rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, t, c])))
        x = rng.standard_normal((r1 - r0, shape[1]), dtype=np.float32)
        x *= np.float32(std)
        if d.dtype == np.uint8:
            d[r0:r1] = quantize_fp8(x)
        elif s is None:
            d[r0:r1] = x
        else:
            q, sc = quantize_i8(x)
            d[r0:r1] = q
            g = shape[1] // 64
            s[r0 * g:r1 * g] = sc

    with ThreadPoolExecutor(threads or os.cpu_count() or 1) as ex:
        for _ in ex.map(job, list(_chunks(cfg))):
            pass
    return w


def model_digest(buf: np.ndarray, stride: int = 1 << 20, block: int = 4096) -> str:
    """sha256 of the header and of one `block`-byte window every `stride` bytes
    of a model binary: a quick fingerprint that tells two multi-GB binaries
    apart without hashing all of them."""
    import hashlib
    import struct

    b = np.ascontiguousarray(buf).view(np.uint8)
    h = hashlib.sha256()
    (hsize,) = struct.unpack("<Q", b[:8].tobytes())
    h.update(b[:8 + hsize].tobytes())
    h.update(str(b.size).encode())
    for o in range(8 + hsize, b.size, stride):
        h.update(b[o:o + block].tobytes())
    return h.hexdigest()


def make_torch_model(cfg: dict, seed: int, quant: str = "int8", std: float = 0.02,
                     norm: str = "ones", device: str = "cuda", quantizer=None,
                     buffer: Optional[np.ndarray] = None, quant_lm_head: bool = False) -> BinWriter:
    """A complete model binary whose random draws happen on ``device``.

    ``quantizer(x_device) -> (q_device, scales_device)`` quantises on the
    device (the CUDA quantiser of this library); without it the fp32 tensor
    is copied to the host and quantised by ``quantize_i8``.
    """
    import torch

    w = BinWriter(metadata_from_hf(cfg, quant), tensor_list(cfg), quant, PLACEHOLDER_TOKENIZER,
                  buffer=buffer, quant_lm_head=quant_lm_head)
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    for name, shape in tensor_list(cfg):
        if _is_norm(name):
            if norm == "ones":
                x = torch.ones(shape, dtype=torch.float32, device=device)
            else:
                x = 1.0 + 0.1 * torch.randn(shape, generator=g, dtype=torch.float32, device=device)
        else:
            x = torch.randn(shape, generator=g, dtype=torch.float32, device=device) * std
        d, s = w.view(name)
        if d.dtype == np.uint8:  # fp8 export: the e5m2 cast, on the device
            d[...] = x.to(torch.float8_e5m2).view(torch.uint8).cpu().numpy()
        elif s is None:
            d[...] = x.cpu().numpy()
        elif quantizer is not None:
            q, sc = quantizer(x)
            d[...] = q.cpu().numpy().reshape(d.shape)
            s[...] = sc.cpu().numpy()
        else:
            q, sc = quantize_i8(x.cpu().numpy())
            d[...] = q
            s[...] = sc
        del x
    return w


def write_hf_dir(path: str, cfg: dict, tensors: Dict[str, np.ndarray],
                 tokenizer: dict = PLACEHOLDER_TOKENIZER) -> None:
    """An HF-style model directory (fp32 safetensors) for export_mistral.py."""
    from safetensors.numpy import save_file

    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)
    with open(os.path.join(path, "tokenizer.json"), "w") as f:
        json.dump({"model": tokenizer}, f)
    save_file(tensors, os.path.join(path, "model.safetensors"))
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"weight_map": {k: "model.safetensors" for k in tensors}}, f)
