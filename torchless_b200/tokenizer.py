"""The model binary's BPE tokenizer (tl_tokenizer_*, tokenizer.cpp restated in
C++): encode text to ids (BOS first) and decode ids to text, as main.cpp does
around its generation loop (main.cpp:60-77)."""
from __future__ import annotations

import ctypes
import json
from typing import List, Sequence

import numpy as np

from . import check, lib


class Tokenizer:
    def __init__(self, handle: ctypes.c_void_p):
        self._h = handle

    @classmethod
    def load(cls, path: str) -> "Tokenizer":
        """From a model binary on disk (its header only is read)."""
        h = ctypes.c_void_p()
        check(lib().tl_tokenizer_load(path.encode(), ctypes.byref(h)))
        return cls(h)

    @classmethod
    def from_buffer(cls, buf: np.ndarray) -> "Tokenizer":
        """From a model binary in host memory."""
        b = np.ascontiguousarray(buf)
        h = ctypes.c_void_p()
        check(lib().tl_tokenizer_load_buffer(b.ctypes.data, b.nbytes, ctypes.byref(h)))
        return cls(h)

    @classmethod
    def from_json(cls, tok) -> "Tokenizer":
        """From the tokenizer object ({"vocab": ..., "merges": ...}, a dict or its JSON text)."""
        text = (tok if isinstance(tok, str) else json.dumps(tok)).encode("utf-8")
        h = ctypes.c_void_p()
        check(lib().tl_tokenizer_load_json(text, len(text), ctypes.byref(h)))
        return cls(h)

    def close(self) -> None:
        if self._h:
            check(lib().tl_tokenizer_destroy(self._h))
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def vocab_size(self) -> int:
        n = ctypes.c_size_t()
        check(lib().tl_tokenizer_vocab_size(self._h, ctypes.byref(n)))
        return n.value

    def encode(self, text) -> List[int]:
        """Tokenizer::encode: ids with <s> first.  `text`: str (UTF-8) or bytes."""
        b = text.encode("utf-8") if isinstance(text, str) else bytes(text)
        cap = 2 * len(b) + 8  # at most one id per byte, plus BOS
        ids = np.empty(cap, dtype=np.uint32)
        n = ctypes.c_size_t()
        check(lib().tl_tokenizer_encode(self._h, b, len(b), ids.ctypes.data, cap, ctypes.byref(n)))
        return ids[:n.value].tolist()

    def decode_bytes(self, ids: Sequence[int]) -> bytes:
        """Tokenizer::decode as raw bytes (pieces may split UTF-8 sequences)."""
        a = np.ascontiguousarray(ids, dtype=np.uint32)
        n = ctypes.c_size_t()
        cap = 64 + 32 * len(a)
        for _ in range(2):
            out = ctypes.create_string_buffer(cap)
            st = lib().tl_tokenizer_decode(self._h, a.ctypes.data, a.size, out, cap, ctypes.byref(n))
            if st == 0:
                return out.raw[:n.value]
            cap = n.value + 1  # TL_ERR_CAPACITY reports the size needed
        check(st)
        return b""

    def decode(self, ids: Sequence[int]) -> str:
        return self.decode_bytes(ids).decode("utf-8", errors="replace")
