"""Model-level host API: Parameters + InferenceState + Model<int8_t> in one handle.

Mirrors the reference's model loop (src/model/mistral/modules.cpp:154-171)
and CLI loop (main.cpp:69-77) over the C ABI; all buffers handed to the
library here are host numpy arrays.
"""
from __future__ import annotations

import ctypes
import weakref
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import TP_HANDLE_BYTES, check, lib, tl_config, tl_kernel_time, tl_model_options


class Model:
    """A device-resident int8 Mistral model (one GPU).

    ``Model.load(path)`` reads the export_mistral.py binary from disk
    (Parameters::load_parameters, parameters.cpp:95-129); ``Model.from_buffer``
    takes the same bytes from host memory.
    """

    def __init__(self, handle: ctypes.c_void_p, tp_size: int = 1, tp_rank: int = 0):
        self._h = handle
        self._batches = weakref.WeakSet()  # live Batch objects, closed before the model
        self.tp_size, self.tp_rank = max(1, tp_size), tp_rank
        cfg = tl_config()
        check(lib().tl_model_config(self._h, ctypes.byref(cfg)))
        self.config = {f: getattr(cfg, f) for f, _ in tl_config._fields_ if f != "quant"}
        self.config["quant"] = cfg.quant.decode()

    #: kernel_mode values: one persistent kernel per step, or one launch per op
    PERSISTENT, PER_OP = 0, 1

    @staticmethod
    def _opts(device: int, max_seq: int, use_graph: bool, kernel_mode: int, tp_size: int = 1,
              tp_rank: int = 0, sliding_window: int = 0, weights_f16: bool = False):
        return tl_model_options(device=device, max_seq=max_seq, use_graph=1 if use_graph else 0,
                                kernel_mode=kernel_mode, tp_size=tp_size, tp_rank=tp_rank,
                                sliding_window=sliding_window, weights_f16=1 if weights_f16 else 0)

    @classmethod
    def load(cls, path: str, device: int = 0, max_seq: int = 1024, use_graph: bool = True,
             kernel_mode: int = 0, tp_size: int = 1, tp_rank: int = 0, sliding_window: int = 0,
             weights_f16: bool = False) -> "Model":
        """sliding_window: 0 attends to every position (the reference); W > 0 to
        the last W; -1 uses the binary's sliding_window.  weights_f16: the
        batched paths keep fp16 copies of the projections (faster prefill, 2 B
        per parameter) instead of reading the int8 weights in place."""
        h = ctypes.c_void_p()
        o = cls._opts(device, max_seq, use_graph, kernel_mode, tp_size, tp_rank, sliding_window, weights_f16)
        check(lib().tl_model_load(path.encode(), ctypes.byref(o), ctypes.byref(h)))
        return cls(h, tp_size, tp_rank)

    @classmethod
    def from_buffer(cls, buf: np.ndarray, device: int = 0, max_seq: int = 1024,
                    use_graph: bool = True, kernel_mode: int = 0, tp_size: int = 1,
                    tp_rank: int = 0, sliding_window: int = 0, weights_f16: bool = False) -> "Model":
        buf = np.ascontiguousarray(buf)
        h = ctypes.c_void_p()
        o = cls._opts(device, max_seq, use_graph, kernel_mode, tp_size, tp_rank, sliding_window, weights_f16)
        check(lib().tl_model_load_buffer(buf.ctypes.data, buf.nbytes, ctypes.byref(o), ctypes.byref(h)))
        return cls(h, tp_size, tp_rank)

    # ---- tensor parallelism ----
    def tp_handle(self) -> bytes:
        """This rank's exchange-buffer handle (to be gathered by every rank)."""
        buf = (ctypes.c_uint8 * TP_HANDLE_BYTES)()
        check(lib().tl_model_tp_handle(self._h, buf))
        return bytes(buf)

    def tp_connect(self, handles: Sequence[bytes]) -> None:
        """Map every rank's exchange buffer; `handles` in rank order."""
        blob = b"".join(handles)
        if len(handles) != self.tp_size or len(blob) != self.tp_size * TP_HANDLE_BYTES:
            raise ValueError(f"need {self.tp_size} handles of {TP_HANDLE_BYTES} bytes")
        arr = (ctypes.c_uint8 * len(blob)).from_buffer_copy(blob)
        check(lib().tl_model_tp_connect(self._h, arr))

    def close(self) -> None:
        if self._h:
            for b in list(self._batches):  # a model outlives its batches
                b.close()
            check(lib().tl_model_destroy(self._h))
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- InferenceState::pos ----
    @property
    def pos(self) -> int:
        p = ctypes.c_size_t()
        check(lib().tl_model_get_pos(self._h, ctypes.byref(p)))
        return p.value

    @pos.setter
    def pos(self, value: int) -> None:
        check(lib().tl_model_set_pos(self._h, int(value)))

    def set_sampling(self, temperature: float, seed: int = 0) -> None:
        """Decode steps sample at `temperature` (main.cpp:23-43) with the draw of
        position p = ops.sample_uniform(seed, p); temperature <= 0: sample_max."""
        check(lib().tl_model_set_sampling(self._h, float(temperature), int(seed)))

    # ---- Model<T>::forward + sample_max ----
    def forward(self, token: int, logits: bool = True):
        """One token at the current position; returns (logits or None, argmax).
        Under tensor parallelism the logits are this rank's vocabulary slice."""
        out = np.empty(self.config["vocab_size"] // self.tp_size, dtype=np.float32) if logits else None
        nxt = ctypes.c_uint32()
        check(lib().tl_model_forward(self._h, int(token), out.ctypes.data if logits else None,
                                     ctypes.byref(nxt)))
        return out, nxt.value

    def prefill(self, tokens: Sequence[int], logits: bool = True):
        """All of `tokens` in one batched pass at the current position (the
        prompt loop of main.cpp:69-71); returns (last token's logits or None, argmax)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(self.config["vocab_size"] // self.tp_size, dtype=np.float32) if logits else None
        nxt = ctypes.c_uint32()
        check(lib().tl_model_prefill(self._h, t.ctypes.data, t.size, out.ctypes.data if logits else None,
                                     ctypes.byref(nxt)))
        return out, nxt.value

    def time_prefill(self, tokens: Sequence[int]):
        """(device ms of a prefill of `tokens`, argmax of the last token)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        ms = ctypes.c_float()
        nxt = ctypes.c_uint32()
        check(lib().tl_model_time_prefill(self._h, t.ctypes.data, t.size, ctypes.byref(nxt), ctypes.byref(ms)))
        return ms.value, nxt.value

    def generate(self, prompt: Sequence[int], n_new: int) -> List[int]:
        """main.cpp:69-77 on the device: returns the n_new greedy ids."""
        p = np.ascontiguousarray(prompt, dtype=np.uint32)
        out = np.empty(n_new, dtype=np.uint32)
        check(lib().tl_model_generate(self._h, p.ctypes.data, p.size, n_new, out.ctypes.data))
        return out.tolist()

    def layer_forward(self, layer: int, hidden: np.ndarray) -> np.ndarray:
        """Layer<T>::forward on a host hidden state at the current position."""
        h = np.array(hidden, dtype=np.float32, copy=True)
        check(lib().tl_model_layer_forward(self._h, int(layer), h.ctypes.data))
        return h

    def read_kv(self, layer: int, pos: int):
        """K and V rows at `pos` (this rank's kv heads under tensor parallelism)."""
        c = self.config
        kv = c["n_kv_heads"] // self.tp_size
        k = np.empty(kv * c["head_dim"], dtype=np.float32)
        v = np.empty_like(k)
        check(lib().tl_model_read_kv(self._h, int(layer), int(pos), k.ctypes.data, v.ctypes.data))
        return k.reshape(kv, c["head_dim"]), v.reshape(kv, c["head_dim"])

    # ---- measurement ----
    def time_decode(self, token: int, n: int):
        """(device ms for n greedy steps, generated ids)."""
        out = np.empty(n, dtype=np.uint32)
        ms = ctypes.c_float()
        check(lib().tl_model_time_decode(self._h, int(token), n, out.ctypes.data, ctypes.byref(ms)))
        return ms.value, out.tolist()

    def profile(self, token: int, n: int) -> List[Dict]:
        kinds = (tl_kernel_time * 32)()
        nk = ctypes.c_int()
        check(lib().tl_model_profile(self._h, int(token), n, kinds, 32, ctypes.byref(nk)))
        return [dict(name=k.name.decode(), launches=k.launches, total_ms=k.total_ms,
                     bytes_per_launch=k.bytes_per_launch) for k in kinds[:nk.value]]

    def trace_step(self, token: int) -> np.ndarray:
        """Phase trace of one persistent decode step: int64 [cta, phase, 8] ns stamps."""
        c = self.config
        n_phases = 5 * c["n_layers"] + 1
        cap = 2 + 1024 * n_phases * 8
        out = np.zeros(cap, dtype=np.uint64)
        n = ctypes.c_size_t()
        check(lib().tl_model_trace_step(self._h, int(token), out.ctypes.data, cap, ctypes.byref(n)))
        grid, phases = int(out[0]), int(out[1])
        return out[2:2 + grid * phases * 8].astype(np.int64).reshape(grid, phases, 8)

    def launches_per_step(self) -> int:
        n = ctypes.c_int()
        check(lib().tl_model_launches_per_step(self._h, ctypes.byref(n)))
        return n.value


class Batch:
    """B independent sequences decoded together on one model's weights
    (tl_batch_*): each sequence has its own KV cache and position."""

    def __init__(self, model: Model, n_seq: int, max_seq: int = 0):
        self.model, self.n_seq = model, n_seq
        h = ctypes.c_void_p()
        check(lib().tl_batch_create(model._h, n_seq, max_seq, ctypes.byref(h)))
        self._h = h
        model._batches.add(self)

    def close(self) -> None:
        if self._h:
            check(lib().tl_batch_destroy(self._h))
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def fill_kv_random(self, seed: int, n_pos: int) -> None:
        check(lib().tl_batch_fill_kv_random(self._h, seed, n_pos))

    def step(self, tokens: Sequence[int], logits: bool = True):
        """One token per sequence; returns (logits [B, V] or None, next tokens [B])."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        v = self.model.config["vocab_size"] // self.model.tp_size  # this rank's vocabulary slice
        out = np.empty((self.n_seq, v), dtype=np.float32) if logits else None
        nxt = np.empty(self.n_seq, dtype=np.uint32)
        check(lib().tl_batch_step(self._h, t.ctypes.data, out.ctypes.data if logits else None, nxt.ctypes.data))
        return out, nxt

    def time_decode(self, tokens: Sequence[int], n_steps: int):
        """(device ms for n_steps greedy steps of every sequence, ids [n_steps, B])."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty((n_steps, self.n_seq), dtype=np.uint32)
        ms = ctypes.c_float()
        check(lib().tl_batch_time_decode(self._h, t.ctypes.data, n_steps, out.ctypes.data, ctypes.byref(ms)))
        return ms.value, out

    def read_kv(self, seq: int, layer: int, pos: int):
        """K and V rows of one sequence at `pos` (this rank's kv heads under tensor parallelism)."""
        c = self.model.config
        kv = c["n_kv_heads"] // self.model.tp_size
        k = np.empty(kv * c["head_dim"], dtype=np.float32)
        v = np.empty_like(k)
        check(lib().tl_batch_read_kv(self._h, seq, layer, pos, k.ctypes.data, v.ctypes.data))
        return k.reshape(kv, c["head_dim"]), v.reshape(kv, c["head_dim"])

    def tp_handle(self) -> bytes:
        """This rank's exchange-buffer handle (tensor parallelism)."""
        from . import TP_HANDLE_BYTES
        buf = ctypes.create_string_buffer(TP_HANDLE_BYTES)
        check(lib().tl_batch_tp_handle(self._h, buf))
        return buf.raw

    def tp_connect(self, handles: Sequence[bytes]) -> None:
        """Maps every other rank's exchange buffer (handles in rank order)."""
        from . import TP_HANDLE_BYTES
        blob = b"".join(handles)
        assert len(blob) == TP_HANDLE_BYTES * len(handles)
        check(lib().tl_batch_tp_connect(self._h, blob))
