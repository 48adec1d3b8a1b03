"""torchless_b200: the torchless int8 Mistral hot path on B200 (sm_100a).

Python host side over the C ABI in include/torchless_b200.h
(libtorchless_b200.so next to this file).  It mirrors the reference's
interfaces for the path:

* ``ops``            - src/common/kernels.h (matmul, row_matmul, softmax, rope,
                       silu, sum, add, mul, pow, sqrt) plus rmsnorm, rotary,
                       argmax (sample_max), the fused gate/up and the quantiser,
                       on CUDA tensors;
* ``Model``          - Parameters::load_parameters + InferenceState +
                       Model<int8_t>::forward (src/loader, src/model/mistral),
                       device resident;
* ``binfmt``/``synthetic`` - the export_mistral.py file format and seeded
                       random-init models.

There is no CPU fallback: importing works without a GPU, but every call
needs the CUDA library, and a missing library raises at first use.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libtorchless_b200.so")

TL_OK = 0
STATUS = {
    0: "TL_OK", 1: "TL_ERR_INVALID_ARGUMENT", 2: "TL_ERR_UNSUPPORTED", 3: "TL_ERR_IO",
    4: "TL_ERR_FORMAT", 5: "TL_ERR_CUDA", 6: "TL_ERR_OUT_OF_MEMORY", 7: "TL_ERR_CAPACITY",
    8: "TL_ERR_TIMEOUT",
}


class TLError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = status


class tl_config(ctypes.Structure):
    _fields_ = [(n, ctypes.c_size_t) for n in (
        "hidden_size", "intermediate_size", "n_layers", "n_heads", "n_kv_heads", "vocab_size",
        "head_dim", "sliding_window", "max_position_embeddings")] + [
        ("rope_theta", ctypes.c_float), ("norm_eps", ctypes.c_float), ("quant", ctypes.c_char * 16)]


class tl_model_options(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("max_seq", ctypes.c_size_t), ("use_graph", ctypes.c_int),
                ("kernel_mode", ctypes.c_int), ("tp_size", ctypes.c_int), ("tp_rank", ctypes.c_int),
                ("sliding_window", ctypes.c_int), ("weights_f16", ctypes.c_int)]


TP_HANDLE_BYTES = 64


class tl_kernel_time(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 32), ("launches", ctypes.c_int), ("total_ms", ctypes.c_double),
                ("bytes_per_launch", ctypes.c_double)]


_P = ctypes.c_void_p
_S = ctypes.c_size_t
_F = ctypes.c_float
_I = ctypes.c_int
_U32 = ctypes.c_uint32

# name -> argtypes (restype is always tl_status / c_int)
SIGNATURES = {
    "tl_matmul_f32": [_P, _P, _P, _S, _S, _P],
    "tl_matmul_i8": [_P, _P, _P, _S, _P, _S, _S, _P],
    "tl_matmul_f8": [_P, _P, _P, _S, _S, _P],
    "tl_row_matmul": [_P, _P, _P, _S, _S, _P],
    "tl_softmax": [_P, _P, _S, _P],
    "tl_rope": [_P, _P, _P, _P, _S, _S, _P],
    "tl_silu": [_P, _P, _S, _P],
    "tl_sum": [_P, _P, _S, _P],
    "tl_add": [_P, _P, _P, _S, _P],
    "tl_add_scalar": [_P, _P, _F, _S, _P],
    "tl_mul": [_P, _P, _P, _S, _P],
    "tl_mul_scalar": [_P, _P, _F, _S, _P],
    "tl_pow": [_P, _P, _I, _S, _P],
    "tl_sqrt": [_P, _P, _S, _P],
    "tl_rmsnorm": [_P, _P, _P, _S, _F, _P],
    "tl_rotary": [_P, _P, _P, _S, _S, _S, _P],
    "tl_argmax": [_P, _P, _S, _P],
    "tl_argmax_noalloc": [_P, _P, _S, _P],
    "tl_sample_multinomial": [_P, _P, _S, _F, _F, _P],
    "tl_sample_uniform": [ctypes.c_uint64, ctypes.c_uint64],  # returns float (set below)
    "tl_model_set_sampling": [_P, _F, ctypes.c_uint64],
    "tl_mlp_gate_up": [_P, _P, _P, _P, _P, _P, _S, _S, _P],
    "tl_quantize_i8": [_P, _P, _P, _S, _S, _P],
    "tl_gemm_f16": [_P, _P, _P, _S, _S, _S, _S, _I, _P],
    "tl_gemm_q8": [_P, _P, _P, _P, _P, _P, _S, _S, _S, _S, _I, _P],
    "tl_model_load": [ctypes.c_char_p, ctypes.POINTER(tl_model_options), ctypes.POINTER(_P)],
    "tl_model_load_buffer": [_P, _S, ctypes.POINTER(tl_model_options), ctypes.POINTER(_P)],
    "tl_model_destroy": [_P],
    "tl_model_config": [_P, ctypes.POINTER(tl_config)],
    "tl_model_forward": [_P, _U32, _P, _P],
    "tl_model_generate": [_P, _P, _S, _S, _P],
    "tl_model_prefill": [_P, _P, _S, _P, _P],
    "tl_model_time_prefill": [_P, _P, _S, _P, ctypes.POINTER(_F)],
    "tl_model_get_pos": [_P, ctypes.POINTER(_S)],
    "tl_model_set_pos": [_P, _S],
    "tl_model_layer_forward": [_P, _I, _P],
    "tl_model_read_kv": [_P, _I, _S, _P, _P],
    "tl_model_time_decode": [_P, _U32, _S, _P, ctypes.POINTER(_F)],
    "tl_model_profile": [_P, _U32, _S, ctypes.POINTER(tl_kernel_time), _I, ctypes.POINTER(_I)],
    "tl_model_launches_per_step": [_P, ctypes.POINTER(_I)],
    "tl_model_trace_step": [_P, _U32, _P, _S, ctypes.POINTER(_S)],
    "tl_batch_create": [_P, _I, _S, ctypes.POINTER(_P)],
    "tl_batch_destroy": [_P],
    "tl_batch_fill_kv_random": [_P, ctypes.c_uint64, _S],
    "tl_batch_step": [_P, _P, _P, _P],
    "tl_batch_time_decode": [_P, _P, _S, _P, ctypes.POINTER(_F)],
    "tl_batch_read_kv": [_P, _I, _I, _S, _P, _P],
    "tl_batch_tp_handle": [_P, _P],
    "tl_batch_tp_connect": [_P, _P],
    "tl_tokenizer_load": [ctypes.c_char_p, ctypes.POINTER(_P)],
    "tl_tokenizer_load_buffer": [_P, _S, ctypes.POINTER(_P)],
    "tl_tokenizer_load_json": [ctypes.c_char_p, _S, ctypes.POINTER(_P)],
    "tl_tokenizer_destroy": [_P],
    "tl_tokenizer_vocab_size": [_P, ctypes.POINTER(_S)],
    "tl_tokenizer_encode": [_P, ctypes.c_char_p, _S, _P, _S, ctypes.POINTER(_S)],
    "tl_tokenizer_decode": [_P, _P, _S, _P, _S, ctypes.POINTER(_S)],
    "tl_model_tp_handle": [_P, _P],
    "tl_model_tp_connect": [_P, _P],
}

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """The CUDA library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run `python -m torchless_b200.build` "
                               "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = ctypes.c_int
        L.tl_last_error.restype = ctypes.c_char_p
        L.tl_last_error.argtypes = []
        L.tl_sample_uniform.restype = ctypes.c_float
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != TL_OK:
        raise TLError(status, lib().tl_last_error().decode(errors="replace"))


from . import ops  # noqa: E402  (needs lib/check)
from .model import Batch, Model  # noqa: E402
from .tokenizer import Tokenizer  # noqa: E402

__all__ = ["lib", "check", "TLError", "ops", "Model", "Batch", "Tokenizer", "LIB_PATH", "SIGNATURES"]
