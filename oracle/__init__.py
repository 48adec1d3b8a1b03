"""CPU checkers for the parity tests (test infrastructure only).

* ``liboracle.so``  (tl_oracle.c): bit-faithful C restatement of the
  reference's int8 Mistral path, multithreaded over output rows.
* ``_ref/libtorchless_ref.so`` (ref_harness.cpp + the reference's own
  sources, built by ``make ref`` where the reference tree exists): the
  reference itself, used to pin the restatement and as the timed CPU
  baseline.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs may
use this package; the product path never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libtorchless_ref.so")
# the same harness and reference sources with the CUDA backend for kernels.h
REF_CUDA_SO = os.path.join(HERE, "_ref", "libtorchless_ref_cuda.so")
# The reference source tree, for building _ref: given by the caller or the
# TORCHLESS_REFERENCE environment variable (no default; absent -> _ref is not built).
REFERENCE_ENV = "TORCHLESS_REFERENCE"

_P, _S, _F, _I, _U32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_float, ctypes.c_int, ctypes.c_uint32


def build(reference: bool = True, tree: Optional[str] = None) -> None:
    """make liboracle.so, and _ref when a reference tree (`tree`, else
    $TORCHLESS_REFERENCE) is given and present."""
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    tree = tree or os.environ.get(REFERENCE_ENV)
    if reference and tree and os.path.isdir(os.path.join(tree, "src")):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={tree}"], check=True)
        # the reference's model loop over the CUDA backend, once the CUDA library exists
        if os.path.exists(os.path.join(os.path.dirname(HERE), "torchless_b200", "libtorchless_b200.so")):
            subprocess.run(["make", "-s", "-C", HERE, "ref-cuda", f"REF={tree}"], check=True)


def _f(a: np.ndarray):
    return a.ctypes.data


class tlo_config(ctypes.Structure):
    _fields_ = [(n, _S) for n in ("hidden", "inter", "n_layers", "n_heads", "n_kv_heads", "vocab",
                                  "head_dim", "max_seq")] + [("rope_theta", _F), ("window", _S)]


_oracle: Optional[ctypes.CDLL] = None
_ref: Optional[ctypes.CDLL] = None


def oracle_lib() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            build(reference=False)
        L = ctypes.CDLL(ORACLE_SO)
        sig = {
            "tlo_matmul_f32": (None, [_P, _P, _P, _S, _S]),
            "tlo_matmul_i8": (None, [_P, _P, _P, _S, _P, _S, _S]),
            "tlo_row_matmul": (None, [_P, _P, _P, _S, _S]),
            "tlo_softmax": (None, [_P, _P, _S]),
            "tlo_rope": (None, [_P, _P, _P, _P, _S, _S]),
            "tlo_silu": (None, [_P, _P, _S]),
            "tlo_sum": (_F, [_P, _S]),
            "tlo_add": (None, [_P, _P, _P, _S]),
            "tlo_add_scalar": (None, [_P, _P, _F, _S]),
            "tlo_mul": (None, [_P, _P, _P, _S]),
            "tlo_mul_scalar": (None, [_P, _P, _F, _S]),
            "tlo_pow": (None, [_P, _P, _I, _S]),
            "tlo_sqrt": (None, [_P, _P, _S]),
            "tlo_rmsnorm": (None, [_P, _P, _S, _F]),
            "tlo_init_freq": (None, [_P, _S, _F]),
            "tlo_rope_cos_sin": (None, [_P, _P, _P, _S, _S, _S]),
            "tlo_argmax": (_U32, [_P, _S]),
            "tlo_sample_multinomial": (_U32, [_P, _S, _F, _F]),
            "tlo_sample_uniform": (_F, [ctypes.c_uint64, ctypes.c_uint64]),
            "tlo_quantize": (None, [_P, _P, _P, _S, _S]),
            "tlo_model_new": (_P, [ctypes.POINTER(tlo_config)]),
            "tlo_model_free": (None, [_P]),
            "tlo_model_set_tensor": (_I, [_P, _I, _I, _P, _P, _S, _S, _S]),
            "tlo_model_set_tensor_fp8": (_I, [_P, _I, _I, _P, _S, _S]),
            "tlo_fp8_to_f32": (_F, [ctypes.c_uint8]),
            "tlo_matmul_f8": (None, [_P, _P, _P, _S, _S]),
            "tlo_model_pos": (_S, [_P]),
            "tlo_model_set_pos": (None, [_P, _S]),
            "tlo_model_logits": (ctypes.POINTER(_F), [_P]),
            "tlo_model_hidden": (ctypes.POINTER(_F), [_P]),
            "tlo_model_layer_forward": (_I, [_P, _S]),
            "tlo_model_k_cache": (ctypes.POINTER(_F), [_P]),
            "tlo_model_v_cache": (ctypes.POINTER(_F), [_P]),
            "tlo_model_forward": (_I, [_P, _U32]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _oracle = L
    return _oracle


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib() -> ctypes.CDLL:
    """The reference's own code (oracle/_ref/libtorchless_ref.so)."""
    global _ref
    if _ref is None:
        _ref = _load_ref(REF_SO)
    return _ref


_ref_cuda: Optional[ctypes.CDLL] = None


def ref_cuda_available() -> bool:
    return os.path.exists(REF_CUDA_SO)


def ref_cuda_lib() -> ctypes.CDLL:
    """The reference's model loop over the CUDA backend of its op API
    (oracle/_ref/libtorchless_ref_cuda.so; same entry points as ref_lib())."""
    global _ref_cuda
    if _ref_cuda is None:
        _ref_cuda = _load_ref(REF_CUDA_SO)
    return _ref_cuda


def _load_ref(path: str) -> ctypes.CDLL:
    if not os.path.exists(path):
        raise RuntimeError(f"{path} not built (make -C oracle ref / ref-cuda needs the reference tree)")
    L = ctypes.CDLL(path)
    sig = {
        "ref_load_file": (_P, [ctypes.c_char_p, _S]),
        "ref_load_buffer": (_P, [_P, _S, _S]),
        "ref_free": (None, [_P]),
        "ref_forward": (_I, [_P, _U32]),
        "ref_logits": (ctypes.POINTER(_F), [_P]),
        "ref_hidden": (ctypes.POINTER(_F), [_P]),
        "ref_sample_max": (_U32, [_P]),
        "ref_sample_logits": (_U32, [_P, _P, _F, _U32, ctypes.POINTER(_F)]),
        "ref_tokenizer_new": (_P, [ctypes.c_char_p, _S]),
        "ref_tokenizer_free": (None, [_P]),
        "ref_tokenizer_encode": (_S, [_P, ctypes.c_char_p, _S, _P, _S]),
        "ref_tokenizer_decode": (_S, [_P, _P, _S, _P, _S]),
        "ref_pos": (_S, [_P]),
        "ref_set_pos": (None, [_P, _S]),
        "ref_layer_forward": (_I, [_P, _I, _P]),
        "ref_time_token": (_I, [_P, _U32, _I, _I, ctypes.POINTER(ctypes.c_double)]),
        "ref_matmul_i8": (None, [_P, _P, _P, _S, _P, _S, _S]),
        "ref_matmul_f32": (None, [_P, _P, _P, _S, _S]),
        "ref_row_matmul": (None, [_P, _P, _P, _S, _S]),
        "ref_softmax": (None, [_P, _P, _S]),
        "ref_rope": (None, [_P, _P, _P, _P, _S, _S]),
        "ref_silu": (None, [_P, _P, _S]),
        "ref_rmsnorm": (None, [_P, _P, _P]),
        "ref_rotary": (None, [_P, _S, _P, _P, _P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


# ---------------------------------------------------------------------------
# Whole-model checkers over a model binary held in host memory.
# ---------------------------------------------------------------------------

_KINDS = {
    "input_layernorm.weight": 3, "post_attention_layernorm.weight": 4,
    "self_attn.q_proj.weight": 5, "self_attn.k_proj.weight": 6, "self_attn.v_proj.weight": 7,
    "self_attn.o_proj.weight": 8, "mlp.gate_proj.weight": 9, "mlp.down_proj.weight": 10,
    "mlp.up_proj.weight": 11,
}
_GLOBAL = {"model.embed_tokens.weight": 0, "model.norm.weight": 1, "lm_head.weight": 2}


class OracleModel:
    """Model<T>::forward restated in C, over a binfmt.ModelFile."""

    def __init__(self, mf, max_seq: int = 1024, window: int = 0):
        """window > 0: sliding-window attention over the last `window` positions
        (an opt-in departure from the reference, which attends to all)."""
        self.mf = mf  # keeps the buffer alive
        c = mf.config
        cfg = tlo_config(c.hidden_size, c.intermediate_size, c.n_layers, c.n_heads, c.n_kv_heads,
                         c.vocab_size, c.head_dim, max_seq, c.rope_theta, window)
        L = oracle_lib()
        self._h = L.tlo_model_new(ctypes.byref(cfg))
        if not self._h:
            raise MemoryError("oracle model allocation failed")
        self.vocab = c.vocab_size
        self.hidden = c.hidden_size
        self.kv_shape = (c.n_layers, c.n_kv_heads, max_seq, c.head_dim)
        for name, info in mf.tensors.items():
            data, scales = mf.tensor(name)
            rows = info.shape[0]
            cols = info.shape[1] if len(info.shape) > 1 else 1
            sp = scales.ctypes.data if scales is not None else None
            ns = scales.size if scales is not None else 0
            if name in _GLOBAL:
                layer, kind = -1, _GLOBAL[name]
            else:
                rest = name[len("model.layers."):]
                lstr, key = rest.split(".", 1)
                layer, kind = int(lstr), _KINDS[key]
            if info.dtype == "fp8":
                rc = L.tlo_model_set_tensor_fp8(self._h, layer, kind, data.ctypes.data, rows, cols)
            else:
                rc = L.tlo_model_set_tensor(self._h, layer, kind, data.ctypes.data, sp, ns, rows, cols)
            if rc:
                raise ValueError(f"oracle rejected tensor {name}")

    def close(self):
        if self._h:
            oracle_lib().tlo_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter teardown: the module's globals may be gone
            pass

    @property
    def pos(self) -> int:
        return oracle_lib().tlo_model_pos(self._h)

    @pos.setter
    def pos(self, p: int):
        oracle_lib().tlo_model_set_pos(self._h, p)

    def forward(self, token: int) -> np.ndarray:
        if oracle_lib().tlo_model_forward(self._h, token):
            raise ValueError("oracle forward rejected (pos >= max_seq or token >= vocab)")
        return np.ctypeslib.as_array(oracle_lib().tlo_model_logits(self._h), (self.vocab,)).copy()

    def read_kv(self, layer: int, pos: int):
        """InferenceState k_cache/v_cache rows (inference_state.h:25-26) at (layer, pos)."""
        n = int(np.prod(self.kv_shape))
        k = np.ctypeslib.as_array(oracle_lib().tlo_model_k_cache(self._h), (n,)).reshape(self.kv_shape)
        v = np.ctypeslib.as_array(oracle_lib().tlo_model_v_cache(self._h), (n,)).reshape(self.kv_shape)
        return k[layer, :, pos].copy(), v[layer, :, pos].copy()

    def write_kv(self, layer: int, pos: int, k: np.ndarray, v: np.ndarray) -> None:
        """Sets the cache rows at (layer, pos) (test set-up of a pre-filled cache)."""
        n = int(np.prod(self.kv_shape))
        kc = np.ctypeslib.as_array(oracle_lib().tlo_model_k_cache(self._h), (n,)).reshape(self.kv_shape)
        vc = np.ctypeslib.as_array(oracle_lib().tlo_model_v_cache(self._h), (n,)).reshape(self.kv_shape)
        kc[layer, :, pos] = k
        vc[layer, :, pos] = v

    def layer_forward(self, layer: int, h: np.ndarray) -> np.ndarray:
        hid = np.ctypeslib.as_array(oracle_lib().tlo_model_hidden(self._h), (self.hidden,))
        hid[:] = h
        if oracle_lib().tlo_model_layer_forward(self._h, layer):
            raise ValueError("oracle layer forward rejected")
        return hid.copy()


class RefModel:
    """The reference's own Model<T> (oracle/_ref) over an in-memory binary, or
    over a file (path=...), which the reference's loader maps read-only
    (Parameters::load_parameters, parameters.cpp:95-129).  lib: ref_lib()
    (default) or ref_cuda_lib()."""

    def __init__(self, buf: Optional[np.ndarray] = None, max_seq: int = 500, path: Optional[str] = None,
                 lib: Optional[ctypes.CDLL] = None):
        self._lib = L = lib or ref_lib()
        from torchless_b200.binfmt import ModelFile
        if path is not None:
            self.buf = None
            self._h = L.ref_load_file(path.encode(), max_seq)
            c = ModelFile.open(path).config
        else:
            self.buf = np.ascontiguousarray(buf)
            self._h = L.ref_load_buffer(self.buf.ctypes.data, self.buf.nbytes, max_seq)
            c = ModelFile(self.buf).config
        if not self._h:
            raise ValueError("reference rejected the model binary")
        self.vocab, self.hidden = c.vocab_size, c.hidden_size

    def close(self):
        if self._h:
            self._lib.ref_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter teardown: the module's globals may be gone
            pass

    @property
    def pos(self) -> int:
        return self._lib.ref_pos(self._h)

    @pos.setter
    def pos(self, p: int):
        self._lib.ref_set_pos(self._h, p)

    def forward(self, token: int) -> np.ndarray:
        if self._lib.ref_forward(self._h, token):
            raise ValueError("reference forward rejected")
        return np.ctypeslib.as_array(self._lib.ref_logits(self._h), (self.vocab,)).copy()

    def sample_max(self) -> int:
        return self._lib.ref_sample_max(self._h)

    def sample_logits(self, logits: np.ndarray, temp: float, seed: int):
        """The reference's sample_multinomial (main.cpp:23-43) on `logits` with its
        generator seeded by `seed`: (index, the uniform draw r it used)."""
        x = np.ascontiguousarray(logits, dtype=np.float32)
        assert x.size == self.vocab
        r = _F()
        idx = self._lib.ref_sample_logits(self._h, x.ctypes.data, float(temp), int(seed), ctypes.byref(r))
        return int(idx), float(r.value)

    def layer_forward(self, layer: int, h: np.ndarray) -> np.ndarray:
        x = np.array(h, dtype=np.float32, copy=True)
        if self._lib.ref_layer_forward(self._h, layer, x.ctypes.data):
            raise ValueError("reference layer forward rejected")
        return x

    def time_token(self, token: int, first_layer: int, n_layers: int):
        out = (ctypes.c_double * 3)()
        if self._lib.ref_time_token(self._h, token, first_layer, n_layers, out):
            raise ValueError("reference timing rejected")
        return tuple(out)


class RefTokenizer:
    """The reference's own Tokenizer (tokenizer.cpp, built into oracle/_ref)."""

    def __init__(self, tok):
        import json
        text = (tok if isinstance(tok, str) else json.dumps(tok)).encode("utf-8")
        self._h = ref_lib().ref_tokenizer_new(text, len(text))
        if not self._h:
            raise ValueError("reference tokenizer rejected the JSON")

    def close(self):
        if self._h:
            ref_lib().ref_tokenizer_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # interpreter teardown: the module's globals may be gone
            pass

    def encode(self, text) -> list:
        b = text.encode("utf-8") if isinstance(text, str) else bytes(text)
        cap = 2 * len(b) + 8
        ids = np.empty(cap, dtype=np.uint32)
        n = ref_lib().ref_tokenizer_encode(self._h, b, len(b), ids.ctypes.data, cap)
        assert n <= cap
        return ids[:n].tolist()

    def decode_bytes(self, ids) -> bytes:
        a = np.ascontiguousarray(ids, dtype=np.uint32)
        cap = 64 + 64 * len(a)
        out = ctypes.create_string_buffer(cap)
        n = ref_lib().ref_tokenizer_decode(self._h, a.ctypes.data, a.size, out, cap)
        assert n <= cap
        return out.raw[:n]


def sample_multinomial(logits: np.ndarray, temp: float, r: float) -> int:
    """sample_multinomial (main.cpp:23-43) with the uniform draw r given."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return int(oracle_lib().tlo_sample_multinomial(x.ctypes.data, x.size, float(temp), float(r)))


def sample_uniform(seed: int, pos: int) -> float:
    """The library's device-side uniform draw for (seed, position)."""
    return float(oracle_lib().tlo_sample_uniform(int(seed), int(pos)))


def greedy(model, prompt, n_new):
    """main.cpp:69-77 greedy loop on any checker model: returns (ids, logits per step)."""
    for t in prompt[:-1]:
        model.forward(int(t))
    t = int(prompt[-1])
    ids, logits = [], []
    for _ in range(n_new):
        lg = model.forward(t)
        t = int(oracle_lib().tlo_argmax(lg.ctypes.data, lg.size))
        ids.append(t)
        logits.append(lg)
    return ids, logits
