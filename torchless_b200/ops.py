"""Device ops with the names and argument order of src/common/kernels.h.

Each function takes CUDA float32 tensors (int8 for quantised weights) and
launches on torch's current stream.  Output first, like the reference:
``matmul(xout, w, x)`` computes ``xout = w @ x``.  Shapes follow the
reference's Tensor shapes; in-place calls (``xout is x``) are allowed where
the reference makes them (rope, softmax, silu, mul in modules.cpp).
"""
from __future__ import annotations

import ctypes

from . import check, lib


def _ptr(t) -> int:
    if not t.is_cuda:
        raise ValueError("ops take CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("ops take contiguous tensors")
    return t.data_ptr()


def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _f32(t):
    import torch
    if t.dtype != torch.float32:
        raise TypeError(f"expected float32, got {t.dtype}")
    return _ptr(t)


def matmul(xout, w, x, scales=None) -> None:
    """kernels.h:11-12: xout[n] = w[n, d] @ x[d]; int8 ``w`` needs its stored
    ``scales``; fp8 ``w`` (torch.float8_e5m2, or uint8 holding e5m2 bit
    patterns: the fp8 export) has none."""
    import torch
    n, d = w.shape
    if x.numel() != d or xout.numel() < n:
        raise ValueError("matmul shape mismatch")  # kernels.cpp:10, 25
    if w.dtype in (torch.float8_e5m2, torch.uint8):
        if scales is not None:
            raise ValueError("fp8 weights have no scales")
        check(lib().tl_matmul_f8(_f32(xout), _ptr(w), _f32(x), n, d, _stream()))
    elif w.dtype == torch.int8:
        if scales is None:
            raise ValueError("int8 matmul needs scales")
        check(lib().tl_matmul_i8(_f32(xout), _ptr(w), _f32(scales), scales.numel(), _f32(x), n, d, _stream()))
    else:
        check(lib().tl_matmul_f32(_f32(xout), _f32(w), _f32(x), n, d, _stream()))


def row_matmul(xout, x, w) -> None:
    """kernels.h:13: xout[d] = x[n] @ w[n, d]."""
    n, d = w.shape
    if x.shape[0] != n or xout.numel() < d:
        raise ValueError("matmul shape mismatch")  # kernels.cpp:42
    check(lib().tl_row_matmul(_f32(xout), _f32(x), _f32(w), n, d, _stream()))


def softmax(xout, x) -> None:
    check(lib().tl_softmax(_f32(xout), _f32(x), x.numel(), _stream()))


def rope(xout, x, cos, sin) -> None:
    """kernels.h:16: x is [n_heads, head_dim]."""
    n_heads, head_dim = x.shape
    check(lib().tl_rope(_f32(xout), _f32(x), _f32(cos), _f32(sin), n_heads, head_dim, _stream()))


def silu(xout, x) -> None:
    check(lib().tl_silu(_f32(xout), _f32(x), x.numel(), _stream()))


def sum(x):
    """kernels.h:20: returns a 1-element device tensor."""
    import torch
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    check(lib().tl_sum(_f32(out), _f32(x), x.numel(), _stream()))
    return out


def add(xout, x, y) -> None:
    if isinstance(y, (int, float)):
        check(lib().tl_add_scalar(_f32(xout), _f32(x), float(y), x.numel(), _stream()))
    else:
        check(lib().tl_add(_f32(xout), _f32(x), _f32(y), x.numel(), _stream()))


def mul(xout, x, y) -> None:
    if isinstance(y, (int, float)):
        check(lib().tl_mul_scalar(_f32(xout), _f32(x), float(y), x.numel(), _stream()))
    else:
        check(lib().tl_mul(_f32(xout), _f32(x), _f32(y), x.numel(), _stream()))


def pow(xout, x, e: int) -> None:  # noqa: A001 - reference name
    check(lib().tl_pow(_f32(xout), _f32(x), int(e), x.numel(), _stream()))


def sqrt(xout, x) -> None:
    check(lib().tl_sqrt(_f32(xout), _f32(x), x.numel(), _stream()))


def rmsnorm(xout, x, g, eps: float = 1e-5) -> None:
    """RMSNorm::forward (modules.cpp:31-46)."""
    check(lib().tl_rmsnorm(_f32(xout), _f32(x), _f32(g), x.numel(), float(eps), _stream()))


def rotary(cos, sin, inv_freq, pos: int) -> None:
    """RotaryEmbedding::forward (modules.cpp:22-27)."""
    check(lib().tl_rotary(_f32(cos), _f32(sin), _f32(inv_freq), inv_freq.numel(), cos.numel(), int(pos),
                          _stream()))


def argmax(logits):
    """sample_max (main.cpp:10-21); returns a 1-element uint32 device tensor (as int32)."""
    import torch
    out = torch.empty(1, dtype=torch.int32, device=logits.device)
    check(lib().tl_argmax(_ptr(out), _f32(logits), logits.numel(), _stream()))
    return out


def sample_multinomial(logits, temperature: float, r: float):
    """sample_multinomial (main.cpp:23-43) with the uniform draw r given; returns a
    1-element device tensor (int32) holding the index."""
    import torch
    out = torch.empty(1, dtype=torch.int32, device=logits.device)
    check(lib().tl_sample_multinomial(_ptr(out), _f32(logits), logits.numel(), float(temperature), float(r),
                                      _stream()))
    return out


def sample_uniform(seed: int, pos: int) -> float:
    """The uniform draw of device-side sampling for the token at position pos."""
    return float(lib().tl_sample_uniform(int(seed), int(pos)))


def mlp_gate_up(out, w1, s1, w3, s3, x) -> None:
    """silu(w1 @ x) * (w3 @ x) with int8 w1/w3 (modules.cpp:99-112)."""
    n, d = w1.shape
    check(lib().tl_mlp_gate_up(_f32(out), _ptr(w1), _f32(s1), _ptr(w3), _f32(s3), _f32(x), n, d, _stream()))


def quantize_i8(x, group: int = 64):
    """quantize (export_mistral.py:53-68) on the device: returns (q int8, scales f32)."""
    import torch
    xc = x.contiguous()
    q = torch.empty(xc.shape, dtype=torch.int8, device=x.device)
    s = torch.empty(xc.numel() // group, dtype=torch.float32, device=x.device)
    check(lib().tl_quantize_i8(_ptr(q), _f32(s), _f32(xc), xc.numel(), group, _stream()))
    return q, s
