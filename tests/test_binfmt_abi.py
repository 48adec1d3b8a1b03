"""File format, quantiser and C-ABI surface checks that need no GPU."""
import ctypes
import hashlib
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT, model_bytes

from torchless_b200 import LIB_PATH, SIGNATURES, binfmt, synthetic as S

HEADER = os.path.join(ROOT, "include", "torchless_b200.h")


def header_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"TL_API\s+[\w\s\*]+?\b(tl_\w+)\s*\(", text)))


@pytest.mark.parametrize("name", ["tiny", "small"])
def test_numpy_exporter_matches_reference_export(name, export_hashes):
    """Byte-identical to export_mistral.py's output for the same fp32 inputs."""
    b = model_bytes(name)
    h = export_hashes[name]
    assert b.size == h["size"]
    assert hashlib.sha256(b.tobytes()).hexdigest() == h["sha256"]


def test_reader_roundtrip(tiny_bin):
    mf = binfmt.ModelFile(tiny_bin)
    c = mf.config
    assert (c.hidden_size, c.n_layers, c.n_heads, c.n_kv_heads, c.head_dim) == (512, 2, 4, 1, 128)
    assert c.quant == "int8" and c.rope_theta == 10000.0
    src = dict(S.numpy_tensors(S.TINY, seed=7, norm="random"))
    for name, t in mf.tensors.items():
        data, scales = mf.tensor(name)
        assert (t.offset % 64) == 0
        if scales is None:
            np.testing.assert_array_equal(data, src[name])
        else:
            assert t.scale_offset % 64 == 0 and scales.size == data.size // 64
            # dequantised weight q / s (tensor.cpp:101-104) is within half a step of the source
            deq = data.reshape(-1, 64).astype(np.float32) / scales[:, None]
            step = 1.0 / scales[:, None]
            # (fp32 rounding of x*s and of q/s allow a hair over half a step)
            assert np.all(np.abs(deq - src[name].reshape(-1, 64)) <= (0.5 + 1e-3) * step)


def test_quantizer_matches_torch_expression():
    """export_mistral.py:53-68 evaluated by torch itself equals the numpy restatement."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(9)
    x = (rng.standard_normal((96, 128)) * 0.02).astype(np.float32)
    # a group with an exact .5 product, and tiny / huge magnitudes
    x[0, :64] = np.linspace(-1, 1, 64, dtype=np.float32)
    x[1, :64] *= 1e-30
    x[2, 64:] *= 1e30
    t = torch.from_numpy(x).reshape(-1, 64)
    scales = 127 / t.abs().max(dim=-1).values.unsqueeze(-1)
    q = (t * scales).round().to(torch.int8)
    q2, s2 = binfmt.quantize_i8(x)
    np.testing.assert_array_equal(q.numpy().reshape(x.shape), q2)
    np.testing.assert_array_equal(scales.squeeze(-1).numpy(), s2)


def test_header_declares_what_python_binds():
    assert set(SIGNATURES) | {"tl_last_error", "tl_status_name"} == set(header_symbols())


def test_library_exports_every_declared_symbol():
    assert os.path.exists(LIB_PATH), "build the library first (python -m torchless_b200.build)"
    out = subprocess.run(["nm", "-D", "--defined-only", LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\sT\s+(tl_\w+)", out))
    missing = set(header_symbols()) - exported
    assert not missing, f"declared but not exported: {sorted(missing)}"
    # nothing else leaks: only the declared C ABI is visible
    assert exported == set(header_symbols())


def test_library_loads_without_gpu():
    import torchless_b200 as tb
    L = tb.lib()
    assert L.tl_last_error() == b""


def _load_status(path):
    import torchless_b200 as tb
    h = ctypes.c_void_p()
    st = tb.lib().tl_model_load(path.encode(), None, ctypes.byref(h))
    return st, tb.lib().tl_last_error().decode()


def test_loader_errors_are_status_codes(tmp_path, tiny_bin):
    """Bad files return TL_ERR_* (the reference calls std::exit(1), parameters.cpp:13-26)."""
    st, msg = _load_status(str(tmp_path / "missing.bin"))
    assert st == 3 and "cannot open" in msg                      # TL_ERR_IO
    p = tmp_path / "trunc.bin"
    p.write_bytes(tiny_bin[:5].tobytes())
    assert _load_status(str(p))[0] == 4                          # TL_ERR_FORMAT
    p.write_bytes(tiny_bin[:4000].tobytes())
    assert _load_status(str(p))[0] == 4                          # header longer than the file
    p.write_bytes(tiny_bin[: tiny_bin.size // 2].tobytes())
    st, msg = _load_status(str(p))
    assert st == 4 and "past the end" in msg                     # payload truncated
    bad = tiny_bin.copy()
    bad[8] = ord("!")                                            # break the JSON
    p.write_bytes(bad.tobytes())
    assert _load_status(str(p))[0] == 4


def test_loader_rejects_unsupported_models(tmp_path):
    """f32 exports and GQA ratios other than the reference's hard-coded 4."""
    cfg = dict(S.TINY)
    w = S.make_numpy_model(cfg, seed=1, quant="f32")
    p = tmp_path / "f32.bin"
    w.save(str(p))
    st, msg = _load_status(str(p))
    assert st == 2 and "int8" in msg                             # TL_ERR_UNSUPPORTED
    cfg = dict(S.TINY, num_key_value_heads=2)
    w = S.make_numpy_model(cfg, seed=1)
    w.save(str(p))
    st, msg = _load_status(str(p))
    assert st == 2 and "h/4" in msg


def test_int8_lm_head_layout():
    """quant_lm_head stores lm_head.weight like a _proj tensor: int8, then its
    per-64-group fp32 scales, each block 64-byte aligned; everything else as
    the reference exporter writes it."""
    from torchless_b200 import synthetic as S
    from torchless_b200.binfmt import ModelFile, quantize_i8
    plain = ModelFile(S.make_numpy_model(S.TINY, seed=7, norm="random").buf)
    i8 = ModelFile(S.make_numpy_model(S.TINY, seed=7, norm="random", quant_lm_head=True).buf)
    t = i8.tensors["lm_head.weight"]
    assert t.dtype == "int8" and t.offset % 64 == 0 and t.scale_offset % 64 == 0
    assert plain.tensors["lm_head.weight"].dtype == "f32"
    w, _ = plain.tensor("lm_head.weight")
    q, s = i8.tensor("lm_head.weight")
    q2, s2 = quantize_i8(np.asarray(w))
    np.testing.assert_array_equal(q, q2)
    np.testing.assert_array_equal(s, s2)
    for name in plain.tensors:
        if name != "lm_head.weight":
            a, b = plain.tensor(name), i8.tensor(name)
            np.testing.assert_array_equal(a[0], b[0])
