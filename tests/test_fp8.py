"""fp8 export (a format extension after the reference's roadmap item "Support
fp8 with a cast tensor.to(torch.float8_e5m2) during model export",
README.md:160): CPU checks of the cast, the e5m2 decode, the file layout and
the oracle's fp8 matmul.  The reference has no fp8 code to compare with, so
the pins are torch's own e5m2 cast and conversion (the roadmap's named
mechanism) and the sequential fp32 sum of kernels.cpp:21-33."""
import numpy as np
import pytest

from torchless_b200 import binfmt, synthetic as S

torch = pytest.importorskip("torch")


def test_e5m2_decode_matches_torch_for_every_code(oracle_lib):
    """All 256 bit patterns: the numpy decode (fp16 high byte) and the C
    oracle's decode (sign, exponent, mantissa from the definition) equal
    torch.float8_e5m2 -> float32, including subnormals, infinities and NaNs."""
    codes = np.arange(256, dtype=np.uint8)
    want = torch.from_numpy(codes.copy()).view(torch.float8_e5m2).float().numpy()
    np.testing.assert_array_equal(binfmt.fp8_to_f32(codes), want)
    got = np.array([oracle_lib.tlo_fp8_to_f32(int(c)) for c in codes], dtype=np.float32)
    np.testing.assert_array_equal(got, want)
    assert np.isinf(want[0x7C]) and np.isnan(want[0x7D]) and want[0x01] == 2.0 ** -16


def test_export_cast_is_torch_cast():
    """quantize_fp8 is x.to(torch.float8_e5m2): round to nearest even, ties
    and subnormals included, overflow to infinity."""
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(4096) * 0.02).astype(np.float32)
    # exact ties between e5m2 neighbours (1.0, 1.25: midpoint 1.125), subnormal
    # range, the largest finite value and beyond
    x[:8] = [1.125, -1.375, 3 * 2.0 ** -18, 2.0 ** -17, 57344.0, 61440.0, 1e6, -0.0]
    q = binfmt.quantize_fp8(x)
    assert q.dtype == np.uint8 and q.shape == x.shape
    np.testing.assert_array_equal(q, torch.from_numpy(x).to(torch.float8_e5m2).view(torch.uint8).numpy())
    d = binfmt.fp8_to_f32(q)
    assert d[0] == 1.0 and d[1] == -1.5 and d[4] == 57344.0 and np.isinf(d[6])
    # round to nearest: within half an e5m2 step (2 mantissa bits) of the source
    mid = np.abs(x[8:]) > 2.0 ** -14
    rel = np.abs(d[8:] - x[8:])[mid] / np.abs(x[8:])[mid]
    assert rel.max() <= 0.125 + 1e-7


def test_fp8_file_layout():
    """quant "fp8": every _proj tensor is one e5m2 byte per element, dtype
    "fp8", no scales, 64-byte aligned; the f32 tensors are the int8 file's."""
    i8 = binfmt.ModelFile(S.make_numpy_model(S.TINY, seed=7, norm="random").buf)
    f8w = S.make_numpy_model(S.TINY, seed=7, norm="random", quant="fp8")
    f8 = binfmt.ModelFile(f8w.buf)
    assert f8.config.quant == "fp8"
    src = dict(S.numpy_tensors(S.TINY, seed=7, norm="random"))
    end = 0
    for name, t in f8.tensors.items():
        assert t.offset % 64 == 0
        data, scales = f8.tensor(name)
        assert scales is None and t.scale_offset is None
        if "_proj" in name:
            assert t.dtype == "fp8" and data.dtype == np.uint8
            np.testing.assert_array_equal(data, binfmt.quantize_fp8(src[name]))
            end = max(end, t.offset + t.numel)
        else:
            assert t.dtype == "f32"
            np.testing.assert_array_equal(data, i8.tensor(name)[0])
            end = max(end, t.offset + 4 * t.numel)
    assert f8w.size == f8.payload_offset + end + binfmt.pad_to_64(end)
    # the lm_head in the projections' format (fp8 here)
    lm = binfmt.ModelFile(S.make_numpy_model(S.TINY, seed=7, norm="random", quant="fp8", quant_lm_head=True).buf)
    t = lm.tensors[binfmt.LM_HEAD]
    assert t.dtype == "fp8" and t.scale_offset is None
    np.testing.assert_array_equal(lm.tensor(binfmt.LM_HEAD)[0], binfmt.quantize_fp8(src[binfmt.LM_HEAD]))


def test_unknown_quant_is_rejected():
    with pytest.raises(ValueError):
        binfmt.build_header({}, [("a_proj", (64, 64))], "int4", S.PLACEHOLDER_TOKENIZER)


def test_oracle_fp8_matmul_is_the_sequential_fp32_sum(oracle_lib):
    """tlo_matmul_f8: per row, acc += w_j * x_j in fp32, j ascending (each
    numpy float32 operation below rounds like the reference's C++)."""
    rng = np.random.default_rng(3)
    n, d = 37, 200
    w = binfmt.quantize_fp8((rng.standard_normal((n, d)) * 0.05).astype(np.float32))
    x = rng.standard_normal(d).astype(np.float32)
    y = np.zeros(n, dtype=np.float32)
    oracle_lib.tlo_matmul_f8(y.ctypes.data, w.ctypes.data, x.ctypes.data, n, d)
    wf = binfmt.fp8_to_f32(w)
    acc = np.zeros(n, dtype=np.float32)
    for j in range(d):
        acc = (acc + (wf[:, j] * x[j]).astype(np.float32)).astype(np.float32)
    np.testing.assert_array_equal(y, acc)


def test_oracle_model_runs_an_fp8_file():
    """The oracle resolves fp8 tensors to its e5m2 matmul (logits finite and
    different from the int8 file's, which quantises differently)."""
    import oracle
    f8 = binfmt.ModelFile(S.make_numpy_model(S.TINY, seed=3, quant="fp8", norm="random").buf)
    i8 = binfmt.ModelFile(S.make_numpy_model(S.TINY, seed=3, norm="random").buf)
    a = oracle.OracleModel(f8, max_seq=8).forward(5)
    b = oracle.OracleModel(i8, max_seq=8).forward(5)
    assert np.all(np.isfinite(a)) and not np.array_equal(a, b)
    assert np.abs(a - b).max() < 0.5 * np.abs(b).max()
