"""The CPU oracle against the reference's own golden data (no GPU).

Pins tl_oracle.c three ways:
  * the weight-independent vectors of test/mistral/expected.txt and the
    known-answer cases of test_cpu_kernels.cpp, with the reference test
    tolerance (atol 5e-2, setup/context.cpp:41-45) and a much tighter one;
  * bit-exact equality with reference kernels on seeded inputs (ref_ops.npz);
  * bit-exact logits and ids of the reference's Model<int8_t> over 40 tokens
    of two seeded models (ref_greedy_*.npz).
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN, golden_greedy

import oracle
from torchless_b200.binfmt import ModelFile


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def test_inv_freq_cos_sin(golden_expected, oracle_lib):
    # test_modules.cpp:166-215 (inv_freq, cos/sin at positions 0 and 3).
    v = golden_expected["vectors"]
    inv = np.zeros(64, np.float32)
    oracle_lib.tlo_init_freq(inv.ctypes.data, 64, 10000.0)
    np.testing.assert_allclose(inv, v["inv_freq"], rtol=1e-6, atol=1e-7)
    for pos in (0, 3):
        c = np.zeros(128, np.float32)
        s = np.zeros(128, np.float32)
        oracle_lib.tlo_rope_cos_sin(c.ctypes.data, s.ctypes.data, inv.ctypes.data, 64, 128, pos)
        np.testing.assert_allclose(c, v[f"cos{pos}"], atol=1e-5)
        np.testing.assert_allclose(s, v[f"sin{pos}"], atol=1e-5)


def test_rope_positions(golden_expected, oracle_lib):
    # test_cpu_kernels.cpp:4-29: q[i] = (i % 128)/256 at positions 0..3.
    v = golden_expected["vectors"]
    inv = np.zeros(64, np.float32)
    oracle_lib.tlo_init_freq(inv.ctypes.data, 64, 10000.0)
    for pos in range(4):
        c = np.zeros(128, np.float32)
        s = np.zeros(128, np.float32)
        oracle_lib.tlo_rope_cos_sin(c.ctypes.data, s.ctypes.data, inv.ctypes.data, 64, 128, pos)
        q = f32((np.arange(128) % 128) / 256.0)
        oracle_lib.tlo_rope(q.ctypes.data, q.ctypes.data, c.ctypes.data, s.ctypes.data, 1, 128)
        np.testing.assert_allclose(q, v[f"rope{pos}"], atol=5e-2)
        np.testing.assert_allclose(q, v[f"rope{pos}"], atol=1e-5)


def test_rmsnorm_fixture(golden_expected, oracle_lib):
    # test_modules.cpp:219-235.  The fixture was made with eps 1e-6
    # (scripts/test/mistral/rmsnorm.py) against the engine's 1e-5; the
    # difference is far below the reference's atol.
    v = golden_expected["vectors"]
    x = f32(v["norm_x"])
    g = f32(v["norm_g"])
    oracle_lib.tlo_rmsnorm(x.ctypes.data, g.ctypes.data, 4096, 1e-5)
    np.testing.assert_allclose(x, v["norm_y"], atol=5e-2)
    np.testing.assert_allclose(x, v["norm_y"], atol=1e-4)


def test_kernel_kats(golden_expected, oracle_lib):
    k = golden_expected["kats"]
    w, x = f32(k["matmul"]["w"]), f32(k["matmul"]["x"])
    y = np.zeros(2, np.float32)
    oracle_lib.tlo_matmul_f32(y.ctypes.data, w.ctypes.data, x.ctypes.data, 2, 3)
    np.testing.assert_array_equal(y, k["matmul"]["y"])
    w, x = f32(k["row_matmul"]["w"]), f32(k["row_matmul"]["x"])
    y = np.zeros(2, np.float32)
    oracle_lib.tlo_row_matmul(y.ctypes.data, x.ctypes.data, w.ctypes.data, 3, 2)
    np.testing.assert_array_equal(y, k["row_matmul"]["y"])
    x = f32(k["softmax"]["x"])
    y = np.zeros(3, np.float32)
    oracle_lib.tlo_softmax(y.ctypes.data, x.ctypes.data, 3)
    np.testing.assert_allclose(y, k["softmax"]["y"], atol=1e-7)
    x = f32(k["silu"]["x"])
    y = np.zeros(5, np.float32)
    oracle_lib.tlo_silu(y.ctypes.data, x.ctypes.data, 5)
    np.testing.assert_allclose(y, k["silu"]["y"], atol=1e-4)


def test_ops_bit_exact_vs_reference(oracle_lib):
    # Materialise every array first: a temporary's .ctypes.data would dangle.
    d = dict(np.load(os.path.join(GOLDEN, "ref_ops.npz")))
    q = d["i8_q"]
    n, dd = q.shape
    for tag in ("g64", "g80", "g7"):
        s, x = d[f"i8_{tag}_s"], d[f"i8_{tag}_x"]
        y = np.zeros(n, np.float32)
        oracle_lib.tlo_matmul_i8(y.ctypes.data, q.ctypes.data, s.ctypes.data, s.size, x.ctypes.data, n, dd)
        np.testing.assert_array_equal(y, d[f"i8_{tag}_y"], err_msg=tag)
    y = np.zeros(7, np.float32)
    oracle_lib.tlo_matmul_f32(y.ctypes.data, d["f32_w"].ctypes.data, d["f32_x"].ctypes.data, 7, 33)
    np.testing.assert_array_equal(y, d["f32_y"])
    y = np.zeros(17, np.float32)
    oracle_lib.tlo_row_matmul(y.ctypes.data, d["row_x"].ctypes.data, d["row_w"].ctypes.data, 9, 17)
    np.testing.assert_array_equal(y, d["row_y"])
    y = np.zeros(13, np.float32)
    oracle_lib.tlo_softmax(y.ctypes.data, d["softmax_x"].ctypes.data, 13)
    np.testing.assert_array_equal(y, d["softmax_y"])
    y = np.zeros((3, 16), np.float32)
    oracle_lib.tlo_rope(y.ctypes.data, d["rope_x"].ctypes.data, d["rope_c"].ctypes.data,
                        d["rope_s"].ctypes.data, 3, 16)
    np.testing.assert_array_equal(y, d["rope_y"])
    y = np.zeros(11, np.float32)
    oracle_lib.tlo_silu(y.ctypes.data, d["silu_x"].ctypes.data, 11)
    np.testing.assert_array_equal(y, d["silu_y"])


@pytest.mark.parametrize("name", ["tiny", "small"])
def test_model_bit_exact_vs_reference(name, request):
    prompt, ids, logits = golden_greedy(name)
    buf = request.getfixturevalue(f"{name}_bin")
    om = oracle.OracleModel(ModelFile(buf), max_seq=64)
    got_ids, got_logits = oracle.greedy(om, prompt, len(ids))
    assert got_ids == ids
    for step, (a, b) in enumerate(zip(got_logits, logits)):
        np.testing.assert_array_equal(a, b, err_msg=f"step {step}")


def test_argmax_first_max_and_nan(oracle_lib):
    # sample_max (main.cpp:10-21): first strict maximum; NaN at 0 pins index 0.
    x = f32([1, 3, 3, 2])
    assert oracle_lib.tlo_argmax(x.ctypes.data, 4) == 1
    x = f32([np.nan, 3, 5])
    assert oracle_lib.tlo_argmax(x.ctypes.data, 3) == 0
    x = f32([-np.inf, -np.inf])
    assert oracle_lib.tlo_argmax(x.ctypes.data, 2) == 0


def test_quantize_matches_numpy(oracle_lib):
    from torchless_b200.binfmt import quantize_i8
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(64 * 300) * 0.02).astype(np.float32)
    q = np.zeros(x.size, np.int8)
    s = np.zeros(x.size // 64, np.float32)
    oracle_lib.tlo_quantize(q.ctypes.data, s.ctypes.data, x.ctypes.data, x.size, 64)
    q2, s2 = quantize_i8(x)
    np.testing.assert_array_equal(q, q2)
    np.testing.assert_array_equal(s, s2)


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built here")
def test_oracle_vs_live_reference_random_ops(oracle_lib):
    """Fresh seeded inputs through both libraries (when the reference build is present)."""
    L = oracle.ref_lib()
    rng = np.random.default_rng(11)
    for n, d in ((5, 64), (33, 128), (64, 1024)):
        q = rng.integers(-127, 128, (n, d), dtype=np.int8)
        s = f32(np.abs(rng.standard_normal(n * d // 64)) * 0.01 + 1e-3)
        x = f32(rng.standard_normal(d))
        a = np.zeros(n, np.float32)
        b = np.zeros(n, np.float32)
        L.ref_matmul_i8(a.ctypes.data, q.ctypes.data, s.ctypes.data, s.size, x.ctypes.data, n, d)
        oracle_lib.tlo_matmul_i8(b.ctypes.data, q.ctypes.data, s.ctypes.data, s.size, x.ctypes.data, n, d)
        np.testing.assert_array_equal(a, b)


def test_sample_multinomial_matches_reference_fixture():
    """tlo_sample_multinomial (the oracle's main.cpp:23-43) against the
    reference's own sample_multinomial on the committed fixture: same uniform
    draw r, same index, bit for bit -- including NaN / inf / all -inf logits,
    ties, temperature <= 0 (sample_max) and the last-index fallback when the
    running sum stops short of r."""
    d = np.load(os.path.join(GOLDEN, "ref_sample.npz"))
    L = d["logits"]
    for j, temp, r, idx in zip(d["set"], d["temp"], d["r"], d["idx"]):
        got = oracle.sample_multinomial(L[j], float(temp), float(r))
        assert got == idx, (int(j), float(temp), float(r), got, int(idx))
    assert (d["idx"] == L.shape[1] - 1).sum() >= 6  # the fallback is exercised


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built here")
def test_sample_multinomial_vs_live_reference():
    """Fresh logits (a forward of the TINY model, scaled) through both samplers."""
    from conftest import model_bytes
    rm = oracle.RefModel(model_bytes("tiny"), max_seq=8)
    lg = rm.forward(3)
    rng = np.random.default_rng(17)
    for k in range(60):
        x = (lg * rng.uniform(0.2, 5.0) + rng.standard_normal(lg.size) * 0.5).astype(np.float32)
        temp = float(rng.choice([0.0, 0.5, 1.0, 1.9]))
        idx, r = rm.sample_logits(x, temp, k)
        assert oracle.sample_multinomial(x, temp, r) == idx
    rm.close()


def test_sample_uniform_is_the_documented_counter_function():
    """The device sampling draw: splitmix64 of seed + (pos + 1) * golden ratio, top 24 bits / 2^24."""
    M = (1 << 64) - 1

    def ref(seed, pos):
        z = (seed + (pos + 1) * 0x9E3779B97F4A7C15) & M
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M
        z ^= z >> 31
        return (z >> 40) / 16777216.0

    for seed, pos in [(0, 0), (1, 5), (123456789, 1000), (M, 7)]:
        assert oracle.sample_uniform(seed, pos) == ref(seed, pos)
