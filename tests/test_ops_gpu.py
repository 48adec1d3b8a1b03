"""Op-level CUDA kernels (the kernels.h mirror) against the CPU oracle.

Tolerances: integer/byte work (quantiser, argmax) is bit-exact; fp32 work
is checked as max|gpu - oracle| / max|oracle| <= 1e-4 (the CUDA kernels sum
in a different order than the reference's sequential loops), far inside the
1e-2 logit tolerance of the model-level parity rule.
"""
import os

import numpy as np
import pytest

from conftest import GOLDEN, rel_err

pytestmark = pytest.mark.gpu
TOL = 1e-4

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    import torchless_b200
    torchless_b200.lib()  # fails loudly if the library is missing
    torch.cuda.set_device(0)


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to("cuda", dtype=dtype) if dtype else t.to("cuda")


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def oracle_i8(q, s, x):
    import oracle
    n, d = q.shape
    y = np.zeros(n, np.float32)
    q, s, x = np.ascontiguousarray(q), f32(s), f32(x)
    oracle.oracle_lib().tlo_matmul_i8(y.ctypes.data, q.ctypes.data, s.ctypes.data, s.size, x.ctypes.data, n, d)
    return y


def oracle_f32(w, x):
    import oracle
    n, d = w.shape
    y = np.zeros(n, np.float32)
    w, x = f32(w), f32(x)
    oracle.oracle_lib().tlo_matmul_f32(y.ctypes.data, w.ctypes.data, x.ctypes.data, n, d)
    return y


# ---- matmul(int8): generic shapes, odd scale groupings, fast-path shapes ----

def test_matmul_i8_reference_fixture():
    from torchless_b200 import ops
    d = dict(np.load(os.path.join(GOLDEN, "ref_ops.npz")))
    q = d["i8_q"]
    for tag in ("g64", "g80", "g7"):
        y = torch.zeros(q.shape[0], device="cuda")
        ops.matmul(y, dev(q), dev(d[f"i8_{tag}_x"]), scales=dev(d[f"i8_{tag}_s"]))
        assert rel_err(host(y), d[f"i8_{tag}_y"]) <= TOL, tag


@pytest.mark.parametrize("n,d", [(1, 64), (3, 192), (1000, 512), (4096, 4096), (1024, 4096),
                                 (14336, 4096), (4096, 14336), (32000, 4096), (777, 1536)])
def test_matmul_i8_sweep(n, d):
    """The GEMV sweep shapes (wq/wo, wk/wv, w1/w3, w2, lm_head-sized) plus ragged ones.
    Weights uniform int8 in [-127, 127], scales |N(0, 0.01)|, x ~ N(0, 1)."""
    from torchless_b200 import ops
    rng = np.random.default_rng(n * 7 + d)
    q = rng.integers(-127, 128, (n, d), dtype=np.int8)
    s = f32(np.abs(rng.standard_normal(n * d // 64)) * 0.01 + 1e-4)
    x = f32(rng.standard_normal(d))
    y = torch.full((n,), float("nan"), device="cuda")
    ops.matmul(y, dev(q), dev(x), scales=dev(s))
    assert rel_err(host(y), oracle_i8(q, s, x)) <= TOL


def test_matmul_i8_inplace_and_unaligned():
    """x offset by one float (16-byte misaligned) takes the generic path and still matches."""
    from torchless_b200 import ops
    rng = np.random.default_rng(3)
    q = rng.integers(-127, 128, (64, 512), dtype=np.int8)
    s = f32(np.abs(rng.standard_normal(64 * 512 // 64)) * 0.01 + 1e-4)
    x = f32(rng.standard_normal(513))
    xt = dev(x)[1:]
    y = torch.zeros(64, device="cuda")
    ops.matmul(y, dev(q), xt, scales=dev(s))
    assert rel_err(host(y), oracle_i8(q, s, x[1:])) <= TOL


@pytest.mark.parametrize("n,d", [(2, 3), (7, 33), (1, 1), (32000, 4096), (100, 512)])
def test_matmul_f32(n, d, golden_expected):
    from torchless_b200 import ops
    if (n, d) == (2, 3):
        k = golden_expected["kats"]["matmul"]
        w, x = f32(k["w"]), f32(k["x"])
    else:
        rng = np.random.default_rng(n + d)
        w, x = f32(rng.standard_normal((n, d)) * 0.02), f32(rng.standard_normal(d))
    y = torch.zeros(n, device="cuda")
    ops.matmul(y, dev(w), dev(x))
    assert rel_err(host(y), oracle_f32(w, x)) <= TOL


def test_row_matmul(golden_expected):
    from torchless_b200 import ops
    import oracle
    k = golden_expected["kats"]["row_matmul"]
    y = torch.zeros(2, device="cuda")
    ops.row_matmul(y, dev(f32(k["x"])), dev(f32(k["w"])))
    np.testing.assert_allclose(host(y), k["y"], rtol=1e-6)
    rng = np.random.default_rng(1)
    for n, d in ((143, 128), (1, 5), (9, 17)):
        w, x = f32(rng.standard_normal((n, d))), f32(rng.standard_normal(n))
        ref = np.zeros(d, np.float32)
        oracle.oracle_lib().tlo_row_matmul(ref.ctypes.data, x.ctypes.data, w.ctypes.data, n, d)
        y = torch.zeros(d, device="cuda")
        ops.row_matmul(y, dev(x), dev(w))
        assert rel_err(host(y), ref) <= TOL


@pytest.mark.parametrize("n", [1, 3, 1000, 32000])
def test_softmax(n, golden_expected):
    from torchless_b200 import ops
    import oracle
    if n == 3:
        x = f32(golden_expected["kats"]["softmax"]["x"])
    else:
        x = f32(np.random.default_rng(n).standard_normal(n) * 5)
    ref = np.zeros(n, np.float32)
    oracle.oracle_lib().tlo_softmax(ref.ctypes.data, x.ctypes.data, n)
    xt = dev(x)
    ops.softmax(xt, xt)  # in place, like modules.cpp:81
    assert rel_err(host(xt), ref) <= TOL


def test_rope_and_rotary(golden_expected):
    """test_cpu_kernels.cpp:4-29 on the device: rotary(pos) then rope of q[i] = (i%128)/256."""
    from torchless_b200 import ops
    v = golden_expected["vectors"]
    inv = dev(f32(v["inv_freq"]))
    for pos in range(4):
        c = torch.zeros(128, device="cuda")
        s = torch.zeros(128, device="cuda")
        ops.rotary(c, s, inv, pos)
        if pos in (0, 3):
            np.testing.assert_allclose(host(c), v[f"cos{pos}"], atol=1e-6)
            np.testing.assert_allclose(host(s), v[f"sin{pos}"], atol=1e-6)
        q = dev(f32((np.arange(128) % 128) / 256.0)).reshape(1, 128)
        ops.rope(q, q, c, s)
        np.testing.assert_allclose(host(q).ravel(), v[f"rope{pos}"], atol=1e-5)


def test_elementwise_and_sum(golden_expected):
    from torchless_b200 import ops
    import oracle
    L = oracle.oracle_lib()
    k = golden_expected["kats"]["silu"]
    y = torch.zeros(5, device="cuda")
    ops.silu(y, dev(f32(k["x"])))
    np.testing.assert_allclose(host(y), k["y"], atol=1e-4)
    rng = np.random.default_rng(2)
    for n in (1, 17, 100003):
        a, b = f32(rng.standard_normal(n)), f32(rng.standard_normal(n) + 2)
        for name, args in (("silu", ()), ("add", (b,)), ("mul", (b,)), ("add_s", (1.5,)), ("mul_s", (-0.25,)),
                           ("sqrt", ()), ("pow", (3,))):
            ref = np.zeros(n, np.float32)
            at = dev(np.abs(a) if name == "sqrt" else a)
            an = np.abs(a) if name == "sqrt" else a
            out = torch.zeros(n, device="cuda")
            if name == "silu":
                L.tlo_silu(ref.ctypes.data, an.ctypes.data, n); ops.silu(out, at)
            elif name == "add":
                L.tlo_add(ref.ctypes.data, an.ctypes.data, b.ctypes.data, n); ops.add(out, at, dev(b))
            elif name == "mul":
                L.tlo_mul(ref.ctypes.data, an.ctypes.data, b.ctypes.data, n); ops.mul(out, at, dev(b))
            elif name == "add_s":
                L.tlo_add_scalar(ref.ctypes.data, an.ctypes.data, 1.5, n); ops.add(out, at, 1.5)
            elif name == "mul_s":
                L.tlo_mul_scalar(ref.ctypes.data, an.ctypes.data, -0.25, n); ops.mul(out, at, -0.25)
            elif name == "sqrt":
                L.tlo_sqrt(ref.ctypes.data, an.ctypes.data, n); ops.sqrt(out, at)
            else:
                L.tlo_pow(ref.ctypes.data, an.ctypes.data, 3, n); ops.pow(out, at, 3)
            np.testing.assert_allclose(host(out), ref, rtol=2e-6, atol=1e-6, err_msg=name)
        got = float(host(ops.sum(dev(a)))[0])
        assert abs(got - float(np.sum(a, dtype=np.float64))) <= 1e-4 * max(1.0, float(np.sum(np.abs(a))))


def test_rmsnorm_fixture(golden_expected):
    from torchless_b200 import ops
    import oracle
    v = golden_expected["vectors"]
    x, g = f32(v["norm_x"]), f32(v["norm_g"])
    ref = x.copy()
    oracle.oracle_lib().tlo_rmsnorm(ref.ctypes.data, g.ctypes.data, ref.size, 1e-5)
    xt = dev(x)
    ops.rmsnorm(xt, xt, dev(g))
    assert rel_err(host(xt), ref) <= 1e-5
    np.testing.assert_allclose(host(xt), v["norm_y"], atol=1e-4)


def test_argmax_rules():
    """sample_max: first strict max wins ties, NaN at index 0 pins 0, -inf everywhere gives 0."""
    from torchless_b200 import ops
    import oracle
    L = oracle.oracle_lib()
    rng = np.random.default_rng(4)
    cases = [f32([1, 3, 3, 2]), f32([np.nan, 3, 5]), f32([-np.inf] * 9), f32([7.0]),
             f32([0, np.nan, 1, 1]), f32(rng.standard_normal(32000)), f32(rng.standard_normal(1 << 20))]
    tie = f32(rng.standard_normal(32000)); tie[[5, 17000, 31999]] = 100.0
    cases.append(tie)
    for x in cases:
        want = L.tlo_argmax(x.ctypes.data, x.size)
        got = int(host(ops.argmax(dev(x)))[0])
        assert got == want, (x[:8], got, want)


@pytest.mark.parametrize("n,d", [(14336, 4096), (96, 1024), (10, 192)])
def test_mlp_gate_up(n, d):
    from torchless_b200 import ops
    import oracle
    L = oracle.oracle_lib()
    rng = np.random.default_rng(n + d)
    q1 = rng.integers(-127, 128, (n, d), dtype=np.int8)
    q3 = rng.integers(-127, 128, (n, d), dtype=np.int8)
    s1 = f32(np.abs(rng.standard_normal(n * d // 64)) * 40 + 40)
    s3 = f32(np.abs(rng.standard_normal(n * d // 64)) * 40 + 40)
    x = f32(rng.standard_normal(d))
    g = oracle_i8(q1, s1, x)
    L.tlo_silu(g.ctypes.data, g.ctypes.data, n)
    u = oracle_i8(q3, s3, x)
    ref = np.zeros(n, np.float32)
    L.tlo_mul(ref.ctypes.data, g.ctypes.data, u.ctypes.data, n)
    out = torch.zeros(n, device="cuda")
    ops.mlp_gate_up(out, dev(q1), dev(s1), dev(q3), dev(s3), dev(x))
    assert rel_err(host(out), ref) <= TOL


def test_quantize_bit_exact():
    """export_mistral.py:53-68 on the device equals the numpy/torch-CPU result bit for bit."""
    from torchless_b200 import ops
    from torchless_b200.binfmt import quantize_i8
    rng = np.random.default_rng(8)
    x = f32(rng.standard_normal((2048, 4096)) * 0.02)
    x[0, :64] = np.linspace(-1, 1, 64, dtype=np.float32)
    x[1, :64] *= 1e-30
    q, s = ops.quantize_i8(dev(x))
    q2, s2 = quantize_i8(x)
    np.testing.assert_array_equal(host(s), s2)
    np.testing.assert_array_equal(host(q), q2)


def test_bad_arguments_are_status_codes():
    import torchless_b200 as tb
    L = tb.lib()
    assert L.tl_matmul_i8(None, None, None, 0, None, 0, 0, None) == 1
    assert L.tl_quantize_i8(1, 1, 1, 100, 64, None) == 1  # numel not a multiple of the group
    assert b"multiple" in L.tl_last_error()
