"""tcgen05 GEMM of the batched paths (tl_gemm_f16) against a torch fp32 reference.

fp16 operands are exact in fp32, so the only difference from A.float() @ B.float().T
is the fp32 accumulation order: max |err| / max |ref| <= 1e-5.
"""
import ctypes

import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TOL = 1e-5


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)


def gemm(c, a, b, m, n, k, ldc, epi):
    from torchless_b200 import check, lib
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    check(lib().tl_gemm_f16(c.data_ptr(), a.data_ptr(), b.data_ptr(), m, n, k, ldc, epi, s))
    torch.cuda.synchronize()


def rel(x, y):
    return float((x.double() - y.double()).abs().max() / y.double().abs().max())


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (300, 520, 192), (77, 1000, 512), (2048, 4096, 4096)])
def test_store_and_add(m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randn(m, k, device="cuda", generator=g).half()
    b = (torch.randn(n, k, device="cuda", generator=g) * 0.05).half()
    ref = a.float() @ b.float().T
    c = torch.full((m, n), float("nan"), device="cuda")
    gemm(c, a, b, m, n, k, n, 0)
    assert rel(c, ref) <= TOL
    base = torch.randn(m, n, device="cuda", generator=g)
    c2 = base.clone()
    gemm(c2, a, b, m, n, k, n, 1)
    assert rel(c2, base + ref) <= TOL


@pytest.mark.parametrize("m,f,k", [(64, 128, 256), (200, 384, 1024)])
def test_swiglu(m, f, k):
    g = torch.Generator(device="cuda").manual_seed(f + k)
    a = torch.randn(m, k, device="cuda", generator=g).half()
    gate = (torch.randn(f, k, device="cuda", generator=g) * 0.05).half()
    up = (torch.randn(f, k, device="cuda", generator=g) * 0.05).half()
    # blocks of 256 rows: 128 gate rows then the matching 128 up rows
    b = torch.cat([torch.cat([gate[i:i + 128], up[i:i + 128]]) for i in range(0, f, 128)]).contiguous()
    gv, uv = a.float() @ gate.float().T, a.float() @ up.float().T
    ref = gv / (1.0 + torch.exp(-gv)) * uv
    out = torch.zeros(m, f, device="cuda", dtype=torch.float16)
    gemm(out, a, b, m, 2 * f, k, f, 2)
    assert rel(out.float(), ref) <= 2e-3  # fp16 output rounding


# ---- tl_gemm_q8: 8-bit weights dequantised inside the GEMM -------------------
def gemm_q8(c, a, q, inv_t, q2, inv_t2, m, n, k, ldc, epi):
    from torchless_b200 import check, lib
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    check(lib().tl_gemm_q8(c.data_ptr(), a.data_ptr(), q.data_ptr(), p(inv_t), p(q2), p(inv_t2), m, n, k, ldc, epi, s))
    torch.cuda.synchronize()


def int8_weights(n, k, g):
    """int8 [n, k] in [-127, 127], 1/s per 64-group [n, k/64], and the fp16
    values the kernel multiplies: fp16(q) * fp16(1/s) rounded to fp16
    (tensor.cpp:101-104's dequantisation in fp16 arithmetic)."""
    q = torch.randint(-127, 128, (n, k), dtype=torch.int8, device="cuda", generator=g)
    inv = torch.rand(n, k // 64, device="cuda", generator=g) * 1e-3 + 1e-4
    w16 = (q.half().view(n, k // 64, 64) * inv.half().view(n, k // 64, 1)).view(n, k)
    return q, inv, w16


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (300, 520, 192), (77, 1000, 512), (64, 4096, 4096),
                                   (2048, 4096, 4096)])
def test_q8_store_and_add(m, n, k):
    g = torch.Generator(device="cuda").manual_seed(7 * m + n + k)
    a = torch.randn(m, k, device="cuda", generator=g).half()
    q, inv, w16 = int8_weights(n, k, g)
    inv_t = inv.T.contiguous()  # [k / 64][n]
    ref = a.float() @ w16.float().T
    c = torch.full((m, n), float("nan"), device="cuda")
    gemm_q8(c, a, q, inv_t, None, None, m, n, k, n, 0)
    assert rel(c, ref) <= TOL
    base = torch.randn(m, n, device="cuda", generator=g)
    c2 = base.clone()
    gemm_q8(c2, a, q, inv_t, None, None, m, n, k, n, 1)
    assert rel(c2, base + ref) <= TOL


@pytest.mark.parametrize("m,f,k", [(64, 128, 256), (200, 384, 1024)])
def test_q8_swiglu(m, f, k):
    g = torch.Generator(device="cuda").manual_seed(3 * f + k)
    a = torch.randn(m, k, device="cuda", generator=g).half()
    qg, ig, gate = int8_weights(f, k, g)
    qu, iu, up = int8_weights(f, k, g)
    gv, uv = a.float() @ gate.float().T, a.float() @ up.float().T
    ref = gv / (1.0 + torch.exp(-gv)) * uv
    out = torch.zeros(m, f, device="cuda", dtype=torch.float16)
    gemm_q8(out, a, qg, ig.T.contiguous(), qu, iu.T.contiguous(), m, 2 * f, k, f, 2)
    assert rel(out.float(), ref) <= 2e-3  # fp16 output rounding


def test_q8_e5m2_weights():
    """Null scales: the bytes are e5m2 weights, widened to fp16 exactly."""
    m, n, k = 96, 512, 256
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn(m, k, device="cuda", generator=g).half()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.05).to(torch.float8_e5m2)
    ref = a.float() @ w.float().T
    c = torch.zeros(m, n, device="cuda")
    gemm_q8(c, a, w.view(torch.uint8), None, None, None, m, n, k, n, 0)
    assert rel(c, ref) <= TOL
