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
