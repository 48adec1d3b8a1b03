"""tl_argmax_noalloc (the allocation-free argmax) through the C ABI.

Its results must equal tl_argmax's (sample_max, main.cpp:10-21: first strict
maximum, NaN at index 0 gives 0) call after call, even though every call on a
device shares one fixed scratch array.  The file is named to be collected
last and must also pass on its own in a fresh process, where its first call
is the one that looks up the scratch address.
"""
import ctypes

import numpy as np
import pytest

from torchless_b200 import LIB_PATH, TL_OK, lib

TL_ERR_CAPACITY = 7
MAX_LOGITS = 512 * 1024  # the static scratch holds 512 partials of 1024 logits


def test_noalloc_rejects_oversize_before_any_device_work():
    """n beyond the scratch limit is refused from the arguments alone."""
    import os
    if not os.path.exists(LIB_PATH):
        pytest.skip("library not built")
    out = ctypes.c_void_p(16)
    x = ctypes.c_void_p(16)
    st = lib().tl_argmax_noalloc(out, x, MAX_LOGITS + 1, None)
    assert st == TL_ERR_CAPACITY
    msg = lib().tl_last_error().decode()
    assert "524288" in msg and "tl_argmax" in msg


@pytest.mark.gpu
def test_noalloc_matches_tl_argmax_on_consecutive_calls():
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.set_device(0)
    L = lib()
    stream = torch.cuda.current_stream().cuda_stream

    def both(logits_np):
        x = torch.from_numpy(np.ascontiguousarray(logits_np, dtype=np.float32)).cuda()
        a = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        b = torch.full((1,), -1, dtype=torch.int32, device="cuda")
        assert L.tl_argmax_noalloc(a.data_ptr(), x.data_ptr(), x.numel(), stream) == TL_OK, \
            L.tl_last_error().decode()
        assert L.tl_argmax(b.data_ptr(), x.data_ptr(), x.numel(), stream) == TL_OK, \
            L.tl_last_error().decode()
        torch.cuda.synchronize()
        return int(a.item()), int(b.item())

    rng = np.random.default_rng(11)
    # Call 1: many partials, a huge maximum late in the vector.
    big = rng.standard_normal(300_000).astype(np.float32)
    big[250_001] = 1e30
    # Call 2, right after: fewer partials; the stale ones of call 1 (which
    # hold 1e30) must not be read.  Its maximum is tied across two partials.
    small = rng.standard_normal(32_000).astype(np.float32)
    small[9_000] = small[20_000] = 50.0
    r1 = both(big)
    r2 = both(small)
    assert r1 == (250_001, 250_001)
    assert r2 == (9_000, 9_000)

    # The limit itself, one element, and NaN at index 0.
    edge = rng.standard_normal(MAX_LOGITS).astype(np.float32)
    edge[MAX_LOGITS - 1] = 99.0
    assert both(edge) == (MAX_LOGITS - 1, MAX_LOGITS - 1)
    assert both(np.array([3.0], dtype=np.float32)) == (0, 0)
    nan0 = rng.standard_normal(5000).astype(np.float32)
    nan0[0] = np.nan
    nan0[4000] = 10.0
    assert both(nan0) == (0, 0)
    allneg = np.full(4096, -np.inf, dtype=np.float32)
    assert both(allneg) == (0, 0)

    # Oversize is refused on the GPU too, and leaves the previous result alone.
    x = torch.zeros(MAX_LOGITS + 1, dtype=torch.float32, device="cuda")
    o = torch.full((1,), 123, dtype=torch.int32, device="cuda")
    assert L.tl_argmax_noalloc(o.data_ptr(), x.data_ptr(), x.numel(), stream) == TL_ERR_CAPACITY
    torch.cuda.synchronize()
    assert int(o.item()) == 123


@pytest.mark.gpu
def test_noalloc_takes_no_device_memory():
    """The call allocates nothing stream-ordered: the high watermark of the
    device's default memory pool (the pool tl_argmax's cudaMallocAsync draws
    from) stays at zero over repeated calls, while one tl_argmax call raises
    it, which shows that the probe sees such allocations.  The watermark is
    per pool, so other processes on the GPU do not move it."""
    torch = pytest.importorskip("torch")
    rt = pytest.importorskip("cuda.bindings.runtime")
    drv = pytest.importorskip("cuda.bindings.driver")
    torch.cuda.set_device(0)
    L = lib()
    stream = torch.cuda.current_stream().cuda_stream
    x = torch.randn(100_000, device="cuda")
    o = torch.empty(1, dtype=torch.int32, device="cuda")
    err, pool = rt.cudaDeviceGetDefaultMemPool(0)
    assert err == rt.cudaError_t.cudaSuccess
    high = rt.cudaMemPoolAttr.cudaMemPoolAttrUsedMemHigh

    def reset_high():
        torch.cuda.synchronize()
        (e,) = rt.cudaMemPoolSetAttribute(pool, high, drv.cuuint64_t(0))
        assert e == rt.cudaError_t.cudaSuccess

    def used_high():
        torch.cuda.synchronize()
        e, v = rt.cudaMemPoolGetAttribute(pool, high)
        assert e == rt.cudaError_t.cudaSuccess
        return int(v)

    assert L.tl_argmax_noalloc(o.data_ptr(), x.data_ptr(), x.numel(), stream) == TL_OK  # set-up call
    reset_high()
    assert L.tl_argmax(o.data_ptr(), x.data_ptr(), x.numel(), stream) == TL_OK
    assert used_high() > 0, "the allocating tl_argmax should show in the pool's watermark"
    reset_high()
    for _ in range(50):
        assert L.tl_argmax_noalloc(o.data_ptr(), x.data_ptr(), x.numel(), stream) == TL_OK
    assert used_high() == 0
    assert int(o.item()) == int(torch.argmax(x).item())
