"""fp8 (e5m2) weights on the device: the standalone matmul op and every decode
path (persistent, per-op, prefill, batched, tensor-parallel) against the
oracle, which runs each fp8 tensor through its e5m2 matmul (kernels.cpp:21-33
with get() = the e5m2 value).  fp8 is a format extension after the roadmap
item README.md:160; the file carries the cast, no scales."""
import os
import tempfile

import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TIE = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)


@pytest.fixture(scope="module", params=[False, True], ids=["lm_f32", "lm_fp8"])
def small_f8_bin(request):
    from torchless_b200 import synthetic as S
    return S.make_numpy_model(S.SMALL, seed=3, norm="random", quant="fp8", quant_lm_head=request.param).buf


def margin(logits):
    top = np.sort(logits)[-2:]
    return float(top[1] - top[0]) / max(float(np.max(np.abs(logits))), 1e-30)


@pytest.mark.parametrize("n,d", [(512, 1024), (1000, 4096), (96, 14336), (37, 200)])
def test_matmul_f8_op(n, d):
    """ops.matmul with float8_e5m2 weights (the fused GEMV where d is a multiple
    of 512, else one warp per row) vs the oracle's sequential fp32 sum."""
    import oracle
    from torchless_b200 import ops
    g = torch.Generator().manual_seed(n * 7 + d)
    w = (torch.randn(n, d, generator=g) * 0.05).to(torch.float8_e5m2)
    x = torch.randn(d, generator=g)
    y = torch.zeros(n, device="cuda")
    ops.matmul(y, w.cuda(), x.cuda())
    torch.cuda.synchronize()
    wb = w.view(torch.uint8).numpy()
    ref = np.zeros(n, dtype=np.float32)
    xn = x.numpy()
    oracle.oracle_lib().tlo_matmul_f8(ref.ctypes.data, wb.ctypes.data, xn.ctypes.data, n, d)
    assert rel_err(y.cpu().numpy(), ref) < 1e-5


@pytest.mark.parametrize("mode", [0, 1])
def test_decode_matches_oracle(small_f8_bin, mode):
    """Persistent kernel (fp16-plane activations x e5m2 tiles on the tensor
    cores) and per-op GEMVs, 24 greedy steps."""
    import oracle
    from torchless_b200 import Model
    from torchless_b200.binfmt import ModelFile
    mf = ModelFile(small_f8_bin)
    assert mf.tensors["model.layers.0.mlp.down_proj.weight"].dtype == "fp8"
    om = oracle.OracleModel(mf, max_seq=64)
    m = Model.from_buffer(small_f8_bin, max_seq=64, kernel_mode=mode)
    tok, worst = 11, 0.0
    for step in range(24):
        ref = om.forward(tok)
        got, nxt = m.forward(tok)
        e = rel_err(got, ref)
        worst = max(worst, e)
        assert e < 1e-4, (step, e)
        if nxt != int(np.argmax(ref)):
            assert margin(ref) < TIE, step
        tok = nxt
    print(f"fp8, lm {mf.tensors['lm_head.weight'].dtype}, kernel_mode {mode}: worst logits rel err {worst:.2e}")
    m.close()
    om.close()


def test_prefill_and_batch_match_oracle(small_f8_bin):
    """The batched paths run the fp16 GEMMs on weights widened exactly from e5m2."""
    import oracle
    from torchless_b200 import Batch, Model
    from torchless_b200.binfmt import ModelFile
    prompt = np.random.default_rng(4).integers(0, 1000, 17).tolist()
    om = oracle.OracleModel(ModelFile(small_f8_bin), max_seq=64)
    for t in prompt:
        ref = om.forward(t)
    m = Model.from_buffer(small_f8_bin, max_seq=64)
    lg, first = m.prefill(prompt)
    assert rel_err(lg, ref) < 5e-3
    assert first == int(np.argmax(ref)) or margin(ref) < TIE
    # decode continues from the prefilled caches
    ref = om.forward(first)
    got, _ = m.forward(first)
    assert rel_err(got, ref) < 5e-3
    m.close()
    om.close()
    m = Model.from_buffer(small_f8_bin, max_seq=64)
    b = Batch(m, 2)
    b.fill_kv_random(1, 0)
    oms = [oracle.OracleModel(ModelFile(small_f8_bin), max_seq=64) for _ in range(2)]
    toks = [5, 900]
    for step in range(4):
        lg, nxt = b.step(toks)
        for q in range(2):
            ref = oms[q].forward(toks[q])
            assert rel_err(lg[q], ref) < 1e-2, (step, q)
        toks = nxt.tolist()
    b.close()
    m.close()


def test_mistral7b_shapes_two_layers():
    """Mistral-7B shapes (2 layers), fp8 projections and lm_head cast on the
    device: 8192-byte e5m2 tiles through every phase of the persistent step."""
    import oracle
    from torchless_b200 import Model, synthetic as S
    from torchless_b200.binfmt import ModelFile
    cfg = dict(S.MISTRAL_7B, num_hidden_layers=2)
    buf = S.make_torch_model(cfg, seed=13, norm="random", device="cuda", quant="fp8", quant_lm_head=True).buf
    om = oracle.OracleModel(ModelFile(buf), max_seq=16)
    m = Model.from_buffer(buf, max_seq=16)
    for step, t in enumerate([17, 31000, 2, 4096]):
        ref = om.forward(t)
        got, nxt = m.forward(t)
        e = rel_err(got, ref)
        assert e < 1e-4, (step, e)
        if nxt != int(np.argmax(ref)):
            assert margin(ref) < TIE
    m.close()


def test_tp2_matches_oracle():
    """2 ranks, fp8 weights sliced like int8 (bytes), against the oracle."""
    import oracle
    from test_tp_gpu import _need, run_tp
    from torchless_b200 import synthetic as S
    from torchless_b200.binfmt import ModelFile
    _need(2)
    buf = S.make_numpy_model(S.SMALL, seed=3, norm="random", quant="fp8").buf
    feed = [11, 500, 3, 999, 42, 7]
    om = oracle.OracleModel(ModelFile(buf), max_seq=64)
    refs = [om.forward(t) for t in feed]
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "small_fp8.bin")
        buf.tofile(path)
        logits, toks = run_tp(path, feed)
    assert toks[0] == toks[1]
    for step, ref in enumerate(refs):
        assert rel_err(logits[step], ref) < 1e-4, step
