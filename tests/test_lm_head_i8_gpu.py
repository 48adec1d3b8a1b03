"""int8 lm_head (a format extension: the reference exporter keeps the lm_head
fp32, export_mistral.py:119): the same per-64-group int8 + scales layout as the
_proj tensors, marked by the tensor's dtype in the header.  Every decode path
against the oracle, which runs an int8 tensor through its int8 matmul
(kernels.cpp:21-33 restated)."""
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


@pytest.fixture(scope="module")
def small_i8_bin():
    from torchless_b200 import synthetic as S
    return S.make_numpy_model(S.SMALL, seed=3, norm="random", quant_lm_head=True).buf


def margin(logits):
    top = np.sort(logits)[-2:]
    return float(top[1] - top[0]) / max(float(np.max(np.abs(logits))), 1e-30)


@pytest.mark.parametrize("mode", [0, 1])
def test_decode_matches_oracle(small_i8_bin, mode):
    import oracle
    from torchless_b200 import Model
    from torchless_b200.binfmt import ModelFile
    mf = ModelFile(small_i8_bin)
    assert mf.tensors["lm_head.weight"].dtype == "int8"
    om = oracle.OracleModel(mf, max_seq=64)
    m = Model.from_buffer(small_i8_bin, max_seq=64, kernel_mode=mode)
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
    print(f"int8 lm_head, kernel_mode {mode}: worst logits rel err {worst:.2e}")
    m.close()
    om.close()


def test_prefill_and_batch_match_oracle(small_i8_bin):
    """The batched paths use an fp16 copy of the lm_head dequantised from int8."""
    import oracle
    from torchless_b200 import Batch, Model
    from torchless_b200.binfmt import ModelFile
    prompt = np.random.default_rng(4).integers(0, 1000, 17).tolist()
    om = oracle.OracleModel(ModelFile(small_i8_bin), max_seq=64)
    for t in prompt:
        ref = om.forward(t)
    m = Model.from_buffer(small_i8_bin, max_seq=64)
    lg, first = m.prefill(prompt)
    assert rel_err(lg, ref) < 5e-3
    assert first == int(np.argmax(ref)) or margin(ref) < TIE
    m.close()
    om.close()
    # batch: two fresh sequences (empty caches) against two oracle models
    m = Model.from_buffer(small_i8_bin, max_seq=64)
    b = Batch(m, 2)
    b.fill_kv_random(1, 0)
    oms = [oracle.OracleModel(ModelFile(small_i8_bin), max_seq=64) for _ in range(2)]
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
    """32000 x 4096 int8 lm_head tiles in the persistent step, 4 steps."""
    import oracle
    from torchless_b200 import Model, ops, synthetic as S
    from torchless_b200.binfmt import ModelFile
    cfg = dict(S.MISTRAL_7B, num_hidden_layers=2)
    buf = S.make_torch_model(cfg, seed=13, norm="random", device="cuda", quantizer=lambda x: ops.quantize_i8(x),
                             quant_lm_head=True).buf
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
