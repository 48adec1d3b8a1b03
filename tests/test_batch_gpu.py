"""Batched decoding (tl_batch_*) through the C ABI, against the oracle.

B sequences share the weights; each has its own pre-filled KV cache (N(0, 1)
rows from the counter-based generator) and position.  For chosen sequences the
oracle gets the same cache rows (read back from the device), runs
Model<int8_t>::forward for the sequence's token, and the batch row must match:
logits within the parity rule (max rel err <= 1e-2; fp16 operands on the
batched path give ~1e-3), argmax identical unless the oracle's top-2 margin is a
near-tie.  Two consecutive steps check the KV append and the position advance.
"""
import numpy as np
import pytest

from conftest import rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
TOL = 1e-2
TIE = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


def margin(logits):
    top = np.sort(logits)[-2:]
    return float(top[1] - top[0]) / max(float(np.max(np.abs(logits))), 1e-30)


def oracle_for(buf, batch, seq, n_pos, max_seq):
    import oracle
    from torchless_b200.binfmt import ModelFile
    om = oracle.OracleModel(ModelFile(buf), max_seq=max_seq)
    for layer in range(batch.model.config["n_layers"]):
        for p in range(n_pos):
            k, v = batch.read_kv(seq, layer, p)
            om.write_kv(layer, p, k, v)
    om.pos = n_pos
    return om


def run_case(buf, n_seq, n_pos, check, max_seq, weights_f16=False):
    from torchless_b200 import Batch, Model
    m = Model.from_buffer(buf, max_seq=max_seq, weights_f16=weights_f16)
    b = Batch(m, n_seq)
    b.fill_kv_random(seed=1234, n_pos=n_pos)
    vocab = m.config["vocab_size"]
    rng = np.random.default_rng(n_seq + n_pos)
    toks = rng.integers(0, vocab, n_seq).tolist()
    oms = {s: oracle_for(buf, b, s, n_pos, max_seq) for s in check}
    worst = 0.0
    for step in range(2):
        lg, nxt = b.step(toks)
        for s in check:
            ref = oms[s].forward(toks[s])
            e = rel_err(lg[s], ref)
            worst = max(worst, e)
            assert e <= TOL, (step, s, e)
            if nxt[s] != int(np.argmax(ref)):
                assert margin(ref) < TIE, (step, s)
            # the row this step appended to the sequence's cache
            for layer in range(m.config["n_layers"]):
                k, v = b.read_kv(s, layer, n_pos + step)
                ko, vo = oms[s].read_kv(layer, n_pos + step)
                assert rel_err(k, ko) <= TOL and rel_err(v, vo) <= TOL, (step, s, layer)
        toks = [int(t) for t in nxt]  # the oracle is fed the same tokens on the next step
    b.close()
    m.close()
    return worst


@pytest.mark.parametrize("weights_f16", [False, True], ids=["int8_in_place", "f16_copies"])
def test_batch_small_matches_oracle(small_bin, weights_f16):
    worst = run_case(small_bin, n_seq=4, n_pos=40, check=[0, 3], max_seq=64, weights_f16=weights_f16)
    print(f"batch small ({'f16 copies' if weights_f16 else 'int8 in place'}): worst logits rel err {worst:.2e}")


def test_batch_7b_shapes_matches_oracle():
    from torchless_b200 import ops, synthetic as S
    cfg = dict(S.MISTRAL_7B, num_hidden_layers=2)
    buf = S.make_torch_model(cfg, seed=17, norm="random", device="cuda",
                             quantizer=lambda x: ops.quantize_i8(x)).buf
    worst = run_case(buf, n_seq=8, n_pos=200, check=[0, 7], max_seq=256)
    print(f"batch 7b shapes: worst logits rel err {worst:.2e}")
