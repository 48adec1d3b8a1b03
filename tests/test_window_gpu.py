"""Sliding-window attention (opt-in; the reference attends to every cached
position, modules.cpp:75-83): with window W the query at position p attends to
positions (p - W, p].  Every attention path against the oracle with the same
window (tlo_config.window: the oracle's attention restricted to those rows)."""
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


def margin(logits):
    top = np.sort(logits)[-2:]
    return float(top[1] - top[0]) / max(float(np.max(np.abs(logits))), 1e-30)


def oracle(buf, window, max_seq=96):
    import oracle as O
    from torchless_b200.binfmt import ModelFile
    return O.OracleModel(ModelFile(buf), max_seq=max_seq, window=window)


# persistent per-head attention, per-op kernels, and the GQA path (every
# position, 8 positions per split, so a 24-position window spans 3 splits that
# start at the window's lower bound)
CASES = {"persistent": (0, {}), "per_op": (1, {}),
         "gqa": (0, {"TL_DECODE_GQA_FROM": "0", "TL_DECODE_GQA_ROWS": "8"})}


@pytest.mark.parametrize("case", list(CASES))
@pytest.mark.parametrize("window", [8, 24])
def test_decode_matches_windowed_oracle(small_bin, case, window, monkeypatch):
    from torchless_b200 import Model
    mode, env = CASES[case]
    for k, v in env.items():
        monkeypatch.setenv(k, v)
    om = oracle(small_bin, window)
    full = oracle(small_bin, 0)
    m = Model.from_buffer(small_bin, max_seq=96, kernel_mode=mode, sliding_window=window)
    tok, worst, differs = 3, 0.0, 0.0
    for step in range(60):
        ref = om.forward(tok)
        differs = max(differs, rel_err(full.forward(tok), ref))
        got, nxt = m.forward(tok)
        e = rel_err(got, ref)
        worst = max(worst, e)
        assert e < 1e-4, (step, e)
        if nxt != int(np.argmax(ref)):
            assert margin(ref) < TIE, step
        tok = nxt
    assert differs > 1e-3  # the window changed the results past W positions
    print(f"window {window} {case}: worst logits rel err {worst:.2e}")
    m.close()


@pytest.mark.parametrize("chunks", [[40], [23, 17]])
def test_prefill_then_decode_matches_windowed_oracle(small_bin, chunks):
    """Causal prefill with the window (one pass, or two passes: the second
    starts at p0 > 0), its KV rows, then decode from the cache."""
    from torchless_b200 import Model
    W = 12
    prompt = np.random.default_rng(6).integers(0, 1000, sum(chunks)).tolist()
    om = oracle(small_bin, W)
    for t in prompt:
        ref = om.forward(t)
    m = Model.from_buffer(small_bin, max_seq=96, sliding_window=W)
    i = 0
    for n in chunks:
        lg, first = m.prefill(prompt[i:i + n])
        i += n
    assert rel_err(lg, ref) < 5e-3
    assert first == int(np.argmax(ref)) or margin(ref) < TIE
    for layer, p in [(0, 5), (1, len(prompt) - 1)]:
        k, v = m.read_kv(layer, p)
        ko, vo = om.read_kv(layer, p)
        assert rel_err(k, np.asarray(ko)) < 5e-3 and rel_err(v, np.asarray(vo)) < 5e-3
    tok = first
    for step in range(8):
        ref = om.forward(tok)
        got, nxt = m.forward(tok)
        assert rel_err(got, ref) < 5e-3, step
        tok = int(np.argmax(ref))
        if nxt != tok:
            assert margin(ref) < TIE
    m.close()


def test_batch_matches_windowed_oracle(small_bin):
    """Batched decode with the window: two sequences with 30 pre-filled
    positions, window 10, against the oracle given the same cache rows."""
    import oracle as O
    from torchless_b200 import Batch, Model
    from torchless_b200.binfmt import ModelFile
    W, n_pos = 10, 30
    m = Model.from_buffer(small_bin, max_seq=64, sliding_window=W)
    b = Batch(m, 2)
    b.fill_kv_random(seed=77, n_pos=n_pos)
    oms = []
    for s in range(2):
        om = O.OracleModel(ModelFile(small_bin), max_seq=64, window=W)
        for layer in range(m.config["n_layers"]):
            for p in range(n_pos):
                k, v = b.read_kv(s, layer, p)
                om.write_kv(layer, p, k, v)
        om.pos = n_pos
        oms.append(om)
    toks = [12, 345]
    for step in range(3):
        lg, nxt = b.step(toks)
        for s in range(2):
            ref = oms[s].forward(toks[s])
            assert rel_err(lg[s], ref) < 1e-2, (step, s)
        toks = nxt.tolist()
    b.close()
    m.close()
