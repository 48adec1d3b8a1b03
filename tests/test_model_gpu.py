"""Model-level parity of the CUDA path against the reference (through the C ABI).

Parity rule, per decode step:
  * logits: max|gpu - ref| / max|ref| <= 1e-2 (the stated tolerance; the
    measured error is reported and is orders of magnitude smaller);
  * greedy ids identical.  Where the reference's top-2 logit margin is below
    1e-3 * max|logit| the step is a near-tie: it is recorded, and the
    comparison continues teacher-forced on the reference's token.
The GPU model is always fed the reference's own token sequence, so a
near-tie cannot derail later steps.
"""
import numpy as np
import pytest

from conftest import golden_greedy, rel_err

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-2
TIE = 1e-3

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"


MODES = {"persistent": 0, "per_op": 1}


def load(buf, **kw):
    from torchless_b200 import Model
    return Model.from_buffer(buf, **kw)


def margin(logits):
    top = np.sort(logits)[-2:]
    return float(top[1] - top[0]) / max(float(np.max(np.abs(logits))), 1e-30)


def check_teacher_forced(model, prompt, ids, ref_logits):
    """Feeds prompt[:-1], then prompt[-1], ids[0], ids[1], ...; compares each step."""
    model.pos = 0
    for t in prompt[:-1]:
        model.forward(t, logits=False)
    feed = [prompt[-1]] + list(ids[:-1])
    worst, near_ties = 0.0, []
    for step, tok in enumerate(feed):
        lg, nxt = model.forward(tok)
        e = rel_err(lg, ref_logits[step])
        worst = max(worst, e)
        assert e <= LOGIT_TOL, f"step {step}: logits rel err {e}"
        if nxt != ids[step]:
            assert margin(ref_logits[step]) < TIE, f"step {step}: token {nxt} != {ids[step]} without a near-tie"
            near_ties.append(step)
    return worst, near_ties


@pytest.mark.parametrize("mode", list(MODES))
@pytest.mark.parametrize("name", ["tiny", "small"])
def test_greedy_matches_reference(name, mode, request):
    prompt, ids, logits = golden_greedy(name)
    m = load(request.getfixturevalue(f"{name}_bin"), max_seq=64, kernel_mode=MODES[mode])
    worst, ties = check_teacher_forced(m, prompt, ids, logits)
    print(f"{name}/{mode}: worst logits rel err {worst:.2e}, near-ties {ties}")
    assert worst < 1e-4  # the CUDA path is far inside the stated bound
    # the on-device greedy loop (main.cpp:69-77) reproduces the reference ids
    m.pos = 0
    assert m.generate(prompt, len(ids)) == ids or ties
    m.close()


@pytest.mark.parametrize("mode", list(MODES))
def test_graph_and_eager_agree(small_bin, mode):
    prompt, ids, logits = golden_greedy("small")
    a = load(small_bin, max_seq=64, use_graph=True, kernel_mode=MODES[mode])
    b = load(small_bin, max_seq=64, use_graph=False, kernel_mode=MODES[mode])
    for t in prompt + ids[:8]:
        la, na = a.forward(t)
        lb, nb = b.forward(t)
        np.testing.assert_array_equal(la, lb)
        assert na == nb
    a.close()
    b.close()


def test_layer_and_kv_push_match_oracle(small_bin):
    """Layer<T>::forward over 3 tokens (test_modules.cpp:3-24) and push_kv (:99-127)."""
    import oracle
    from torchless_b200.binfmt import ModelFile
    om = oracle.OracleModel(ModelFile(small_bin), max_seq=64)
    m = load(small_bin, max_seq=64)
    rng = np.random.default_rng(0)
    for pos in range(3):
        h = rng.standard_normal(m.config["hidden_size"]).astype(np.float32)
        om.pos = pos
        m.pos = pos
        for layer in (0, 1):
            want = om.layer_forward(layer, h)
            got = m.layer_forward(layer, h)
            assert rel_err(got, want) <= 1e-4, (pos, layer)
    # push_kv: the rotated k and raw v of each token sit at (layer, pos)
    for layer in (0, 1):
        for pos in range(3):
            k, v = m.read_kv(layer, pos)
            ko, vo = om.read_kv(layer, pos)
            assert rel_err(k, ko) <= 1e-4 and rel_err(v, vo) <= 1e-4, (layer, pos)
    m.close()


@pytest.mark.parametrize("mode", list(MODES))
def test_capacity_and_token_errors(tiny_bin, mode):
    from torchless_b200 import TLError
    m = load(tiny_bin, max_seq=4, kernel_mode=MODES[mode])
    for t in range(4):
        m.forward(t, logits=False)
    with pytest.raises(TLError) as e:
        m.forward(0)
    assert e.value.status == 7  # TL_ERR_CAPACITY (the reference overruns silently)
    m.pos = 0
    with pytest.raises(TLError) as e:
        m.forward(10**6)
    assert e.value.status == 1
    m.close()


@pytest.fixture(scope="module")
def m7b_two_layers():
    """Mistral-7B layer shapes (D 4096, F 14336, 32/8 heads, V 32000) with 2 layers."""
    from torchless_b200 import synthetic as S
    from torchless_b200 import ops
    cfg = dict(S.MISTRAL_7B, num_hidden_layers=2)
    return S.make_torch_model(cfg, seed=11, norm="random", device="cuda",
                              quantizer=lambda x: ops.quantize_i8(x)).buf


@pytest.mark.parametrize("mode", list(MODES))
def test_mistral7b_shapes_two_layers(m7b_two_layers, mode):
    """Every kernel at its real size against the oracle, 6 steps."""
    import oracle
    from torchless_b200.binfmt import ModelFile
    om = oracle.OracleModel(ModelFile(m7b_two_layers), max_seq=32)
    m = load(m7b_two_layers, max_seq=32, kernel_mode=MODES[mode])
    rng = np.random.default_rng(1)
    toks = rng.integers(0, 32000, 6).tolist()
    for step, t in enumerate(toks):
        ref = om.forward(t)
        got, nxt = m.forward(t)
        e = rel_err(got, ref)
        assert e <= LOGIT_TOL, (step, e)
        assert e < 1e-4, (step, e)
        if nxt != int(np.argmax(ref)):
            assert margin(ref) < TIE
    m.close()


# Persistent-kernel attention variants: per-head CTAs (the default below
# 1024 positions), and GQA CTAs (one per kv group and split) from the first
# position with 16 positions per split, so 200 positions run up to 13 splits
# merged by the last split of each group.
ATTN_ENV = {"per_head": {}, "gqa": {"TL_DECODE_GQA_FROM": "0", "TL_DECODE_GQA_ROWS": "16"}}


@pytest.mark.parametrize("attn", list(ATTN_ENV))
def test_persistent_and_per_op_agree_at_long_positions(small_bin, attn, monkeypatch):
    """Both decode paths over 200 positions (attention spans many splits)."""
    for k, v in ATTN_ENV[attn].items():
        monkeypatch.setenv(k, v)
    a = load(small_bin, max_seq=256, kernel_mode=0)
    b = load(small_bin, max_seq=256, kernel_mode=1)
    rng = np.random.default_rng(5)
    toks = rng.integers(0, 1000, 200).tolist()
    worst = 0.0
    for t in toks:
        la, _ = a.forward(t)
        lb, _ = b.forward(t)
        worst = max(worst, rel_err(la, lb))
    assert worst < 1e-4, worst
    for layer, pos in [(0, 0), (1, 99), (1, 199)]:  # KV pushed by both paths
        ka, va = a.read_kv(layer, pos)
        kb, vb = b.read_kv(layer, pos)
        assert rel_err(ka, kb) < 1e-5 and rel_err(va, vb) < 1e-5, (layer, pos)
    a.close()
    b.close()


def test_gqa_attention_mistral7b_shapes(m7b_two_layers, monkeypatch):
    """GQA attention at Mistral-7B head counts (8 kv groups x 4 q heads) with
    up to 5 splits per group, against the per-op path, 40 steps."""
    monkeypatch.setenv("TL_DECODE_GQA_FROM", "0")
    monkeypatch.setenv("TL_DECODE_GQA_ROWS", "8")
    a = load(m7b_two_layers, max_seq=64, kernel_mode=0)
    b = load(m7b_two_layers, max_seq=64, kernel_mode=1)
    rng = np.random.default_rng(9)
    worst = 0.0
    for t in rng.integers(0, 32000, 40).tolist():
        la, _ = a.forward(t)
        lb, _ = b.forward(t)
        worst = max(worst, rel_err(la, lb))
    assert worst < 1e-4, worst
    a.close()
    b.close()
