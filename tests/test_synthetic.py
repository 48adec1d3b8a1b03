"""The seeded workload generator (synthetic.make_seeded_model): its bytes are
a function of the seed and the shapes only, not of the thread count, and
each row block is the export_mistral.py quantisation of its own PCG64 draws."""
import numpy as np

from torchless_b200 import synthetic as S
from torchless_b200.binfmt import ModelFile, quantize_i8


def test_seeded_model_independent_of_threads():
    cfg = dict(S.SMALL, num_hidden_layers=1)
    a = S.make_seeded_model(cfg, seed=5, threads=1).buf
    b = S.make_seeded_model(cfg, seed=5, threads=4).buf
    assert np.array_equal(a, b)
    assert S.model_digest(a) == S.model_digest(b)
    c = S.make_seeded_model(cfg, seed=6, threads=4).buf
    assert S.model_digest(a) != S.model_digest(c)


def test_seeded_model_blocks_are_quantised_draws():
    cfg = dict(S.TINY, num_hidden_layers=1)
    mf = ModelFile(S.make_seeded_model(cfg, seed=9).buf)
    names = [n for n, _ in S.tensor_list(cfg)]
    t = names.index("model.layers.0.mlp.down_proj.weight")
    rows, cols = mf.tensors[names[t]].shape
    per = max(1, S.CHUNK_ELEMS // cols)
    q, s = mf.tensor(names[t])
    # block 0 of the tensor: rows [0, per) from SeedSequence([seed, t, 0])
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([9, t, 0])))
    x = rng.standard_normal((min(per, rows), cols), dtype=np.float32) * np.float32(0.02)
    q0, s0 = quantize_i8(x)
    assert np.array_equal(q[:min(per, rows)], q0)
    assert np.array_equal(s[:q0.size // 64], s0)
    # norms are ones, embedding / lm_head fp32 draws
    g, _ = mf.tensor("model.layers.0.input_layernorm.weight")
    assert np.all(g == 1.0)
    emb, sc = mf.tensor("model.embed_tokens.weight")
    assert sc is None and emb.dtype == np.float32 and 0.015 < float(emb.std()) < 0.025
