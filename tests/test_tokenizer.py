"""The model binary's tokenizer (tl_tokenizer_*) against the reference's own
Tokenizer (tokenizer.cpp): the committed fixture (tests/golden/ref_tokenizer.json,
made by the reference build from a synthetic BPE tokenizer), and the live
reference build when present.  Host code: no GPU."""
import json
import os

import numpy as np
import pytest

import oracle
from conftest import GOLDEN


@pytest.fixture(scope="module")
def fixture():
    with open(os.path.join(GOLDEN, "ref_tokenizer.json")) as f:
        return json.load(f)


def test_encode_decode_match_reference_fixture(fixture):
    from torchless_b200 import Tokenizer
    t = Tokenizer.from_json(fixture["tokenizer"])
    assert t.vocab_size == len(fixture["tokenizer"]["vocab"])
    for c in fixture["cases"]:
        text = bytes.fromhex(c["text"])
        assert t.encode(text) == c["ids"], text
        assert t.decode_bytes(c["ids"]).hex() == c["decoded"], text
    t.close()


def test_tokenizer_from_model_binary(fixture, tmp_path):
    """The header's tokenizer object, read from a model binary in memory and
    on disk (the header only), tokenizes like the JSON it was written from."""
    from torchless_b200 import Tokenizer, synthetic as S
    buf = S.make_numpy_model(S.TINY, seed=7, tokenizer=fixture["tokenizer"]).buf
    path = tmp_path / "m.bin"
    buf.tofile(path)
    a = Tokenizer.from_json(fixture["tokenizer"])
    for t in (Tokenizer.from_buffer(buf), Tokenizer.load(str(path))):
        for c in fixture["cases"][:20]:
            text = bytes.fromhex(c["text"])
            assert t.encode(text) == a.encode(text)
        t.close()


def test_errors_where_the_reference_is_undefined():
    """A byte-fallback piece or <s> missing from the vocabulary, an id outside
    it: errors (the reference dereferences a missing entry)."""
    from torchless_b200 import TLError, Tokenizer
    t = Tokenizer.from_json({"vocab": {"<s>": 0, "▁": 1, "a": 2}, "merges": []})
    assert t.encode("a a") == [0, 1, 2, 1, 2]
    with pytest.raises(TLError):
        t.encode("b")  # no <0x62> piece
    with pytest.raises(TLError):
        t.decode([7])
    t.close()
    t = Tokenizer.from_json({"vocab": {"▁": 0}, "merges": []})
    with pytest.raises(TLError):
        t.encode("")  # no <s>
    with pytest.raises(TLError):
        Tokenizer.from_json({"vocab": {"a": 5}})  # id past the vocabulary


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built here")
def test_random_texts_vs_live_reference():
    from torchless_b200 import Tokenizer, synthetic as S
    tok = S.make_bpe_tokenizer(n_merges=120)
    a, r = Tokenizer.from_json(tok), oracle.RefTokenizer(tok)
    rng = np.random.default_rng(33)
    alphabet = list("the model abé中\U0001F600 ▁") + ["\t", "x"]
    for _ in range(200):
        s = "".join(alphabet[int(i)] for i in rng.integers(0, len(alphabet), int(rng.integers(0, 40))))
        b = s.encode("utf-8")
        if rng.random() < 0.2:
            b += bytes([int(rng.integers(128, 256))])
        ids = r.encode(b)
        assert a.encode(b) == ids, b
        assert a.decode_bytes(ids) == r.decode_bytes(ids)
    a.close()
    r.close()


@pytest.mark.gpu
def test_generate_cli_matches_model_and_tokenizer(fixture, tmp_path):
    """python -m torchless_b200.generate: the printed text is the decode of the
    ids the model generates greedily after the encoded prompt."""
    import subprocess
    import sys
    from torchless_b200 import Model, Tokenizer, synthetic as S
    path = str(tmp_path / "m.bin")
    buf = S.make_numpy_model(dict(S.TINY, vocab_size=len(fixture["tokenizer"]["vocab"])), seed=7,
                             norm="random", tokenizer=fixture["tokenizer"]).buf
    buf.tofile(path)
    prompt = "the model reads"
    tok = Tokenizer.load(path)
    ids = tok.encode(prompt)
    m = Model.load(path, max_seq=64)
    m.prefill(ids[:-1], logits=False)  # as the CLI ingests the prompt
    t, want = ids[-1], []
    for _ in range(12):
        _, t = m.forward(t, logits=False)
        want.append(t)
    m.close()
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-m", "torchless_b200.generate", path, prompt, "--tokens", "12",
                        "--max-seq", "64"], capture_output=True, cwd=root, timeout=300)
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    text = b"".join(tok.decode_bytes([i]) for i in want).decode("utf-8", errors="replace") + "\n"
    assert r.stdout.decode("utf-8") == text
    tok.close()
