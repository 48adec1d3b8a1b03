"""Regenerates the golden fixtures in tests/golden/ from the reference itself.

Run in a container that has the reference tree, given by --reference or the
TORCHLESS_REFERENCE environment variable:

    python tests/golden/make_golden.py --reference <reference tree>

Writes:
  reference_expected.json  weight-independent vectors of the reference's own
                           fixture file test/mistral/expected.txt (inv_freq,
                           cos0/sin0/cos3/sin3, rope0..3, norm_x/norm_g/norm_y)
                           and the known-answer cases of
                           test/mistral/test_cpu_kernels.cpp:32-105.
  export_hashes.json       sha256 of the binaries produced by the reference's
                           own export_mistral.py for the seeded TINY and SMALL
                           models (torchless_b200.synthetic); the numpy writer
                           must reproduce them byte for byte.
  ref_greedy_<cfg>.npz     the reference's Model<int8_t> (oracle/_ref, built
                           from its own sources) on those models: prompt,
                           greedy ids and per-step logits.
  ref_ops.npz              reference kernels.cpp ops on seeded inputs.
  ref_tokenizer.json       the reference's Tokenizer (tokenizer.cpp) with the
                           synthetic BPE tokenizer of torchless_b200.synthetic:
                           the tokenizer object, then for fixed and seeded random
                           byte strings (words, multi-byte UTF-8, invalid bytes,
                           spaces) the ids encode() returns and the bytes decode()
                           returns for them.
  ref_sample.npz           the reference's sample_multinomial (main.cpp:23-43)
                           on TINY-vocabulary logits (the greedy fixture's plus
                           NaN / inf / tie / flat edge cases) at several
                           temperatures, its generator seeded: the uniform draw
                           r of each call and the index it returned.

The tests read only these files; nothing at test time touches the reference
tree.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from torchless_b200 import synthetic as S  # noqa: E402
from torchless_b200.binfmt import ModelFile  # noqa: E402

WEIGHT_INDEPENDENT = ["inv_freq", "cos0", "sin0", "cos3", "sin3", "rope0", "rope1", "rope2", "rope3",
                      "norm_x", "norm_g", "norm_y"]

# Seeds and sizes of the checked models (shared with tests/conftest.py).
MODELS = {"tiny": (S.TINY, 7), "small": (S.SMALL, 3)}
PROMPT_LEN, N_NEW = 16, 24
REF_TREE = None  # set from --reference / $TORCHLESS_REFERENCE in main()


def read_expected(path: str) -> dict:
    """Name line then value line, as load_expected_values (setup/context.cpp:22-39)."""
    out = {}
    with open(path) as f:
        lines = f.read().split("\n")
    i = 0
    while i < len(lines):
        name = lines[i].strip()
        i += 1
        if not name or name.startswith("#"):
            continue
        vals = [float(v) for v in lines[i].split()] if i < len(lines) else []
        i += 1
        out[name] = vals
    return out


def kats() -> dict:
    """Known answers written in test_cpu_kernels.cpp (file:line)."""
    return {
        "matmul": {"src": "test/mistral/test_cpu_kernels.cpp:32-48",
                   "w": [[1, 2, 3], [4, 5, 6]], "x": [10, 20, 30], "y": [140, 320]},
        "row_matmul": {"src": "test/mistral/test_cpu_kernels.cpp:50-68",
                       "w": [[1, 2], [3, 4], [5, 6]], "x": [10, 20, 30], "y": [220, 280]},
        "softmax": {"src": "test/mistral/test_cpu_kernels.cpp:71-85",
                    "x": [1.0, 2.0, 3.0], "y": [0.09003057, 0.24472848, 0.66524094]},
        "silu": {"src": "test/mistral/test_cpu_kernels.cpp:88-105",
                 "x": [-2.0, -1.0, 0.0, 1.0, 2.0], "y": [-0.2384, -0.2689, 0.0, 0.7311, 1.7616]},
        "rope_input": {"src": "test/mistral/test_cpu_kernels.cpp:4-29",
                       "rule": "q[i] = (i % 128) / 256, shape [1, 128], positions 0..3"},
        "tolerance": {"src": "test/mistral/setup/context.cpp:41-45", "atol": 5e-2},
    }


def sha256(b) -> str:
    return hashlib.sha256(bytes(b)).hexdigest()


def sample_fixture() -> None:
    """ref_sample.npz: main.cpp:23-43 through the reference build (oracle/_ref)."""
    oracle.build(reference=True, tree=REF_TREE)
    cfg, seed = MODELS["tiny"]
    V = cfg["vocab_size"]
    rm = oracle.RefModel(S.make_numpy_model(cfg, seed=seed, norm="random").buf, max_seq=16)
    sets = [l.astype(np.float32) for l in np.load(os.path.join(HERE, "ref_greedy_tiny.npz"))["logits"][:4]]
    base = sets[0]
    edge = []
    x = base.copy(); x[0] = np.nan; edge.append(x)                  # NaN at 0
    x = base.copy(); x[100] = np.nan; edge.append(x)                # NaN inside
    x = base.copy(); x[5] = np.inf; edge.append(x)                  # +inf
    x = np.full(V, -np.inf, np.float32); x[321] = 1.5; edge.append(x)  # one finite
    edge.append(np.full(V, -np.inf, np.float32))                    # all -inf
    edge.append((base * 1e30).astype(np.float32))                   # huge
    x = np.zeros(V, np.float32); x[[7, 8, 700]] = 3.0; edge.append(x)  # ties
    flat = np.zeros(V, np.float32); edge.append(flat)               # flat: running sum may stop short of r
    sets += edge
    temps = [0.0, -1.0, 0.3, 0.8, 1.0, 2.5]
    rows = []
    for j, lg in enumerate(sets):
        for temp in temps:
            for sd in range(6):
                idx, r = rm.sample_logits(lg, temp, 1000 * j + sd)
                rows.append((j, temp, 1000 * j + sd, r, idx))
    # seeds whose draw is within 1e-4 of 1, on the flat set (the last-index fallback)
    hi = [sd for sd in range(200000) if rm.sample_logits(flat, 1.0, sd)[1] > 0.9999][:6]
    for sd in hi:
        idx, r = rm.sample_logits(flat, 1.0, sd)
        rows.append((len(sets) - 1, 1.0, sd, r, idx))
    rm.close()
    a = np.array(rows, dtype=np.float64)
    np.savez_compressed(os.path.join(HERE, "ref_sample.npz"), logits=np.stack(sets),
                        set=a[:, 0].astype(np.int64), temp=a[:, 1].astype(np.float32),
                        seed=a[:, 2].astype(np.int64), r=a[:, 3].astype(np.float32), idx=a[:, 4].astype(np.int64))


def tokenizer_texts(seed: int = 21, n: int = 60):
    """Fixed strings, then seeded random byte strings."""
    fixed = ["the model reads its weights once", "", " ", "  two  spaces ", "caf\u00e9 \u4e2d\u6587 \U0001F600",
             "Unknown Words Here", "tokenizer tokens token", "a", "the", "e "]
    out = [t.encode("utf-8") for t in fixed] + [b"\xff\xfe\x80 raw", b"\xe4\xb8", b"abc\xf0"]
    rng = np.random.default_rng(seed)
    words = S.TOKENIZER_CORPUS.split()
    extra = ["\u00e9", "\u00df", "\u4e2d", "\u6587", "\U0001F600", "\u2581", "Z", "Q", "\t", "7"]
    for _ in range(n):
        parts = []
        for _ in range(int(rng.integers(1, 12))):
            r = rng.random()
            if r < 0.6:
                parts.append(words[int(rng.integers(len(words)))].encode("utf-8"))
            elif r < 0.9:
                parts.append(extra[int(rng.integers(len(extra)))].encode("utf-8"))
            else:
                parts.append(bytes([int(rng.integers(128, 256))]))
            parts.append(b" " * int(rng.integers(0, 3)))
        out.append(b"".join(parts))
    return out


def tokenizer_fixture() -> None:
    """ref_tokenizer.json: tokenizer.cpp through the reference build (oracle/_ref)."""
    oracle.build(reference=True, tree=REF_TREE)
    tok = S.make_bpe_tokenizer()
    rt = oracle.RefTokenizer(tok)
    cases = []
    for t in tokenizer_texts():
        ids = rt.encode(t)
        cases.append({"text": t.hex(), "ids": ids, "decoded": rt.decode_bytes(ids).hex()})
    rt.close()
    with open(os.path.join(HERE, "ref_tokenizer.json"), "w") as f:
        json.dump({"tokenizer": tok, "cases": cases}, f)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TORCHLESS_REFERENCE"),
                    help="the reference source tree (default: $TORCHLESS_REFERENCE)")
    ap.add_argument("--only-sample", action="store_true", help="regenerate ref_sample.npz only")
    ap.add_argument("--only-tokenizer", action="store_true", help="regenerate ref_tokenizer.json only")
    args = ap.parse_args()
    global REF_TREE
    if not args.reference:
        ap.error("the reference tree is needed: --reference <tree> or TORCHLESS_REFERENCE")
    ref = REF_TREE = args.reference
    if args.only_sample:
        sample_fixture()
        return
    if args.only_tokenizer:
        tokenizer_fixture()
        return

    exp = read_expected(os.path.join(ref, "test/mistral/expected.txt"))
    with open(os.path.join(HERE, "reference_expected.json"), "w") as f:
        json.dump({"source": "test/mistral/expected.txt",
                   "vectors": {k: exp[k] for k in WEIGHT_INDEPENDENT},
                   "kats": kats()}, f)

    oracle.build(reference=True, tree=REF_TREE)
    hashes = {}
    for name, (cfg, seed) in MODELS.items():
        tmp = tempfile.mkdtemp()
        tensors = dict(S.numpy_tensors(cfg, seed=seed, norm="random"))
        S.write_hf_dir(os.path.join(tmp, "hf"), cfg, tensors)
        out = os.path.join(tmp, "ref.bin")
        subprocess.run([sys.executable, os.path.join(ref, "export_mistral.py"), "--model_dir",
                        os.path.join(tmp, "hf"), "--out", out, "--quant", "int8"], check=True,
                       capture_output=True)
        ref_bytes = np.fromfile(out, dtype=np.uint8)
        mine = S.make_numpy_model(cfg, seed=seed, norm="random").buf
        assert np.array_equal(ref_bytes, mine), f"numpy exporter differs from export_mistral.py ({name})"
        hashes[name] = {"seed": seed, "norm": "random", "sha256": sha256(ref_bytes), "size": int(ref_bytes.size)}

        rng = np.random.default_rng(1000 + seed)
        prompt = rng.integers(0, cfg["vocab_size"], PROMPT_LEN).astype(np.int64)
        rm = oracle.RefModel(ref_bytes, max_seq=PROMPT_LEN + N_NEW + 8)
        ids, logits = oracle.greedy(rm, prompt.tolist(), N_NEW)
        rm.close()
        np.savez_compressed(os.path.join(HERE, f"ref_greedy_{name}.npz"), prompt=prompt,
                            ids=np.array(ids, dtype=np.int64), logits=np.stack(logits))

    with open(os.path.join(HERE, "export_hashes.json"), "w") as f:
        json.dump(hashes, f, indent=1)

    # Op-level outputs of the reference kernels on seeded inputs.
    L = oracle.ref_lib()
    rng = np.random.default_rng(42)
    ops = {}
    n, d = 48, 320
    q = rng.integers(-127, 128, (n, d), dtype=np.int8)
    for tag, ns in (("g64", n * d // 64), ("g80", n * d // 80), ("g7", 7)):
        s = np.abs(rng.standard_normal(ns).astype(np.float32)) * 0.01 + 0.001
        x = rng.standard_normal(d).astype(np.float32)
        y = np.zeros(n, np.float32)
        L.ref_matmul_i8(y.ctypes.data, q.ctypes.data, s.ctypes.data, ns, x.ctypes.data, n, d)
        ops[f"i8_{tag}_s"], ops[f"i8_{tag}_x"], ops[f"i8_{tag}_y"] = s, x, y
    ops["i8_q"] = q
    w = rng.standard_normal((7, 33)).astype(np.float32)
    x = rng.standard_normal(33).astype(np.float32)
    y = np.zeros(7, np.float32)
    L.ref_matmul_f32(y.ctypes.data, w.ctypes.data, x.ctypes.data, 7, 33)
    ops.update(f32_w=w, f32_x=x, f32_y=y)
    w = rng.standard_normal((9, 17)).astype(np.float32)
    x = rng.standard_normal(9).astype(np.float32)
    y = np.zeros(17, np.float32)
    L.ref_row_matmul(y.ctypes.data, x.ctypes.data, w.ctypes.data, 9, 17)
    ops.update(row_w=w, row_x=x, row_y=y)
    x = (rng.standard_normal(13) * 3).astype(np.float32)
    y = np.zeros(13, np.float32)
    L.ref_softmax(y.ctypes.data, x.ctypes.data, 13)
    ops.update(softmax_x=x, softmax_y=y)
    x = rng.standard_normal((3, 16)).astype(np.float32)
    c = rng.standard_normal(16).astype(np.float32)
    sn = rng.standard_normal(16).astype(np.float32)
    y = np.zeros((3, 16), np.float32)
    L.ref_rope(y.ctypes.data, x.ctypes.data, c.ctypes.data, sn.ctypes.data, 3, 16)
    ops.update(rope_x=x, rope_c=c, rope_s=sn, rope_y=y)
    x = (rng.standard_normal(11) * 4).astype(np.float32)
    y = np.zeros(11, np.float32)
    L.ref_silu(y.ctypes.data, x.ctypes.data, 11)
    ops.update(silu_x=x, silu_y=y)
    np.savez_compressed(os.path.join(HERE, "ref_ops.npz"), **ops)
    sample_fixture()
    tokenizer_fixture()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
