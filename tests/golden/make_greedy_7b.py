"""Full-depth Mistral-7B greedy fixture: the CPU oracle's decode of the
benchmark workload, pinned to the reference itself on its first steps.

    python tests/golden/make_greedy_7b.py [--steps 144] [--ref-steps 3]

Workload (the bs1 decode benchmark's): the Mistral-7B architecture with
seeded N(0, 0.02) weights quantised to int8 per 64-group
(torchless_b200.synthetic.make_seeded_model, seed 0, norms 1.0), a prompt of
16 uniform ids in [0, 32000) from numpy's default_rng(0), driven like
main.cpp:69-77: 15 prompt forwards, then `steps` x (forward + sample_max).

The oracle (oracle/tl_oracle.c, the bit-faithful restatement of
Model<int8_t>::forward, modules.cpp:154-171) produces every step.  The
reference's own Model<int8_t> (oracle/_ref, built from its sources) then
re-runs the first `ref_steps` steps on the same binary and its logits must
equal the oracle's bit for bit; the script fails otherwise.

Writes tests/golden/greedy_7b.npz:
  prompt [16], ids [steps]      greedy ids (the token each step produced)
  margin, maxabs [steps]        top-2 logit margin and max |logit| per step
                                (near-tie rule: margin < 1e-3 * maxabs)
  stride, slices [steps, V/stride]  logits[::stride] of every step
  logits_first, logits_last     all logits of the first and last step
  digest                        synthetic.model_digest of the binary
  ref_steps, ref_bitexact       how many steps the reference re-ran, and the outcome

The oracle needs about 3.5 s per token on 8 cores, the reference about 25 s
(its int8 matmul is single-threaded), so a default run takes ~25 minutes.
"""
from __future__ import annotations

import argparse
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402
from torchless_b200 import synthetic as S  # noqa: E402
from torchless_b200.binfmt import ModelFile  # noqa: E402

SEED, PROMPT_LEN, STRIDE = 0, 16, 125
OUT = os.path.join(HERE, "greedy_7b.npz")


def prompt_ids():
    """The bs1 benchmark's prompt: 16 uniform ids from default_rng(0)."""
    return np.random.default_rng(SEED).integers(0, 32000, PROMPT_LEN).tolist()


def top2(lg: np.ndarray):
    i = int(oracle.oracle_lib().tlo_argmax(lg.ctypes.data, lg.size))
    rest = np.delete(lg, i)
    return i, float(lg[i] - rest.max()), float(np.abs(lg).max())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--steps", type=int, default=144)
    ap.add_argument("--ref-steps", type=int, default=3)
    args = ap.parse_args()

    t0 = time.time()
    w = S.make_seeded_model(S.MISTRAL_7B, seed=SEED)
    buf = w.buf
    digest = S.model_digest(buf)
    print(f"model {w.size / 1e9:.2f} GB in {time.time() - t0:.0f} s, digest {digest[:16]}", flush=True)

    prompt = prompt_ids()
    max_seq = PROMPT_LEN + args.steps + 1
    om = oracle.OracleModel(ModelFile(buf), max_seq=max_seq)
    t0 = time.time()
    for t in prompt[:-1]:
        om.forward(int(t))
    tok = int(prompt[-1])
    ids, margin, maxabs, slices, first, last, ref_logits = [], [], [], [], None, None, []
    for step in range(args.steps):
        lg = om.forward(tok)
        i, m, a = top2(lg)
        ids.append(i)
        margin.append(m)
        maxabs.append(a)
        slices.append(lg[::STRIDE].copy())
        if step < args.ref_steps:
            ref_logits.append(lg.copy())
        if step == 0:
            first = lg.copy()
        last = lg.copy()
        tok = i
        if step % 16 == 0:
            print(f"oracle step {step}: id {i} margin {m:.4g} max|logit| {a:.4g} "
                  f"({(time.time() - t0) / (PROMPT_LEN + step):.2f} s/forward)", flush=True)
    om.close()
    near = int(np.sum(np.array(margin) < 1e-3 * np.array(maxabs)))
    print(f"oracle done: {args.steps} steps, {near} near-ties, {time.time() - t0:.0f} s", flush=True)

    bitexact = True
    if args.ref_steps:
        oracle.build(reference=True)
        rm = oracle.RefModel(buf, max_seq=max_seq)
        t0 = time.time()
        for t in prompt[:-1]:
            rm.forward(int(t))
        tok = int(prompt[-1])
        for step in range(args.ref_steps):
            lg = rm.forward(tok)
            same = bool(np.array_equal(lg.view(np.uint32), ref_logits[step].view(np.uint32)))
            sm = rm.sample_max()
            print(f"reference step {step}: bit-exact {same}, sample_max {sm} (oracle {ids[step]})", flush=True)
            bitexact &= same and sm == ids[step]
            tok = ids[step]
        rm.close()
        print(f"reference: {PROMPT_LEN - 1 + args.ref_steps} forwards in {time.time() - t0:.0f} s", flush=True)
        if not bitexact:
            raise SystemExit("the oracle and the reference disagree at full depth")

    np.savez_compressed(
        OUT, prompt=np.array(prompt, np.int64), ids=np.array(ids, np.int64),
        margin=np.array(margin, np.float32), maxabs=np.array(maxabs, np.float32),
        stride=np.int64(STRIDE), slices=np.stack(slices).astype(np.float32),
        logits_first=first, logits_last=last, digest=np.array(digest), seed=np.int64(SEED),
        ref_steps=np.int64(args.ref_steps), ref_bitexact=np.bool_(bitexact))
    print(f"wrote {OUT}")


if __name__ == "__main__":
    main()
