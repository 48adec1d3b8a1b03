"""Text generation from the command line, the loop of main.cpp:51-82 on the GPU:

    python -m torchless_b200.generate MODEL.bin "prompt" [--tokens 50] [--temperature T --seed S]

Encodes the prompt with the binary's tokenizer (BOS first), runs all prompt
tokens but the last through the batched prompt pass, then generates: each
step forwards the previous token and picks the next with sample_max
(main.cpp:10-21) or, at --temperature > 0, sample_multinomial (main.cpp:23-43)
on the device; every token is decoded and printed as it arrives.
"""
from __future__ import annotations

import argparse
import sys
import time


def generate(model_path: str, prompt: str, n_tokens: int = 50, temperature: float = 0.0, seed: int = 0,
             max_seq: int = 1024, device: int = 0, sliding_window: int = 0, out=sys.stdout) -> list:
    from . import Model, Tokenizer
    tok = Tokenizer.load(model_path)
    ids = tok.encode(prompt)
    m = Model.load(model_path, device=device, max_seq=max(max_seq, len(ids) + n_tokens + 1),
                   sliding_window=sliding_window)
    if temperature > 0:
        m.set_sampling(temperature, seed)
    if len(ids) > 1:
        m.prefill(ids[:-1], logits=False)
    t = ids[-1]
    got = []
    for _ in range(n_tokens):
        _, t = m.forward(t, logits=False)
        got.append(t)
        out.write(tok.decode_bytes([t]).decode("utf-8", errors="replace"))
        out.flush()
    out.write("\n")
    m.close()
    tok.close()
    return got


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("model", help="model binary (export_mistral.py format)")
    ap.add_argument("prompt")
    ap.add_argument("--tokens", type=int, default=50, help="tokens to generate (main.cpp: 50)")
    ap.add_argument("--temperature", type=float, default=0.0, help="0: greedy (sample_max)")
    ap.add_argument("--seed", type=int, default=0, help="seed of the device-side uniform draws")
    ap.add_argument("--max-seq", type=int, default=1024)
    ap.add_argument("--device", type=int, default=0)
    ap.add_argument("--sliding-window", type=int, default=0, help="0: attend to all positions (reference)")
    a = ap.parse_args(argv)
    t0 = time.time()
    got = generate(a.model, a.prompt, a.tokens, a.temperature, a.seed, a.max_seq, a.device, a.sliding_window)
    print(f"[{len(got)} tokens in {time.time() - t0:.2f} s]", file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
