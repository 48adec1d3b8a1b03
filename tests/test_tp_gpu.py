"""Tensor-parallel decode: 2 ranks, one process per GPU, through the C ABI.

Each rank loads its slice of the model (q/k/v heads, gate/up rows, o/down
columns, lm_head rows), maps the other rank's exchange buffer, and runs the
persistent decode kernel; o_proj and down_proj partials are summed inside the
kernel over NVLink.  Checks, per step:
  * both ranks return the same token;
  * the gathered logits (rank slices in vocabulary order) match the
    reference's (golden model) within the parity rule, and match the 1-GPU
    run of the same weights (7B-shaped model) to within fp32 reordering.
Skipped with fewer than 2 GPUs.
"""
import os
import sys
import tempfile

import numpy as np
import pytest

from conftest import golden_greedy, model_bytes, rel_err

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
LOGIT_TOL = 1e-2
TIE = 1e-3
WORLD = 2


def _need(n):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def _rank_main(rank, world, init_file, model_path, feed, max_seq, out_dir):
    """Child process: load this rank's slice, connect, feed tokens, save results."""
    import datetime

    import torch
    import torch.distributed as dist

    from torchless_b200 import Model, tp

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    m = Model.load(model_path, device=rank, max_seq=max_seq, tp_size=world, tp_rank=rank)
    tp.connect(m)
    logits, toks = [], []
    for t in feed:
        lg, nxt = m.forward(int(t))
        logits.append(lg)
        toks.append(nxt)
    dist.barrier()  # no rank unmaps a buffer a peer kernel may still use
    m.close()
    dist.barrier()
    dist.destroy_process_group()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), logits=np.stack(logits), toks=np.array(toks))


def run_tp(model_path, feed, max_seq=64, world=WORLD):
    """Runs `feed` through a `world`-rank model; returns (full logits per step, tokens per rank)."""
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as d:
        init_file = os.path.join(d, "init")
        mp.start_processes(_rank_main, args=(world, init_file, model_path, list(feed), max_seq, d), nprocs=world,
                           join=True, start_method="spawn")
        res = [np.load(os.path.join(d, f"rank{r}.npz")) for r in range(world)]
        logits = np.concatenate([r["logits"] for r in res], axis=1)
        return logits, [r["toks"].tolist() for r in res]


def margin(logits):
    top = np.sort(logits)[-2:]
    return float(top[1] - top[0]) / max(float(np.max(np.abs(logits))), 1e-30)


def test_tp2_greedy_matches_reference():
    """SMALL golden model (8 q heads / 2 kv heads): 2 ranks vs the reference's own logits."""
    _need(WORLD)
    prompt, ids, ref_logits = golden_greedy("small")
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "small.bin")
        model_bytes("small").tofile(path)
        feed = list(prompt) + list(ids[:-1])
        logits, toks = run_tp(path, feed)
    assert toks[0] == toks[1], "ranks disagree on the token"
    n0 = len(prompt) - 1  # logits of the last prompt token and after are the reference's steps
    worst = 0.0
    for step in range(len(ids)):
        e = rel_err(logits[n0 + step], ref_logits[step])
        worst = max(worst, e)
        assert e <= LOGIT_TOL, (step, e)
        if toks[0][n0 + step] != ids[step]:
            assert margin(ref_logits[step]) < TIE, step
    print(f"tp{WORLD} small: worst logits rel err {worst:.2e}")
    assert worst < 1e-4


# Attention of the persistent step: per-head CTAs (the default at short
# context), or GQA CTAs from the first position with 8 positions per split
# (the long-context path, here with up to 3 splits per kv group).
ATTN_ENV = {"per_head": {}, "gqa": {"TL_DECODE_GQA_FROM": "0", "TL_DECODE_GQA_ROWS": "8"}}


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("attn", list(ATTN_ENV))
def test_tp_matches_one_gpu_7b_shapes(attn, world, monkeypatch):
    """Mistral-7B layer shapes (2 layers, N = 2, 4, 8 splits of every
    projection; at N = 8 one kv head per rank) vs 1 GPU."""
    _need(world)
    for k, v in ATTN_ENV[attn].items():
        monkeypatch.setenv(k, v)  # read at load, here and in the spawned ranks
    from torchless_b200 import Model, ops, synthetic as S
    cfg = dict(S.MISTRAL_7B, num_hidden_layers=2)
    buf = S.make_torch_model(cfg, seed=5, norm="random", device="cuda",
                             quantizer=lambda x: ops.quantize_i8(x)).buf
    rng = np.random.default_rng(2)
    feed = rng.integers(0, 32000, 10 if attn == "per_head" else 24).tolist()
    one = Model.from_buffer(buf, max_seq=32)
    ref, ref_toks = [], []
    for t in feed:
        lg, nxt = one.forward(t)
        ref.append(lg)
        ref_toks.append(nxt)
    one.close()
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m7b2.bin")
        buf.tofile(path)
        del buf
        logits, toks = run_tp(path, feed, max_seq=32, world=world)
    assert all(t == toks[0] for t in toks), "ranks disagree on the token"
    for step in range(len(feed)):
        e = rel_err(logits[step], ref[step])
        assert e < 1e-4, (step, e)
        if toks[0][step] != ref_toks[step]:
            assert margin(ref[step]) < TIE, step


BATCH_SEED = 99


def _rank_batch_main(rank, world, init_file, model_path, n_seq, n_pos, steps, out_dir):
    """Child process: a tensor-parallel Batch of n_seq sequences, KV filled with
    the counter-based generator (keyed by global kv head), `steps` greedy steps."""
    import datetime

    import torch
    import torch.distributed as dist

    from torchless_b200 import Batch, Model, tp

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    m = Model.load(model_path, device=rank, max_seq=n_pos + steps + 8, tp_size=world, tp_rank=rank)
    tp.connect(m)
    b = Batch(m, n_seq)
    tp.connect_batch(b)
    b.fill_kv_random(BATCH_SEED, n_pos)
    toks = [(7 * i + 3) % m.config["vocab_size"] for i in range(n_seq)]
    logits, ids = [], []
    for _ in range(steps):
        lg, nxt = b.step(toks)
        logits.append(lg)
        ids.append(nxt.copy())
        toks = nxt.tolist()
    dist.barrier()  # no rank unmaps a buffer a peer kernel may still use
    b.close()
    m.close()
    dist.barrier()
    dist.destroy_process_group()
    np.savez(os.path.join(out_dir, f"batch{rank}.npz"), logits=np.stack(logits), ids=np.stack(ids))


def _one_gpu_batch(buf, n_seq, n_pos, steps):
    from torchless_b200 import Batch, Model
    m = Model.from_buffer(buf, max_seq=n_pos + steps + 8)
    b = Batch(m, n_seq)
    b.fill_kv_random(BATCH_SEED, n_pos)
    toks = [(7 * i + 3) % m.config["vocab_size"] for i in range(n_seq)]
    logits, ids = [], []
    for _ in range(steps):
        lg, nxt = b.step(toks)
        logits.append(lg)
        ids.append(nxt.copy())
        toks = nxt.tolist()
    b.close()
    m.close()
    return np.stack(logits), np.stack(ids)


@pytest.mark.parametrize("which,world", [("small", 2), ("7b_shapes", 2), ("7b_shapes", 4), ("7b_shapes", 8)])
def test_tp_batch_matches_one_gpu(which, world):
    """Batched decode on `world` ranks (o / down rows summed across ranks inside
    the residual + RMSNorm kernel, argmax merged over the vocabulary slices) vs
    the same batch on 1 GPU: every step's logits of every sequence and the
    tokens."""
    _need(world)
    import torch.multiprocessing as mp
    if which == "small":
        buf, n_seq, n_pos, steps = model_bytes("small"), 3, 40, 5
    else:
        from torchless_b200 import ops, synthetic as S
        cfg = dict(S.MISTRAL_7B, num_hidden_layers=2)
        buf = S.make_torch_model(cfg, seed=5, norm="random", device="cuda",
                                 quantizer=lambda x: ops.quantize_i8(x)).buf
        n_seq, n_pos, steps = 4, 100, 4
    ref, ref_ids = _one_gpu_batch(buf, n_seq, n_pos, steps)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.bin")
        buf.tofile(path)
        init_file = os.path.join(d, "init")
        mp.start_processes(_rank_batch_main, args=(world, init_file, path, n_seq, n_pos, steps, d), nprocs=world,
                           join=True, start_method="spawn")
        res = [np.load(os.path.join(d, f"batch{r}.npz")) for r in range(world)]
    logits = np.concatenate([r["logits"] for r in res], axis=2)  # vocabulary slices in rank order
    assert all(np.array_equal(res[0]["ids"], r["ids"]) for r in res), "ranks disagree on the tokens"
    # The batched path feeds its GEMMs fp16 activations: a last-bit change of the
    # fp32 residual (another summation order: split-K ranges and ranks) can flip
    # an fp16 rounding, so the two runs agree to the batched path's own
    # tolerance against the reference (~1.5e-3 at these shapes), not to fp32 noise.
    worst = 0.0
    for s in range(steps):
        for q in range(n_seq):
            e = rel_err(logits[s, q], ref[s, q])
            worst = max(worst, e)
            assert e < 3e-3, (s, q, e)
            if res[0]["ids"][s, q] != ref_ids[s, q]:
                assert margin(ref[s, q]) < TIE, (s, q)
    print(f"tp{world} batch {which}: worst logits rel err {worst:.2e}")


def _rank_depth_main(rank, world, init_file, model_path, prompt, n_new, out_dir):
    """Child process: prompt token by token, then n_new greedy steps through the
    timed loop (tl_model_time_decode) and again through forward() with logits."""
    import datetime

    import torch
    import torch.distributed as dist

    from torchless_b200 import Model, tp

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=300))
    m = Model.load(model_path, device=rank, max_seq=64, tp_size=world, tp_rank=rank)
    tp.connect(m)
    for t in prompt[:-1]:
        m.forward(int(t), logits=False)
    p0 = m.pos
    _, ids = m.time_decode(int(prompt[-1]), n_new)
    m.pos = p0
    logits, t = [], int(prompt[-1])
    for _ in range(n_new):
        lg, t = m.forward(t)
        logits.append(lg)
    dist.barrier()
    m.close()
    dist.barrier()
    dist.destroy_process_group()
    np.savez(os.path.join(out_dir, f"depth{rank}.npz"), ids=np.array(ids), logits=np.stack(logits))


def test_tp2_full_depth_7b():
    """All 32 Mistral-7B layers at N = 2 vs 1 GPU: tokens of the timed loop and
    of forward(), and logits.  Loading a full-size slice exercises the upload
    ordering (pageable copies against kernels on the model's stream)."""
    _need(2)
    import torch.multiprocessing as mp
    from torchless_b200 import Model, ops, synthetic as S
    buf = S.make_torch_model(dict(S.MISTRAL_7B), seed=21, device="cuda", quantizer=lambda x: ops.quantize_i8(x)).buf
    prompt = np.random.default_rng(21).integers(0, 32000, 8).tolist()
    n_new = 6
    one = Model.from_buffer(buf, max_seq=64)
    for t in prompt[:-1]:
        one.forward(t, logits=False)
    p0 = one.pos
    _, ref_ids = one.time_decode(prompt[-1], n_new)
    one.pos = p0
    ref, t = [], prompt[-1]
    for _ in range(n_new):
        lg, t = one.forward(t)
        ref.append(lg)
    one.close()
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m7b.bin")
        buf.tofile(path)
        del buf
        mp.start_processes(_rank_depth_main, args=(2, os.path.join(d, "init"), path, prompt, n_new, d), nprocs=2,
                           join=True, start_method="spawn")
        res = [np.load(os.path.join(d, f"depth{r}.npz")) for r in range(2)]
    logits = np.concatenate([r["logits"] for r in res], axis=1)
    assert np.all(np.isfinite(logits))
    assert res[0]["ids"].tolist() == res[1]["ids"].tolist()
    for step in range(n_new):
        e = rel_err(logits[step], ref[step])
        assert e < 1e-4, (step, e)
        if res[0]["ids"][step] != ref_ids[step]:
            assert margin(ref[step]) < TIE, step


def _rank_timeout_main(rank, world, init_file, model_path, feed, out_dir):
    """Child: step 0 on both ranks; at step 1 rank 1 stays away (no kernel of its
    own in flight), so rank 0's exchange wait runs out; then both reload."""
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["TL_WAIT_TIMEOUT_MS"] = "200"  # read at load: a short bound for the test
    from torchless_b200 import Model, TLError, tp

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    m = Model.load(model_path, device=rank, max_seq=32, tp_size=world, tp_rank=rank)
    tp.connect(m)
    _, first = m.forward(int(feed[0]))
    statuses = []
    if rank == 0:
        for _ in range(2):  # the run-out wait, then the model refuses further steps
            try:
                m.forward(int(feed[1]))
                statuses.append(0)
            except TLError as e:
                statuses.append(e.status)
    dist.barrier()  # rank 0's failed step has ended before anyone unmaps its buffers
    m.close()
    dist.barrier()
    # recovery: reload on every rank and run the steps again
    m = Model.load(model_path, device=rank, max_seq=32, tp_size=world, tp_rank=rank)
    tp.connect(m)
    toks = [m.forward(int(t))[1] for t in feed]
    dist.barrier()
    m.close()
    dist.barrier()
    dist.destroy_process_group()
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), first=first, statuses=np.array(statuses, np.int64),
             toks=np.array(toks))


def test_tp2_peer_absent_times_out_and_reload_recovers(small_bin):
    """A rank that does not join a step: the other rank's bounded exchange wait
    ends the step with TL_ERR_TIMEOUT (no GPU fault, no hang), the model then
    refuses further steps, and a reload on both ranks decodes as before."""
    _need(2)
    import torch.multiprocessing as mp
    from torchless_b200 import STATUS
    prompt, ids, _ = golden_greedy("small")
    feed = [prompt[0], prompt[1], prompt[2]]
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "m.bin")
        np.asarray(small_bin).tofile(path)
        init_file = os.path.join(d, "init")
        mp.start_processes(_rank_timeout_main, args=(2, init_file, path, feed, d), nprocs=2, join=True,
                           start_method="spawn")
        r0, r1 = (np.load(os.path.join(d, f"rank{r}.npz")) for r in range(2))
    timeout = [k for k, v in STATUS.items() if v == "TL_ERR_TIMEOUT"][0]
    assert r0["statuses"].tolist() == [timeout, timeout]
    assert int(r0["first"]) == int(r1["first"])
    assert r0["toks"].tolist() == r1["toks"].tolist()
    assert int(r0["toks"][0]) == int(r0["first"])  # the reloaded model repeats the clean step 0
