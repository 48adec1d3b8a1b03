"""Benchmark: int8 Mistral-7B batch-1 greedy decode tok/s on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one "step" = one decode token, forward + argmax): the Mistral-7B
architecture with seeded random-init weights N(0, 0.02), quantised to int8
per 64-group in the export_mistral.py layout (synthetic.make_seeded_model:
the same bytes on every host, so both arms and the full-depth parity fixture
decode the identical binary); a 16-token uniform-random prompt is forwarded
first (15 forwards, untimed, as main.cpp:69-71), then W warm-up and K timed
greedy steps, each feeding its argmax to the next.  The 7.9 GB of weights
read per step are far larger than the 126 MB L2, so no L2 flush is needed
between steps.  The W + K greedy ids are checked against the oracle's ids in
tests/golden/greedy_7b.npz (the "parity" key).

Prints one JSON line (rank 0).  `value` is device time (CUDA events around
K back-to-back CUDA-graph replays); `e2e` is the same K steps through the
public C ABI call tl_model_forward with the token copied in from and the
argmax copied back to host memory each step.  For N > 1 the one sequence is
tensor-parallel over the N GPUs (each rank holds 1/N of every projection and
of the lm_head; o_proj and down_proj partials are summed inside the decode
kernel over NVLink): strong scaling, the timed region is bracketed by
barriers and the slowest rank's time counts.

--impl reference times the reference's own CPU code (oracle/_ref, built from
the reference sources) on this host, on the same binary: W untimed and K
timed whole decode tokens (Model<int8_t>::forward over all 32 layers +
sample_max, main.cpp:69-77), starting from position 0.  Its int8 matmul is
single-threaded, so a token takes ~20 s; the run takes (W + K) x that.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "int8 Mistral-7B decode tok/s @bs1 (1/2/4/8 GPU); GEMV HBM GB/s vs peak"
PROMPT_LEN, SEED = 16, 0
FALLBACK_HBM_GBS = 6650.0


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def dist_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(
        os.environ.get("LOCAL_RANK", "0"))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


LM_HEAD_INT8 = False  # --lm-head-int8: the int8 lm_head format extension
WEIGHTS = "int8"      # --fp8: projection weights as the fp8 (e5m2) cast, a format extension


def weight_bytes_per_token(lm_8bit: bool) -> float:
    """Weight bytes one Mistral-7B decode token reads: the projections (int8 +
    fp32 scale per 64, or fp8 bytes), the lm_head (fp32, or the projections'
    format), the final and per-layer norms, one embedding row."""
    proj, lm = 6979321856, 32000 * 4096
    qb = 1.0 if WEIGHTS == "fp8" else 1 + 4 / 64
    return proj * qb + lm * (qb if lm_8bit else 4.0) + 1064960 + 16384


def make_model_bytes(layers: int = 32):
    """The seeded Mistral-7B binary (int8, or with --fp8 the e5m2 cast), built
    on the host CPU by synthetic.make_seeded_model: identical bytes on every
    host and for both arms."""
    from torchless_b200 import synthetic as S
    t0 = time.time()
    cfg = dict(S.MISTRAL_7B, num_hidden_layers=layers)
    w = S.make_seeded_model(cfg, seed=SEED, quant=WEIGHTS, quant_lm_head=LM_HEAD_INT8)
    log(f"generated {w.size / 1e9:.2f} GB model on {os.cpu_count()} host threads in {time.time() - t0:.1f}s")
    return w.buf


def decode_config(args, max_seq: int) -> dict:
    """The bs1 decode workload, as both arms name it."""
    return {"workload": f"Mistral-7B int8 bs1 greedy decode (seeded N(0,0.02) weights, 16-token random prompt, "
                        f"{args.warmup} warm-up + {args.steps} timed tokens)",
            "global_batch": 1, "seq_len": max_seq,
            "l2": "inputs larger than L2 (7.94 GB of weights per step)",
            "weights_bytes_per_token": int(weight_bytes_per_token(LM_HEAD_INT8))}


def fixture_ids():
    """The oracle's greedy ids of the bs1 workload (tests/golden/greedy_7b.npz), or None."""
    p = os.path.join(ROOT, "tests", "golden", "greedy_7b.npz")
    if not os.path.exists(p):
        return None
    d = np.load(p)
    return d["ids"].tolist(), d["margin"], d["maxabs"]


def ids_parity(ids) -> dict:
    """Greedy ids produced after the prompt against the oracle fixture's."""
    fx = fixture_ids()
    if fx is None:
        return {"checked": 0, "note": "fixture missing"}
    want, margin, maxabs = fx
    n = min(len(ids), len(want))
    bad = next((i for i in range(n) if ids[i] != want[i]), None)
    out = {"checked": n, "identical": bad is None, "against": "oracle greedy ids (tests/golden/greedy_7b.npz)"}
    if bad is not None:
        out["first_mismatch"] = bad
        out["near_tie_there"] = bool(margin[bad] < 1e-3 * maxabs[bad])
    return out


def prompt_ids():
    return np.random.default_rng(SEED).integers(0, 32000, PROMPT_LEN).tolist()


class ClockSampler:
    """SM clock and throttle reasons via NVML, sampled every 10 ms while running."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, cuda_index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nv = pynvml
            p = torch.cuda.get_device_properties(cuda_index)
            try:  # NVML numbers GPUs differently from a masked CUDA view: match the PCI bus id
                bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
                self.h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # NVML missing: report no clocks rather than guess
            log(f"NVML unavailable: {e}")
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for k, bit in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(k)
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self.nv:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self.nv:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


def cpu_reference_sample(buf, n_layers: int):
    """The reference's own modules (oracle/_ref) for one Mistral-7B decode token:
    embedding + n_layers layers + norm + lm_head; returns (tok/s, seconds, cores)."""
    import oracle
    rm = oracle.RefModel(buf, max_seq=64)
    t_emb, t_layers, t_head = rm.time_token(prompt_ids()[0], 0, n_layers)
    rm.close()
    per_token = t_emb + t_layers * (32.0 / n_layers) + t_head
    return 1.0 / per_token, t_emb + t_layers + t_head, os.cpu_count()


def run_reference(args, rank, world):
    """The reference's own CPU decode (oracle/_ref) on the same binary, whole tokens."""
    if rank != 0:
        return
    import oracle
    if not oracle.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref was not built (needs the reference tree at build time)"}))
        return
    buf = make_model_bytes(args.layers)
    n = args.warmup + args.steps
    max_seq = max(PROMPT_LEN, n) + 8
    rm = oracle.RefModel(buf, max_seq=max_seq)
    toks = prompt_ids()
    tok, ids, times = toks[0], [], []
    # A whole token takes ~20 s on the CPU: time at most as many of the
    # requested K as fit in ~150 s (at least 3), so the run ends in minutes.
    timed = args.steps
    for i in range(n):  # main.cpp:69-77 from position 0: prompt tokens, then greedy
        t0 = time.perf_counter()
        rm.forward(tok)
        nxt = rm.sample_max()
        t1 = time.perf_counter()
        if i == 0:
            timed = max(3, min(args.steps, int(150.0 / max(t1 - t0, 1e-3))))
        if i >= args.warmup:
            times.append(t1 - t0)
        if i + 1 < len(toks):
            tok = toks[i + 1]
        else:
            ids.append(nxt)
            tok = nxt
        log(f"reference token {i}: {t1 - t0:.2f} s")
        if len(times) >= timed:
            break
    rm.close()
    total = sum(times)
    timed = len(times)
    value = timed / total
    cores = os.cpu_count()
    sample = (f"the reference's own Model<int8_t>::forward (all 32 layers) + sample_max on the same binary, "
              f"{args.warmup} untimed + {timed} timed whole tokens (of the {args.steps} requested: those that "
              f"fit in ~150 s) at positions 0..{args.warmup + timed - 1} "
              f"(prompt forwards, then greedy); int8 matmul single-threaded, fp32 lm_head on OpenMP")
    out = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": timed, "warmup": args.warmup, "ms_per_step": 1000.0 * total / timed,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "parallelism": "cpu", "config": decode_config(args, PROMPT_LEN + n + 8),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "ids_head": ids[:8],
    }
    if args.layers == 32 and WEIGHTS == "int8" and not LM_HEAD_INT8:
        out["parity"] = ids_parity(ids)
    print(json.dumps(out))


def load_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


def run_ours(args, rank, world, local):
    import torch
    import torch.distributed as dist
    from torchless_b200 import Model, tp

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600),
                                device_id=torch.device(f"cuda:{local}"))
    ctx = args.context
    max_seq = (ctx if ctx > 0 else PROMPT_LEN) + args.warmup + args.steps + 8
    if world == 1:
        buf = make_model_bytes(args.layers)
        m = Model.from_buffer(buf, device=local, max_seq=max_seq)
    else:
        # N > 1: one sequence, tensor-parallel over the N GPUs.  Rank 0 writes
        # the model file once; every rank maps it and loads its slice.
        import tempfile
        path = os.path.join(tempfile.gettempdir(), f"tl_bench_model_{os.environ.get('MASTER_PORT', '0')}.bin")
        if rank == 0:
            make_model_bytes(args.layers).tofile(path)
        dist.barrier()
        m = Model.load(path, device=local, max_seq=max_seq, tp_size=world, tp_rank=rank)
        dist.barrier()
        if rank == 0:
            os.remove(path)
        tp.connect(m)
        buf = None
    if ctx > 0:
        # long context: a random prompt of ctx ids, ingested untimed (the batched
        # prompt pass on one GPU; token by token under tensor parallelism)
        prompt = np.random.default_rng(SEED + 1).integers(0, 32000, ctx).tolist()
        if world == 1:
            m.prefill(prompt[:-1], logits=False)
        else:
            for t in prompt[:-1]:
                m.forward(t, logits=False)
    else:
        prompt = prompt_ids()
        for t in prompt[:-1]:
            m.forward(t, logits=False)
    start_pos = m.pos
    # warm-up greedy steps, then the timed ones continue from the last argmax
    _, warm_ids = m.time_decode(prompt[-1], args.warmup)
    first = warm_ids[-1]

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    with ClockSampler(local) as clocks:
        barrier()
        ms, ids = m.time_decode(first, args.steps)
        barrier()
        # e2e: the same positions again through the public per-token call
        m.pos = start_pos + args.warmup
        tok = first
        barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            _, tok = m.forward(tok, logits=False)
        t1 = time.perf_counter()
        barrier()
    e2e_s = t1 - t0
    if world > 1:
        t = torch.tensor([ms, e2e_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_s = float(t[0]), float(t[1])
    # one sequence on all N GPUs: tokens of that sequence per second
    value = args.steps / (ms / 1000.0)
    e2e = args.steps / e2e_s

    # Per-kernel device times (eager launches with an event pair around each)
    m.pos = start_pos
    prof = m.profile(prompt[-1], 4)
    launches = m.launches_per_step()
    if world > 1:
        dist.barrier()  # no rank unmaps its exchange buffer while a peer kernel runs
    m.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    top = max(prof, key=lambda k: k["total_ms"])  # the dominant kernel
    # one launch per step (the persistent kernel): its average duration is the
    # timed region's; otherwise the per-launch event pairs of the profile pass
    avg_ms = ms / args.steps if launches == 1 else top["total_ms"] / top["launches"]
    achieved = top["bytes_per_launch"] / (avg_ms / 1000.0) / 1e9
    peak, peak_kind = peaks()
    # ncu traffic of the 1-GPU launch; a rank's launch under tensor parallelism is not captured
    ext = LM_HEAD_INT8 or WEIGHTS != "int8"  # a format-extension run
    traffic = load_traffic().get(top["name"]) if world == 1 and ctx == 0 and not ext else None
    total_prof = sum(k["total_ms"] for k in prof)

    # bytes of one token at the mean timed position: weights + the K/V rows read
    w_bytes = weight_bytes_per_token(LM_HEAD_INT8)
    kv_per_pos = 2 * args.layers * 8 * 128 * 4
    tok_bytes = w_bytes + kv_per_pos * (start_pos + args.warmup + (args.steps + 1) / 2.0) if ctx > 0 \
        else w_bytes
    cfg = decode_config(args, max_seq)
    if ctx > 0:
        cfg["workload"] = (f"Mistral-7B int8 bs1 greedy decode ({ctx}-token random prompt, "
                           f"{args.warmup} warm-up + {args.steps} timed tokens)")
    if LM_HEAD_INT8:
        cfg["workload"] += f" [format extension: {WEIGHTS} lm_head]"
    if WEIGHTS == "fp8":
        cfg["workload"] = cfg["workload"].replace("int8 bs1", "fp8 (e5m2) bs1") + " [format extension: fp8 weights, no scales]"
    if args.layers != 32:
        cfg["workload"] += f" [profiling case: {args.layers} of 32 layers]"
    dtype = ("f16 x f16 -> f32 (e5m2 weights widened exactly, x as two fp16 planes)" if WEIGHTS == "fp8" else
             "s8 x s8 -> s32 (int8 weights x 22-bit fixed-point activation digits), f32 group combine")
    out = {
        "metric": (METRIC if ctx == 0 else f"int8 Mistral-7B decode tok/s @bs1, {ctx}-token context")
        if WEIGHTS == "int8" else f"fp8 Mistral-7B decode tok/s @bs1{f', {ctx}-token context' if ctx else ''}",
        "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        # one sequence: the total work is fixed however many GPUs share it
        "scaling": "strong", "vs_baseline": None, "dtype": dtype,
        "data": "synthetic", "parallelism": f"tp{world}" if world > 1 else "single",
        "config": cfg,
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 4},
        "gpu_launches": launches * args.steps,
        "roofline": {"bound": "hbm", "kernel": top["name"], "achieved": achieved, "peak": peak,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "algorithmic_bytes": top["bytes_per_launch"]},
        # N GPUs share the bytes of a token: the roofline is N x peak / bytes
        "model_roofline": {"bytes_per_token": tok_bytes, "tok_s_at_peak": world * peak * 1e9 / tok_bytes,
                           "frac": value / (world * peak * 1e9 / tok_bytes)},
        "kernel_shares": {k["name"]: round(k["total_ms"] / total_prof, 4) for k in prof},
        "clocks": clocks.summary(),
        "ids_head": ids[:8],
    }
    if ctx == 0 and args.layers == 32 and not ext:
        out["parity"] = ids_parity(warm_ids + ids)
    if not args.no_cpu_baseline and world == 1 and ctx == 0 and not ext:
        try:
            v, secs, cores = cpu_reference_sample(buf, args.cpu_layers)
            out["cpu_baseline"] = {
                "value": v, "unit": "tok/s", "cores": cores, "kind": "reference",
                "sample": (f"one decode token of the same model through the reference's own modules "
                           f"(oracle/_ref): embedding + {args.cpu_layers} of 32 layers (x{32 // args.cpu_layers}) "
                           f"+ norm + lm_head; {secs:.1f} s of CPU; int8 matmul is single-threaded, "
                           f"OpenMP fp32 lm_head uses all cores")}
        except Exception as e:
            out["cpu_baseline"] = {"value": None, "unit": "tok/s", "cores": os.cpu_count(), "kind": "reference",
                                   "sample": f"not run: {e}"}
    print(json.dumps(out))


# ---------------------------------------------------------------------------
# Isolated int8 GEMV sweep at Mistral-7B shapes (batch 1), through the op-level
# C ABI (tl_matmul_i8 = kernels.h matmul(int8); tl_mlp_gate_up = w1|w3 fused
# with SiLU * up).  Weights int8 uniform in [-127, 127], stored scales
# |N(0, 0.01)| (divisors, tensor.cpp:101-104), x ~ N(0, 1).  Enough weight
# copies rotate that every launch streams its weights from HBM (> L2).
# ---------------------------------------------------------------------------
SWEEP = [("wq/wo 4096->4096", 4096, 4096, "matmul"), ("wk/wv 4096->1024", 1024, 4096, "matmul"),
         ("w1|w3 4096->14336 fused SiLU*up", 14336, 4096, "gate_up"), ("w2 14336->4096", 4096, 14336, "matmul"),
         ("lm_head int8 4096->32000", 32000, 4096, "matmul")]


def run_gemv_sweep(args):
    import torch
    from torchless_b200 import ops
    torch.cuda.set_device(0)
    peak, peak_kind = peaks()
    g = torch.Generator(device="cuda")
    g.manual_seed(SEED)
    for name, n, d, kind in SWEEP:
        if args.gemv_shape and not name.startswith(args.gemv_shape):
            continue
        mats = 2 if kind == "gate_up" else 1
        wbytes = mats * (n * d + 4 * n * d // 64)
        copies = max(2, -(-(256 << 20) // wbytes))  # > 256 MB in rotation: no L2 reuse
        ws = []
        for _ in range(copies):
            one = []
            for _ in range(mats):
                w = torch.randint(-127, 128, (n, d), dtype=torch.int8, device="cuda", generator=g)
                sc = torch.randn(n * d // 64, device="cuda", generator=g).abs_() * 0.01 + 1e-6
                one.append((w, sc))
            ws.append(one)
        x = torch.randn(d, device="cuda", generator=g)
        y = torch.empty(n, device="cuda")

        def launch(i):
            one = ws[i % copies]
            if kind == "gate_up":
                ops.mlp_gate_up(y, one[0][0], one[0][1], one[1][0], one[1][1], x)
            else:
                ops.matmul(y, one[0][0], x, scales=one[0][1])

        # parity against a torch fp32 restatement (w / scale per 64-group)
        launch(0)
        torch.cuda.synchronize()

        def deq(w, sc):
            return (w.float().view(n, d // 64, 64) / sc.view(n, d // 64, 1)).view(n, d)
        if kind == "gate_up":
            gate = deq(*ws[0][0]) @ x
            ref = gate / (1.0 + torch.exp(-gate)) * (deq(*ws[0][1]) @ x)
        else:
            ref = deq(*ws[0][0]) @ x
        err = float((y - ref).abs().max() / ref.abs().max())
        for i in range(args.warmup):
            launch(i)
        # the K timed launches as one CUDA graph: device time of the kernels
        # back to back, without a Python / ctypes call between them
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(args.steps):
                launch(args.warmup + i)
        graph.replay()  # warm the graph itself
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1000.0 / args.steps
        del graph
        algo = wbytes + 4 * d + 4 * n
        gbs = algo / (us * 1e-6) / 1e9
        line = {"metric": "int8 GEMV HBM GB/s (bs1)", "shape": name, "n": n, "d": d,
                "value": gbs, "unit": "GB/s", "us_per_launch": us, "algorithmic_bytes": algo,
                "peak": peak, "peak_kind": peak_kind, "frac": gbs / peak, "rel_err_vs_fp32": err,
                "launches": args.steps, "copies_rotated": copies, "timing": "CUDA graph of the timed launches"}
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_gemv_sample(ws[0][0][0], ws[0][0][1], x, mats)
        print(json.dumps(line), flush=True)
        del ws


def cpu_gemv_sample(w, sc, x, mats, rows=256):
    """The reference's matmul(int8) (kernels.cpp:21-33, oracle/_ref) on the first
    `rows` rows of the same weights; GB/s of weight + scale bytes (single thread,
    as the reference's int8 matmul is)."""
    import ctypes
    import oracle
    if not oracle.ref_available():
        return {"value": None, "unit": "GB/s", "cores": 1, "kind": "reference", "sample": "oracle/_ref not built"}
    n, d = w.shape
    r = min(rows, n)
    wh = np.ascontiguousarray(w[:r].cpu().numpy())
    sh = np.ascontiguousarray(sc[: r * d // 64].cpu().numpy())
    xh = np.ascontiguousarray(x.cpu().numpy())
    yh = np.empty(r, dtype=np.float32)
    L = oracle.ref_lib()
    P = ctypes.c_void_p
    t0 = time.perf_counter()
    reps = 0
    while reps < 3 or time.perf_counter() - t0 < 1.0:
        L.ref_matmul_i8(P(yh.ctypes.data), P(wh.ctypes.data), P(sh.ctypes.data), sh.size, P(xh.ctypes.data), r, d)
        reps += 1
    secs = (time.perf_counter() - t0) / reps
    return {"value": (r * d + 4 * r * d // 64) / secs / 1e9, "unit": "GB/s", "cores": 1, "kind": "reference",
            "sample": f"first {r} rows of the same weights, x{mats} matrices for the fused shape not included, "
                      f"{reps} repetitions"}


# ---------------------------------------------------------------------------
# Prefill: Mistral-7B, 2048-token random prompt in one batched pass (tensor
# cores), then 32 greedy decode steps from the filled KV cache.
# ---------------------------------------------------------------------------
def run_prefill(args):
    import torch
    from torchless_b200 import Model
    torch.cuda.set_device(0)
    T, N_DEC = args.prefill_tokens, 32
    buf = make_model_bytes(args.layers)
    m = Model.from_buffer(buf, max_seq=T + N_DEC + 8, weights_f16=args.weights_f16)
    rng = np.random.default_rng(SEED)
    prompt = rng.integers(0, 32000, T).tolist()
    times = []
    for i in range(args.warmup + args.steps):  # each step: the whole prompt from position 0
        m.pos = 0
        ms, first = m.time_prefill(prompt)
        if i >= args.warmup:
            times.append(ms)
    ms_prefill = float(np.mean(times))
    # decode continues from the cache
    m.pos = 0
    _, first = m.prefill(prompt, logits=False)
    ms_dec, ids = m.time_decode(first, N_DEC)
    m.close()
    L, D, F, H, KV, HD = args.layers, 4096, 14336, 32, 8, 128
    lin = 2.0 * T * L * ((H + 2 * KV) * HD * D + D * H * HD + 3 * F * D)
    attn = 4.0 * HD * H * L * T * (T + 1) / 2
    flops = lin + attn + 2.0 * 32000 * D
    tflops = flops / (ms_prefill * 1e-3) / 1e12
    pk = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak = json.load(open(pk))["bf16_tflops"] if os.path.exists(pk) else 1590.0
    out = {"metric": f"{WEIGHTS} Mistral-7B prefill tok/s (2048-token prompt)", "value": T / (ms_prefill * 1e-3),
           "unit": "tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_prefill,
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": ("resident f16 weight copies" if args.weights_f16 else
                     "int8 weights dequantised to f16 in shared memory") + ", f16 x f16 -> f32 tcgen05 MMA",
           "data": "synthetic",
           "config": {"workload": f"Mistral-7B int8 ({L} layers), prefill of {T} random token ids, "
                                  f"then {N_DEC} greedy decode steps", "prompt": T, "decode": N_DEC},
           "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s",
                        "frac": tflops / peak, "flops_per_step": flops,
                        "note": "whole prefill (GEMMs + attention + row kernels) against the dense fp16 peak"},
           "decode_after_prefill": {"tok_s": N_DEC / (ms_dec * 1e-3), "ms_per_token": ms_dec / N_DEC,
                                    "ids_head": ids[:8]},
           "first_token": first}
    print(json.dumps(out))


# ---------------------------------------------------------------------------
# Batched decode: 64 sequences, each with a 4096-position KV cache of N(0, 1)
# values (counter-based generator), 64 greedy steps per sequence.
# ---------------------------------------------------------------------------
def run_batch(args, rank=0, world=1, local=0):
    import torch
    import torch.distributed as dist
    from torchless_b200 import Batch, Model, tp
    torch.cuda.set_device(local)
    B, P, K = args.batch_seqs, args.batch_context, args.steps
    max_seq = P + args.warmup + K + 8
    if world == 1:
        buf = make_model_bytes(args.layers)
        m = Model.from_buffer(buf, max_seq=max_seq, weights_f16=args.weights_f16)
        del buf
    else:
        # N > 1: the same B sequences on every rank, each rank holding its
        # tensor-parallel slice of the weights and of every sequence's KV heads
        import tempfile
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=600),
                                device_id=torch.device(f"cuda:{local}"))
        path = os.path.join(tempfile.gettempdir(), f"tl_bench_model_{os.environ.get('MASTER_PORT', '0')}.bin")
        if rank == 0:
            make_model_bytes(args.layers).tofile(path)
        dist.barrier()
        m = Model.load(path, device=local, max_seq=max_seq, tp_size=world, tp_rank=rank,
                       weights_f16=args.weights_f16)
        dist.barrier()
        if rank == 0:
            os.remove(path)
        tp.connect(m)
    b = Batch(m, B)
    if world > 1:
        tp.connect_batch(b)
    b.fill_kv_random(SEED, P)
    toks = np.random.default_rng(SEED).integers(0, 32000, B).tolist()
    _, ids = b.time_decode(toks, args.warmup)
    first = ids[-1].tolist()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    with ClockSampler(local) as clocks:
        barrier()
        ms, ids = b.time_decode(first, K)
        barrier()
    if world > 1:
        t = torch.tensor([ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
        dist.barrier()  # no rank unmaps an exchange buffer while a peer kernel runs
    b.close()
    m.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    L, D, F, H, KV, HD, V = args.layers, 4096, 14336, 32, 8, 128, 32000
    pos_mean = P + args.warmup + (K - 1) / 2.0
    kv_bytes = B * L * 2 * KV * HD * 4 * (pos_mean + 1)  # cache rows read per step (all sequences)
    w_int8 = L * ((H + 2 * KV) * HD * D + D * H * HD + 3 * F * D) * (1 + 4.0 / 64) + V * D * 4
    # the int8 weights and their scales in place (or, with --weights-f16, fp16 copies), and a
    # resident fp16 copy of the fp32 lm_head
    params = L * ((H + 2 * KV) * HD * D + D * H * HD + 3 * F * D)
    w_here = params * (2.0 if args.weights_f16 else 1 + 4.0 / 64) + V * D * 2
    step_s = ms * 1e-3 / K
    peak, peak_kind = peaks()
    algo = kv_bytes + w_int8
    out = {"metric": f"{WEIGHTS} Mistral-7B batched decode tok/s (64 seqs x 4096-token KV)", "value": B * K / (ms * 1e-3),
           "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": ms / K,
           "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
           "dtype": ("resident f16 weight copies" if args.weights_f16 else
                     "int8 weights dequantised to f16 in shared memory") + ", f16 x f16 -> f32 tcgen05 MMA, f32 KV",
           "data": "synthetic",
           "config": {"workload": f"Mistral-7B int8 ({L} layers), {B} sequences, KV pre-filled with {P} positions "
                                  f"of N(0,1) (counter-based generator), {K} greedy steps", "global_batch": B,
                      "seq_len": P + args.warmup + K,
                      "parallelism": f"tp{world}" if world > 1 else "single"},
           # N GPUs share the step's bytes: whole-job bandwidth against N x the per-GPU peak
           "roofline": {"bound": "hbm", "achieved": algo / step_s / 1e9, "peak": world * peak,
                        "peak_kind": peak_kind + (f" x {world} GPUs" if world > 1 else ""),
                        "unit": "GB/s", "frac": algo / step_s / 1e9 / (world * peak), "algorithmic_bytes": algo,
                        "bytes_read_by_this_path": kv_bytes + w_here,
                        "note": "algorithmic = int8 weights + scales + fp32 lm_head + fp32 KV; this path reads "
                                + ("fp16 copies of the weights" if args.weights_f16 else
                                   "the int8 weights + scales (dequantised to fp16 in shared memory inside the "
                                   "tensor-core GEMM)") + " and an fp16 copy of the lm_head"},
           "clocks": clocks.summary(), "ids_head": ids[0][:8].tolist()}
    print(json.dumps(out))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-layers", type=int, default=8)
    ap.add_argument("--batch", action="store_true",
                    help="batched decode: --batch-seqs sequences with --batch-context pre-filled KV positions")
    ap.add_argument("--batch-seqs", type=int, default=64)
    ap.add_argument("--batch-context", type=int, default=4096)
    ap.add_argument("--prefill", action="store_true",
                    help="batched prefill of a --prefill-tokens prompt, then 32 decode steps")
    ap.add_argument("--prefill-tokens", type=int, default=2048)
    ap.add_argument("--gemv-sweep", action="store_true",
                    help="isolated int8 GEMV sweep at Mistral-7B shapes (one JSON line per shape)")
    ap.add_argument("--gemv-shape", default="",
                    help="--gemv-sweep: only the shape whose name starts with this (e.g. lm_head)")
    ap.add_argument("--lm-head-int8", action="store_true",
                    help="bs1 decode of the same model with its lm_head stored int8 (format extension)")
    ap.add_argument("--fp8", action="store_true",
                    help="the same workloads on the fp8 (e5m2) export of the model (format extension)")
    ap.add_argument("--context", type=int, default=0,
                    help="bs1 decode after a random prompt of this many tokens (0: the 16-token prompt)")
    ap.add_argument("--weights-f16", action="store_true",
                    help="--prefill / --batch with resident fp16 weight copies instead of int8 in place")
    ap.add_argument("--layers", type=int, default=32,
                    help="transformer layers (32 = Mistral-7B; fewer only for small profiling captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    global LM_HEAD_INT8, WEIGHTS
    LM_HEAD_INT8 = args.lm_head_int8
    WEIGHTS = "fp8" if args.fp8 else "int8"
    rank, world, local = dist_env()
    if args.gemv_sweep:
        run_gemv_sweep(args)
        return
    if args.prefill:
        run_prefill(args)
        return
    if args.batch:
        run_batch(args, rank, world, local)
        return
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local)


if __name__ == "__main__":
    main()
