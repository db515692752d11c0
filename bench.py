#!/usr/bin/env python
"""Needle 3 batched agent decode on B200 (the headline throughput workload).

1024 concurrent sequences in all, partitioned across
the N GPUs (1024 / N each, one process per GPU, no collective on the data
path; strong scaling). Every sequence gets a 118-token random prompt
(prefilled outside the timed region) and then the config's 45 greedy
decode steps, each under its own seeded random vocabulary mask that allows
5-50% of the ids. A bench "step" is one decode step of all sequences:
masked argmax of the last logits, then the forward of the chosen ids
through all 20 layers and the lm_head. Of the 45 steps, W are warm-up, K
are timed and the rest run untimed afterwards, so the KV lengths are the
config's whatever K is.

`value` times K steps with masks and ids resident in HBM (CUDA events on the
engine's stream, max over ranks); `e2e` times K steps through the C ABI with
host buffers: each step copies the masks in from pinned host memory and the
chosen ids back. `--impl reference` times the CPU restatement of the
reference engine on the host's cores (the reference itself is Rust and cannot
be built in this image).
"""

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "needle-rs_b200"))

import numpy as np  # noqa: E402

PROMPT, STEPS_CFG = 118, 45
METRIC = "batched agent decode tok/s (1024 seqs over all GPUs, 118-token prompt, 45 masked greedy steps)"
CACHE = os.environ.get("NEEDLE_BENCH_CACHE", "/tmp/needle_b200_bench_cache")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--seqs", type=int, default=1024, help="sequences in all, partitioned across the GPUs")
    ap.add_argument("--roofline-site", default="attention",
                    help="the kernel site the roofline object reports (auto: the slowest in the sweep)")
    ap.add_argument("--cpu-baseline", type=int, default=1, help="time the oracle on rank 0 (N=1 only)")
    ap.add_argument("--secondary", type=int, default=1, help="also time batch-1 decode and 256x700 prefill (N=1)")
    ap.add_argument("--sweep", action="store_true",
                    help="instead of the decode bench: the CQ-W4/A8 matmul sweep (M in 1, 16, 128, 2048 over the "
                         "model's four matrix shapes), one JSON line")
    ap.add_argument("--ops", action="store_true",
                    help="instead of the decode bench: the fused-ops sweep (RMSNorm, RoPE, SiLU, embedding gather at "
                         "T in 1, 64, 1024, 8192), L2 flushed before every timed launch, one JSON line")
    ap.add_argument("--profile", action="store_true",
                    help="untimed case for ncu: one batch of --seqs sequences, the 118-token prefill, then --warmup "
                         "decode steps (--profile-case decode); or three call-sampler launches over 1024 rows of "
                         "logits (candidates); or one 256 x 64 embedding (embed)")
    ap.add_argument("--profile-case", default="decode", choices=["decode", "candidates", "embed", "ops", "prefill_matmul"],
                    help="decode uses --seqs sequences (1 for the batch-1 step)")
    return ap.parse_args()


def archive_bytes(writer="engine"):
    """The random-init Needle 3 archive (seed 0). The GPU arm writes it with
    the engine's writer; the reference arm with the oracle's, which is
    byte-identical (tests/test_archive_writer.py), so that arm never loads
    the product library."""
    if writer == "engine":
        import needle_b200 as nb

        write = nb.synth_cact
    else:
        from oracle import oracle as orc

        write = orc.synth_cact
    path = os.path.join(CACHE, f"needle3-seed0-{writer}.cact")
    if not os.path.exists(path):
        os.makedirs(CACHE, exist_ok=True)
        data = write(seed=0)
        tmp = f"{path}.{os.getpid()}.tmp"
        with open(tmp, "wb") as f:
            f.write(data)
        os.replace(tmp, path)
    with open(path, "rb") as f:
        return f.read()


# A low-width plan for the batch-1 decode leg (record bits per CQ role, 5 =
# ternary): the attention projections ternary, the out and engram
# projections 2-bit, the engram tables 3-bit, embedding and mHC rows 4-bit.
LOW_WIDTH = dict(q=5, k=5, v=5, gate=5, out=2, key=2, value=2, table=3)


def low_width_archive():
    import needle_b200 as nb

    path = os.path.join(CACHE, "needle3-seed0-low-width.cact")
    if not os.path.exists(path):
        os.makedirs(CACHE, exist_ok=True)
        data = nb.synth_cact(seed=0, bits=LOW_WIDTH)
        tmp = f"{path}.{os.getpid()}.tmp"
        with open(tmp, "wb") as f:
            f.write(data)
        os.replace(tmp, path)
    with open(path, "rb") as f:
        return f.read()


def decode_weight_bytes(bits=None, L=20, sites=5, vocab=16384):
    """Codes and f16 norms one decode token streams through the matmuls
    (q|k|v|gate, out, lm_head, engram key|value; 6 groups a row) plus the
    int8 mHC rows (24 x 3072 a layer)."""
    import needle_b200 as nb

    bits = bits or {}
    w = lambda role: nb.code_width(bits.get(role, 4))
    row = lambda role: 6 * (16 * w(role) + 2)
    per_layer = 576 * row("q") + 96 * row("k") + 128 * row("v") + 768 * row("gate") + 768 * row("out") + 24 * 3072
    return L * per_layer + vocab * row("embedding") + sites * 768 * (row("key") + row("value"))


def make_inputs(first, S, steps, vocab):
    """Prompts [S, 118] and masks [steps, S, vocab/8] (bit set = allowed) of
    sequences first .. first + S - 1 of the workload: each sequence draws
    from its own seeded stream, so a sequence's inputs do not depend on how
    the sequences are partitioned across GPUs."""
    prompts = np.empty((S, PROMPT), np.int32)
    masks = np.empty((steps, S, (vocab + 7) // 8), np.uint8)
    for i in range(S):
        rng = np.random.default_rng([1000, first + i])
        prompts[i] = rng.integers(0, vocab, PROMPT)
        frac = rng.uniform(0.05, 0.5, (steps, 1))
        allow = rng.random((steps, vocab), np.float32) < frac
        allow[np.arange(steps), rng.integers(0, vocab, steps)] = True
        masks[:, i] = np.packbits(allow, axis=1, bitorder="little")
    return prompts, masks


def shard(total, world, rank):
    """This rank's contiguous share of `total` sequences: (first, count)."""
    base, extra = divmod(total, world)
    return rank * base + min(rank, extra), base + (1 if rank < extra else 0)


class Clocks:
    """nvidia-smi samples of the SM clock and throttle reasons while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


# DRAM traffic of one decode launch from one ncu capture of
# `bench.py --profile --seqs 1024 --warmup 2` (dram__bytes_read.sum +
# dram__bytes_write.sum; profiles/<kernel>_decode_1024.md), with the
# algorithmic bytes of that launch: the roofline scales the traffic to this
# run's launch by the ratio of algorithmic bytes (sequences and keys).
PROFILED_TRAFFIC = {
    "attention": (35_249_152, 37_896_192),
    "post": (22_288_896, 40_992_768),
    "qkvg": (2_047_744, 7_854_464),
    "mhc": (12_709_120, 19_857_408),
}


def site_algorithmic(site, S, n_keys):
    """Algorithmic work of one launch of a site at a decode step (T = 1, S
    rows): (amount, unit, bound). Bytes count every input once and every
    output once; int8 ops count a multiply-add as two."""
    act = S * (768 + 6 * 4)
    gemm = {"qkvg": 1568, "out": 768, "lm_head": 16384, "engram_kv": 1536}
    if site in gemm:
        n = gemm[site]
        return n * 396 + act + S * n * 4, "bytes", "hbm"
    if site == "attention":
        # per row: 12 q heads read the 2 kv heads' keys/values of n positions
        kv = S * 2 * n_keys * (48 + 4 + 64 + 4)
        return kv + S * (576 + 768 + 768) * 4, "bytes", "hbm"
    if site == "post":
        return S * (768 * 5 + 3072 * 2 + 24) * 4, "bytes", "hbm"
    if site == "mhc":
        # read xs; write u, gates, x1 and the A8 row (engram-site reads aside)
        return S * (3072 + 768 + 24 + 768 + 6) * 4 + S * 768 + 24 * 3072, "bytes", "hbm"
    if site == "conv":
        return S * (1568 + 576) * 4 + S * 2 * (48 + 64 + 8), "bytes", "hbm"
    raise KeyError(site)


def run_reference(args, rank, world):
    """The reference arm: the CPU restatement of needle-rs's engine on every
    host thread, the same metric on a bounded sample of sequences."""
    if rank != 0:
        return
    from oracle import oracle as orc

    threads = os.cpu_count() or 1
    data = archive_bytes("oracle")
    model = orc.Model(data)
    S = threads
    prompts, masks = make_inputs(0, S, args.warmup + args.steps, model.out_rows)
    b = orc.Batch(model, S, threads)
    b.prefill(prompts)
    for k in range(args.warmup):
        b.step(masks[k])
    t0 = time.perf_counter()
    for k in range(args.steps):
        b.step(masks[args.warmup + k])
    dt = time.perf_counter() - t0
    value = S * args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "i8/f32", "data": "synthetic",
        "config": {"workload": "agent_decode", "seqs": S, "prompt": PROMPT, "decode_steps": args.warmup + args.steps,
                   "parallelism": "host threads (rank 0 only)", "model": "needle3-121M random-init CQ-W4 seed 0"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"{S} sequences (one per host thread), {args.steps} timed masked greedy steps after "
                                   f"a 118-token prefill and {args.warmup} warm-up steps"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_sample(data):
    from oracle import oracle as orc

    threads = os.cpu_count() or 1
    model = orc.Model(data)
    S, steps = threads, 20
    prompts, masks = make_inputs(0, S, steps, model.out_rows)
    b = orc.Batch(model, S, threads)
    b.prefill(prompts)
    t0 = time.perf_counter()
    for k in range(steps):
        b.step(masks[k])
    dt = time.perf_counter() - t0
    return {"value": S * steps / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{S} sequences (one per host thread), {steps} masked greedy decode steps after a 118-token "
                      f"prefill (decode timed only)"}


def matmul_sweep(local):
    """The CQ-W4/A8 matmul alone (A8 of the rows + the matmul, inputs resident
    on the GPU, nd_cqmat_apply's event timing): codes uniform over the 16
    values, f16 norms |N(0, 0.02)|, activations N(0, 1). Every M runs the
    decode combine (T = 1, one token a row); M >= 16 also runs the prefill
    combine as chunks of T = min(M, 32) tokens (the tensor-core kernel). One
    matrix (at most 6.5 MB) stays in L2 across the runs. Bytes: weight codes and norms +
    int8 activations and scales + f32 outputs; ops: 2 M N K. The oracle's
    single-thread time for a sample of the same rows is the CPU baseline."""
    import needle_b200 as nb
    from oracle import oracle as orc

    rng = np.random.default_rng(3)
    shapes = [("qkvg", 1568), ("out", 768), ("engram_kv", 1536), ("lm_head", 16384)]
    rows = []
    for name, n in shapes:
        codes = rng.integers(0, 256, (n, 6, 64), dtype=np.uint8)
        norms = np.abs(rng.standard_normal((n, 6)) * 0.02).astype(np.float16).view(np.uint16)
        mat = nb.CQMat(codes, norms, local)
        for M in (1, 16, 128, 2048):
            x = rng.standard_normal((M, 768)).astype(np.float32)
            for T in ([1] if M == 1 else [1, min(M, 32)]):
                reps = 200 if M * n <= 16 * 16384 else 50
                _, ms = mat(x, T=T, reps=reps)
                byt = n * 6 * (64 + 2) + M * 768 + M * 6 * 4 + M * n * 4
                sample = min(M, 32 if T > 1 else 4)
                t0 = time.perf_counter()
                orc.cq_matmul(codes.reshape(n, -1), norms, 768, x[:sample] if T > 1 else x[:1])
                cpu_s = (time.perf_counter() - t0) * (M / sample if T > 1 else M)
                rows.append({"matrix": name, "N": n, "K": 768, "M": M, "T": T,
                             "combine": "decode" if T == 1 else "prefill", "us": round(ms * 1e3, 2),
                             "GB_s": round(byt / (ms * 1e-3) / 1e9, 1),
                             "int8_TOPS": round(2 * M * n * 768 / (ms * 1e-3) / 1e12, 2),
                             "cpu_us": round(cpu_s * 1e6, 1)})
        del mat
    return rows


def prefill_matmul_case(local, reps=20):
    """The q|k|v|gate matmul of one 256-sequence prefill chunk (M = 8192 rows,
    T = 32, the prefill combine on the tensor cores) through nd_cqmat_apply,
    for a one-kernel profiler capture: one run, 3 warm-up runs, `reps` timed."""
    import needle_b200 as nb

    rng = np.random.default_rng(1)
    n, M, T = 1568, 8192, 32
    codes = rng.integers(0, 256, (n, 6, 64), dtype=np.uint8)
    norms = np.abs(rng.standard_normal((n, 6)) * 0.02).astype(np.float16).view(np.uint16)
    mat = nb.CQMat(codes, norms, local)
    x = rng.standard_normal((M, 768)).astype(np.float32)
    _, ms = mat(x, T=T, reps=reps)
    return {"matrix": "qkvg 1568 x 768", "M": M, "T": T, "us_a8_and_matmul": round(ms * 1e3, 2)}


OPS_T = (1, 64, 1024, 8192)


def ops_inputs(T, rng):
    """BASELINE configs[2]'s inputs at T tokens: rows N(0, 1) of the model
    width (RMSNorm), of the q|k heads (RoPE) and of the MLP's 1024 (SiLU);
    RMSNorm weights N(1, 0.1) rounded to f16; uniform-random token ids."""
    return {"zcn": rng.standard_normal((T, 768)).astype(np.float32),
            "s": (1.0 + 0.1 * rng.standard_normal(768)).astype(np.float16).astype(np.float32),
            "rope": rng.standard_normal((T, 672)).astype(np.float32),
            "silu": rng.standard_normal((T, 1024)).astype(np.float32),
            "ids": rng.integers(0, 16384, T).astype(np.int32)}


def ops_bytes(op, T):
    """Algorithmic bytes of one launch: every input and output once."""
    return {"zcn": 2 * T * 768 * 4 + 768 * 4, "rope": 2 * T * 672 * 4, "silu": 2 * T * 1024 * 4,
            "gather": T * (6 * 66 + 768 * 4 + 4)}[op]


def ops_sweep(local, model, reps=20, profile=False):
    """Each fused row op alone through its C entry (device buffers): `reps`
    launches, each after a 256 MB write that evicts L2 (126 MB) and a short
    device spin (so the launch is queued before its start event), timed by
    CUDA events around the launch alone (median); GB/s of the algorithmic bytes
    against the measured HBM copy bandwidth. The oracle's single-thread time
    for the same op and T is the CPU baseline."""
    import torch

    import needle_b200 as nb
    from oracle import oracle as orc

    dev = f"cuda:{local}"
    hbm, _, kind = peaks()
    rng = np.random.default_rng(2)
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    rows = []
    orc_model = None
    for T in OPS_T:
        inp = ops_inputs(T, rng)
        d = {k: torch.from_numpy(v).to(dev) for k, v in inp.items()}
        outs = {"zcn": torch.empty_like(d["zcn"]), "rope": torch.empty_like(d["rope"]),
                "silu": torch.empty_like(d["silu"]), "gather": torch.empty((T, 768), dtype=torch.float32, device=dev)}
        calls = {"zcn": lambda: nb.op_zcn(d["zcn"], d["s"], outs["zcn"]),
                 "rope": lambda: nb.op_rope(d["rope"], 100000.0, outs["rope"]),
                 "silu": lambda: nb.op_silu(d["silu"], outs["silu"]),
                 "gather": lambda: nb.op_gather(model, d["ids"], outs["gather"])}
        for op, call in calls.items():
            call()
            if profile:
                continue
            times = []
            for _ in range(reps):
                flush.fill_(float(len(times)))
                # a 100 us device spin first, so the launch is queued before
                # the start event fires and the events see the kernel alone
                torch.cuda._sleep(200000)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                call()
                e1.record()
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1))
            us = float(np.median(times)) * 1e3
            byt = ops_bytes(op, T)
            t0 = time.perf_counter()
            if op == "zcn":
                orc.op_zcn(inp["zcn"], inp["s"])
            elif op == "rope":
                orc.op_rope(inp["rope"])
            elif op == "silu":
                orc.op_silu(inp["silu"])
            else:
                if orc_model is None:
                    orc_model = orc.Model(archive_bytes("oracle"))
                orc_model.gather(inp["ids"].astype(np.uint32))
            cpu_s = time.perf_counter() - t0
            rows.append({"op": op, "T": T, "us": round(us, 2), "bytes": byt, "gb_s": round(byt / (us * 1e-6) / 1e9, 1),
                         "frac": round(byt / (us * 1e-6) / 1e9 / hbm, 4),
                         "cpu_gb_s": round(byt / cpu_s / 1e9, 2), "cpu_us": round(cpu_s * 1e6, 1)})
    torch.cuda.synchronize()
    return {"peak": hbm, "peak_kind": kind, "l2": "flushed before every timed launch (256 MB write)",
            "cpu_baseline": {"kind": "port", "cores": 1, "sample": "the same op and T, once, one host thread"},
            "rows": rows}


def decode_b1(model, rng, dev):
    """One sequence: the 118-token prompt, then 45 greedy steps with host
    buffers, one call per step like the reference's bench loop; a throwaway
    sequence first, so that no kernel runs cold in the timing."""
    import torch

    wb = model.batch(1, PROMPT + 8)
    wb.forward(rng.integers(0, model.vocab, (1, PROMPT)).astype(np.int32))
    for _ in range(4):
        wb.step(None)
    torch.cuda.synchronize()
    del wb
    b = model.batch(1, PROMPT + STEPS_CFG + 1)
    st = torch.cuda.ExternalStream(b.stream, device=dev)
    prompt = rng.integers(0, model.vocab, (1, PROMPT)).astype(np.int32)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    e[0].record(st)
    b.forward(prompt)
    e[1].record(st)
    nxt = np.zeros(1, np.int32)
    for _ in range(STEPS_CFG):
        b.step(None, nxt)
    e[2].record(st)
    torch.cuda.synchronize()
    res = {"prefill_tok_s": PROMPT / (e[0].elapsed_time(e[1]) / 1e3),
           "decode_tok_s": STEPS_CFG / (e[1].elapsed_time(e[2]) / 1e3),
           "decode_ms_per_token": e[1].elapsed_time(e[2]) / STEPS_CFG}
    del b
    return res


def call_candidates(model, dev, S=1024, k=128, reps=20):
    """nd_batch_candidates over 1024 rows of Needle 3 logits in HBM (the
    agent's call step start: softmax stats and the top 128 in the
    reference's order), device pointers, CUDA events on the batch's stream."""
    import ctypes

    import torch

    import needle_b200 as nb

    V = model.out_rows
    b = model.batch(S, 8)
    st = torch.cuda.ExternalStream(b.stream, device=dev)
    g = torch.Generator(device=dev).manual_seed(5)
    logits = torch.randn((S, V), generator=g, device=dev) * 3
    allow = torch.randint(0, 256, (S, (V + 7) // 8), generator=g, device=dev, dtype=torch.uint8)
    ids = torch.empty((S, k), dtype=torch.int32, device=dev)
    m = torch.empty(S, dtype=torch.float32, device=dev)
    z = torch.empty(S, dtype=torch.float64, device=dev)
    live = torch.empty(S, dtype=torch.int32, device=dev)
    P = lambda t: ctypes.c_void_p(t.data_ptr())
    call = lambda: nb.lib().nd_batch_candidates(b._h, P(logits), P(allow), None, k, P(ids), P(m), P(z), P(live),
                                                nb.ND_DEVICE)
    torch.cuda.synchronize()
    for _ in range(3):
        if call() != 0:
            raise nb._err()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for _ in range(reps):
        call()
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / max(reps, 1)
    del b
    return {"rows": S, "vocab": V, "k": k, "us_per_call": round(us, 2),
            "logit_gbs": round(S * V * 4 / (us * 1e-6) / 1e9, 1)}


def embed_texts(local, dev, S=256, T=64):
    """needle_embed's computation (heads.rs:63-90) for 256 texts of 64
    tokens at once on a Needle 3 archive with embedding and confidence
    heads: the forward with cells, the probe pool, the projection. Host ids
    in, unit vectors out, one nd_batch_embed call timed by CUDA events."""
    import torch

    import needle_b200 as nb

    path = os.path.join(CACHE, "needle3-seed0-heads.cact")
    if not os.path.exists(path):
        os.makedirs(CACHE, exist_ok=True)
        data = nb.synth_cact(seed=0, heads=(nb.HEAD_EMBEDDING, nb.HEAD_CONFIDENCE))
        tmp = f"{path}.{os.getpid()}.tmp"
        with open(tmp, "wb") as f:
            f.write(data)
        os.replace(tmp, path)
    with open(path, "rb") as f:
        model = nb.Model(f.read(), local)
    ids = np.random.default_rng(11).integers(0, model.vocab, (S, T)).astype(np.int32)
    model.batch(S, T).embed(ids)  # warm
    torch.cuda.synchronize()
    b = model.batch(S, T)
    st = torch.cuda.ExternalStream(b.stream, device=dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    v = b.embed(ids)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    del b, model
    return {"texts": S, "tokens_per_text": T, "dim": int(v.shape[1]), "ms": round(ms, 3),
            "texts_per_s": round(S / (ms * 1e-3), 1), "tok_s": round(S * T / (ms * 1e-3), 1)}


def cpu_decode_b1(data):
    """The oracle on one sequence: the 118-token prompt
    in chunks of 32, then 45 greedy decode steps, with each token's matmul
    rows, attention heads and post-block rows split over every host thread
    (the reference's worker team), and again on one thread."""
    from oracle import oracle as orc

    # the threads this process may run on (the team's workers spin between
    # a token's parallel regions, so never more than there are), at most 32
    threads = max(1, min(32, len(os.sched_getaffinity(0))))
    m = orc.Model(data)
    prompt = np.random.default_rng(78).integers(0, m.vocab, PROMPT).astype(np.uint32)

    def run(team):
        orc.set_team(team)
        try:
            s = m.session()
            t0 = time.perf_counter()
            logits = s.forward(prompt)[0]
            t1 = time.perf_counter()
            for _ in range(STEPS_CFG):
                logits = s.forward(np.array([int(np.argmax(logits))], np.uint32))[0]
            t2 = time.perf_counter()
        finally:
            orc.set_team(1)
        return STEPS_CFG / (t2 - t1), PROMPT / (t1 - t0)

    dec, pre = run(threads)
    dec1, pre1 = run(1)
    return {"value": dec, "unit": "decode tok/s", "prefill_tok_s": pre, "cores": threads, "kind": "port",
            "one_thread": {"value": dec1, "prefill_tok_s": pre1},
            "sample": f"one sequence: {PROMPT}-token prefill, {STEPS_CFG} greedy decode steps, each token's work "
                      f"split over {threads} host threads (one_thread: the same on one)"}


def cpu_prefill(data, n=700):
    """The oracle with one 700-token sequence per host thread (BASELINE
    configs[3]'s sequences, a bounded number of them), last-position logits."""
    from oracle import oracle as orc

    threads = os.cpu_count() or 1
    m = orc.Model(data)
    ids = np.random.default_rng(79).integers(0, m.vocab, (threads, n)).astype(np.uint32)
    t0 = time.perf_counter()
    m.prefill_batch(ids, threads=threads)
    dt = time.perf_counter() - t0
    return {"value": threads * n / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{threads} sequences of {n} tokens (one per host thread), logits of the last position"}


def gemv_l2_cold(local, copies=32, n=16384, reps=5):
    """The batch-1 decode matmul (M = 1: the GEMV on the 4-bit codes) at the
    lm_head's shape, L2-cold: `copies` distinct 16384 x 768 matrices (6.5 MB
    of codes and norms each, 208 MB in all, above the 126 MB L2) launched
    back to back in turn, so every launch streams its weights from HBM.
    Bytes: codes and norms + the int8 activation row and scales + the f32
    outputs."""
    import needle_b200 as nb

    rng = np.random.default_rng(5)
    mats = []
    for _ in range(copies):
        codes = rng.integers(0, 256, (n, 6, 64), dtype=np.uint8)
        norms = np.abs(rng.standard_normal((n, 6)) * 0.02).astype(np.float16).view(np.uint16)
        mats.append(nb.CQMat(codes, norms, local))
    mats[0](rng.standard_normal((1, 768)).astype(np.float32))
    ms = nb.CQMat.time_rotating(mats, 1, 1, reps)
    hot = nb.CQMat.time_rotating(mats[:1], 1, 1, 50)
    byt = n * 6 * (64 + 2) + 768 + 24 + n * 4
    hbm, _, kind = peaks()
    del mats
    return {"matrix": f"{n} x 768 CQ-W4 (lm_head shape), M = 1", "copies": copies,
            "bytes_per_launch": byt, "us_cold": round(ms * 1e3, 2), "gbs_cold": round(byt / (ms * 1e-3) / 1e9, 1),
            "frac_cold": round(byt / (ms * 1e-3) / 1e9 / hbm, 4), "peak": hbm, "peak_kind": kind,
            "us_l2_warm": round(hot * 1e3, 2), "gbs_l2_warm": round(byt / (hot * 1e-3) / 1e9, 1)}


def prefill_sites(model, local, ids, S, n):
    """Per-kernel breakdown of the 256 x 700 prefill: one more prefill per
    launch site with every launch of that site timed by CUDA events (ms in
    all and per launch), plus int8 tensor ops per ms for the matmul sites."""
    import needle_b200 as nb

    sites = {}
    macs = {"qkvg": 1568 * 768 * 20, "out": 768 * 768 * 20, "engram_kv": 1536 * 768 * 5}
    for site in ["qkvg", "out", "engram_kv", "attention", "post", "mhc", "conv", "lm_head"]:
        b = model.batch(S, n + 1)
        b.time_site(site)
        b.forward(ids, nb.OUT_LAST_LOGITS, out=np.zeros((S, 1, model.out_rows), np.float32))
        ms, launches = b.site_time()
        b.time_site("none")
        del b
        row = {"ms": round(ms, 3), "launches": launches, "us_per_launch": round(ms * 1e3 / max(launches, 1), 2)}
        if site in macs:
            row["int8_tops"] = round(2 * macs[site] * S * n / (ms * 1e-3) / 1e12, 1)
        sites[site] = row
    return sites


def secondary(model, local, data):
    """The other throughput workloads on this GPU, reported beside the
    headline: batch-1 decode (118-token prompt, 45 greedy
    steps, as `needle bench --decode 45` drives the engine; again on a
    low-width archive of the same geometry) and batched prefill (256
    sequences x 700 tokens, logits of the last position). CUDA events on
    the engine's stream. Each carries the oracle's time on the host's
    cores for the same workload (a bounded sample)."""
    import torch

    import needle_b200 as nb

    out = {}
    rng = np.random.default_rng(77)
    dev = f"cuda:{local}"
    out["decode_b1"] = decode_b1(model, rng, dev)
    out["decode_b1"]["weight_mb_per_token"] = round(decode_weight_bytes() / 1e6, 2)
    out["decode_b1"]["gemv_roofline"] = gemv_l2_cold(local)
    # the same on a low-width archive (mixed 2-bit, 3-bit, ternary records)
    low = nb.Model(low_width_archive(), local)
    out["decode_b1_low_width"] = decode_b1(low, rng, dev)
    out["decode_b1_low_width"]["weight_mb_per_token"] = round(decode_weight_bytes(LOW_WIDTH) / 1e6, 2)
    out["decode_b1_low_width"]["bits"] = LOW_WIDTH
    del low
    out["call_candidates_1024"] = call_candidates(model, dev)
    out["embed_256x64"] = embed_texts(local, dev)
    # 256 x 700 prefill, ids resident in HBM
    S, n = 256, 700
    b = model.batch(S, n + 1)
    st = torch.cuda.ExternalStream(b.stream, device=dev)
    ids_h = rng.integers(0, model.vocab, (S, n)).astype(np.int32)
    ids = torch.from_numpy(ids_h).to(dev)
    logits = torch.empty((S, 1, model.out_rows), dtype=torch.float32, device=dev)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st)
    b.forward(ids, nb.OUT_LAST_LOGITS, out=logits)
    e1.record(st)
    torch.cuda.synchronize()
    out["prefill_256x700"] = {"tok_s": S * n / (e0.elapsed_time(e1) / 1e3), "ms": e0.elapsed_time(e1)}
    del b
    out["prefill_256x700"]["sites"] = prefill_sites(model, local, ids_h, S, n)
    out["decode_b1"]["cpu_baseline"] = cpu_decode_b1(data)
    out["prefill_256x700"]["cpu_baseline"] = cpu_prefill(data, n)
    return out


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch

    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    torch.cuda.set_device(local)
    import needle_b200 as nb

    if args.profile and args.profile_case == "prefill_matmul":
        if rank == 0:
            print(json.dumps(prefill_matmul_case(local)), flush=True)
        return
    if args.sweep:
        if rank == 0:
            print(json.dumps({"sweep": "cq_w4a8_matmul", "cpu_baseline": {"kind": "port", "cores": 1,
                                                                           "sample": "the oracle on 1-32 rows of the same "
                                                                                     "matmul, scaled to M rows"},
                              "rows": matmul_sweep(local)}), flush=True)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    W, K = args.warmup, args.steps
    first, S = shard(args.seqs, world, rank)
    data = archive_bytes()
    model = nb.Model(data, device=local)
    V = model.out_rows
    if args.ops or (args.profile and args.profile_case == "ops"):
        res = ops_sweep(local, model, profile=args.profile)
        if rank == 0 and not args.profile:
            print(json.dumps({"sweep": "fused_row_ops", **res}), flush=True)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.profile and args.profile_case == "candidates":
        call_candidates(model, f"cuda:{local}", reps=0)
        torch.cuda.synchronize()
        return
    if args.profile and args.profile_case == "embed":
        embed_texts(local, f"cuda:{local}")
        torch.cuda.synchronize()
        return
    if args.profile:
        prompts, masks = make_inputs(first, S, W, V)
        b = model.batch(S, PROMPT + W + 1)
        b.forward(prompts, nb.OUT_LAST_LOGITS, out=np.zeros((S, 1, V), np.float32))
        for k in range(W):
            b.step(masks[k])
        torch.cuda.synchronize()
        return
    # Per-kernel sites. With at most one sequence an SM on a GPU (the
    # 8-GPU partition), each layer's post block launch also runs the next
    # layer's mHC read: "post" then includes it and "mhc" is layer 0's alone.
    sites = ["qkvg", "out", "lm_head", "engram_kv", "attention", "post", "mhc", "conv"]
    # The config's 45 steps: W warm-up, K timed, the rest untimed after them
    # (per-kernel site timing runs there); past 45 only when W + K leaves
    # too few steps for that.
    tail = max(STEPS_CFG - W - K, len(sites))
    n_steps = W + K + tail
    prompts, masks = make_inputs(first, S, n_steps, V)
    cap = PROMPT + n_steps + 1
    dev = f"cuda:{local}"

    # --- device-resident run (value)
    bA = model.batch(S, cap)
    bA.forward(prompts, nb.OUT_LAST_LOGITS, out=np.zeros((S, 1, V), np.float32))
    d_masks = torch.from_numpy(masks).to(dev)
    d_next = torch.zeros(S, dtype=torch.int32, device=dev)
    stream = torch.cuda.ExternalStream(bA.stream, device=dev)
    # --- host-buffer run (e2e)
    bB = model.batch(S, cap)
    bB.forward(prompts, nb.OUT_LAST_LOGITS, out=np.zeros((S, 1, V), np.float32))
    site = args.roofline_site if args.roofline_site != "auto" else "attention"

    def barrier():
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if not dist:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with Clocks(local) as clocks:
        for k in range(W):
            bA.step(d_masks[k], d_next)
        barrier()
        l0 = nb.launch_count()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for k in range(K):
            bA.step(d_masks[W + k], d_next)
        ev1.record(stream)
        launches = nb.launch_count() - l0
        barrier()
        t_value = ev0.elapsed_time(ev1) / 1e3
        # the rest of the config's steps, with the roofline site's kernels
        # timed by events around every launch (each step queued whole behind
        # a hold kernel, so the events see kernel time, not launch gaps)
        bA.time_site(site)
        for k in range(W + K, n_steps):
            bA.step(d_masks[k], d_next)
        site_ms, site_n = bA.site_time()
        bA.time_site("none")
        site_keys = np.mean([PROMPT + k + 1 for k in range(W + K, n_steps)])
        # e2e: host masks in pinned memory, ids back to the host, every step
        h_masks = torch.from_numpy(masks).pin_memory().numpy()
        h_next = torch.zeros(S, dtype=torch.int32).pin_memory().numpy()
        streamB = torch.cuda.ExternalStream(bB.stream, device=dev)
        for k in range(W):
            bB.step(h_masks[k], h_next)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(streamB)
        for k in range(K):
            bB.step(h_masks[W + k], h_next)
        e1.record(streamB)
        barrier()
        t_e2e = e0.elapsed_time(e1) / 1e3
    # the rest of the e2e batch's steps: one per site, every launch of that
    # site timed (untimed as far as value and e2e go)
    sweep = {}
    for j, k in enumerate(range(W + K, n_steps)):
        if j < len(sites):
            bB.time_site(sites[j])
        bB.step(h_masks[k], h_next)
        if j < len(sites):
            ms, n = bB.site_time()
            sweep[sites[j]] = {"ms_per_step": ms, "launches": n, "keys": PROMPT + k + 1}
    bB.time_site("none")
    t_value = max_over_ranks(t_value)
    t_e2e = max_over_ranks(t_e2e)
    clk = clocks.summary()
    del bA, bB
    extra = secondary(model, local, data) if (args.secondary and world == 1) else None

    if rank == 0:
        hbm, bf16, kind = peaks()
        amount, unit, bound = site_algorithmic(site, S, site_keys)
        avg_s = site_ms / 1e3 / max(site_n, 1)
        achieved = amount / avg_s / 1e9
        traffic = None
        if site in PROFILED_TRAFFIC:
            dram, alg = PROFILED_TRAFFIC[site]
            traffic = dram * amount / alg
        roofline = {"bound": bound, "kernel_site": site, "achieved": achieved, "peak": hbm,
                    "unit": "GB/s", "frac": achieved / hbm, "peak_kind": kind,
                    "algorithmic_bytes_per_launch": amount, "avg_launch_us": avg_s * 1e6, "launches": site_n,
                    "mean_keys": site_keys, "traffic": traffic}
        per_site = {}
        for nm, v in sweep.items():
            amt, _, _ = site_algorithmic(nm, S, v["keys"])
            us = v["ms_per_step"] * 1e3 / max(v["launches"], 1)
            per_site[nm] = {"ms_per_step": round(v["ms_per_step"], 4), "us_per_launch": round(us, 2),
                            "achieved_gbs": round(amt / (us * 1e-6) / 1e9, 1), "frac": round(amt / (us * 1e-6) / 1e9 / hbm, 4)}
        cpu = None
        if args.cpu_baseline and world == 1:
            cpu = cpu_baseline_sample(data)
        line = {
            "metric": METRIC, "value": args.seqs * K / t_value, "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": t_value / K * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "i8/f32", "data": "synthetic",
            "config": {"workload": "agent_decode", "seqs": args.seqs, "seqs_per_gpu": S, "prompt": PROMPT,
                       "decode_steps": n_steps, "timed_steps": [W, W + K],
                       "mask_allow": "uniform 5-50% of 16384 ids per (seq, step)",
                       "l2": "inputs larger than L2: ~0.8 GB of int8 KV read every step at 1024 sequences; the "
                             "31 MB of weights stay L2-resident as in serving",
                       "parallelism": f"{args.seqs} sequences partitioned over {world} GPU(s), no collective",
                       "model": "needle3-121M random-init CQ-W4 seed 0"},
            "e2e": {"value": args.seqs * K / t_e2e, "unit": "tok/s", "h2d_bytes_per_step": args.seqs * int(masks.shape[2]),
                    "d2h_bytes_per_step": args.seqs * 4},
            "gpu_launches": int(launches),
            "roofline": roofline,
            "sites": per_site,
            "cpu_baseline": cpu,
            "clocks": clk,
            "secondary": extra,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
