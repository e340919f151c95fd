"""Benchmark of the B200 HardShell backend: fold (prefill) throughput in input MB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload ("fold throughput"): the synthetic GPT-2 124M .hsm
(taco_b200/synth.py), 512 independent 1024-token windows of seeded Zipf text per GPU, all
positions of every window scored in one forward pass of its slot, each row answered by the coder
op (the interval of the coded token in FreqTable::from_weights(weights, 32)). One step = one
run_coded call over the 512 windows (passes of --max-rows rows). Windows are dealt to GPUs
(weak scaling: 512 per GPU, no collective on the data path; torch.distributed only for the
barrier and the max over ranks of the timings).

value  = input bytes of all ranks / max over ranks of the device time of the K steps (CUDA
         events around every pass on the batch stream, the token rows already on the device);
e2e    = the same bytes / wall time of K more C-ABI calls with host buffers, without the
         profiling events (row upload, planning, interval read back inside);
roofline = the kernel with the largest share of the pass time: algorithmic int8 ops (tensor-bound
         kernels) or algorithmic bytes (HBM-bound kernels) per launch / its mean CUDA-event launch
         time, against the int8 tensor peak measured in this run (torch._int_mm, cuBLASLt) or the
         measured HBM copy bandwidth (MEASURED_PEAKS.json); `rooflines` has every kernel class;
cpu_baseline = the CPU oracle's fast path (a C++ restatement of the reference CPU engine) on a
         bounded sample of the same windows, all host threads, rank 0 at N = 1.
Extra fields: the GEMM microbench, the unfold decode step, the unfold of
coded blocks with the range decoder on the device, the encoder op of the profile logs
(run_coded_dual), and the fold and unfold of the host library end to end (hs_fold, hs_unfold).
`--only fold_dual|fold_glue` runs one of the last two alone (profiling cases).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "fold/unfold input MB/s at 1/2/4/8 B200 (bit-exact); int8 GEMM % of peak"
WINDOWS, WINDOW = 512, 1024
NOMINAL_INT8_TOPS = 4500.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--windows", type=int, default=WINDOWS)
    ap.add_argument("--max-rows", type=int, default=16384)
    ap.add_argument("--no-extras", action="store_true", help="skip the GEMM microbench and the unfold step")
    ap.add_argument("--cpu-threads", type=int, default=0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline (profiling runs)")
    ap.add_argument("--no-peak", action="store_true", help="skip the int8 peak measurement (profiling runs)")
    ap.add_argument("--only", default="", choices=["", "fold_dual", "fold_glue"],
                    help="run one extra alone (profiling runs)")
    return ap.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def window_rows(tokens: np.ndarray, eot: int, slot0: int = 0):
    """The rows of whole windows (gpu_fold.rs:145 Window::rows for window 0 of a block): the
    inputs [EOT, t0 .. t(n-2)], each row coding the next token."""
    n_win, n = tokens.shape
    slots = np.repeat(np.arange(n_win, dtype=np.uint32) + slot0, n)
    inputs = np.concatenate([np.full((n_win, 1), eot, np.uint32), tokens[:, :-1]], axis=1).reshape(-1)
    coded = tokens.reshape(-1).astype(np.uint64)
    return slots, inputs, coded


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for name, v in zip(names, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def measured_int8_peak_tops(device: int) -> dict:
    """The dense int8 tensor peak of this GPU: torch._int_mm (cuBLASLt) on 8192^3, best of 10."""
    import torch

    torch.cuda.set_device(device)
    n = 8192
    a = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda")
    b = torch.randint(-127, 128, (n, n), dtype=torch.int8, device="cuda").t()
    for _ in range(3):
        torch._int_mm(a, b)
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch._int_mm(a, b)
        e1.record()
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    del a, b
    torch.cuda.empty_cache()
    return {"tops": 2.0 * n ** 3 / (best * 1e-3) / 1e12, "how": "torch._int_mm int8 8192^3, best of 10, CUDA events"}


def read_traffic() -> dict:
    """DRAM bytes (read + write) per launch of each kernel class, from the committed ncu summary of
    one 16384-row fold pass (the same pass shape as every pass of this benchmark)."""
    p = ROOT / "profiles" / "fold_pass_traffic.md"
    if not p.exists():
        return {}
    return {m.group(1): float(m.group(2))
            for m in re.finditer(r"traffic_bytes_per_launch\[(\w+)\]:\s*([0-9.eE+]+)", p.read_text())}


def measured_hbm_gbs() -> float | None:
    """The HBM copy bandwidth of MEASURED_PEAKS.json (driver-written), if present."""
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"])
    except (OSError, ValueError, KeyError):
        return None


def rooflines(prof: dict, info, peak_tops: float | None, hbm_gbs: float | None, traffic: dict) -> dict:
    """Achieved work per launch / mean launch time for each kernel class of the fold pass."""
    d, V, L = info.d_model, info.vocab, info.n_layer
    vt = (V + 127) // 128
    rows = prof["pass"]["ops"]  # the rows of the timed passes
    out = {}

    def add(name, keys, bound, work, unit):
        ms = sum(prof[k]["ms"] for k in keys if k in prof)
        launches = sum(prof[k]["launches"] for k in keys if k in prof)
        if not ms or not launches:
            return
        per_launch = work / launches
        achieved = per_launch / (ms * 1e-3 / launches) / (1e12 if bound == "tensor" else 1e9)
        peak = peak_tops if bound == "tensor" else hbm_gbs
        out[name] = {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                     "frac": achieved / peak if peak else None,
                     "traffic": traffic.get(name), "work_per_launch": per_launch,
                     "share": ms / prof["pass"]["ms"], "launches": launches,
                     "mean_launch_us": 1000 * ms / launches}

    gemm_keys = [k for k in prof if k.startswith("gemm")]
    add("gemm", gemm_keys, "tensor", sum(prof[k]["ops"] for k in gemm_keys), "TOP/s")
    add("attention", ["attention"], "tensor", prof["attention"]["ops"], "TOP/s")
    # LayerNorm: layer 0's first one reads x and writes a (5d bytes per row); the other 2L ones
    # also read the residual delta and write x back (13d bytes per row).
    add("layernorm", ["layernorm"], "hbm", rows * d * (5 + 13 * 2 * L), "GB/s")
    # The coder op: the row's logit distances (2V bytes) and tile maxima (8 per 128 symbols) in,
    # one interval (24 bytes) out.
    add("coder", ["coder"], "hbm", rows * (2 * V + 8 * vt + 24), "GB/s")
    # The embedding: two int8 rows in, the i32 residual row out.
    add("embed", ["embed"], "hbm", rows * (2 * d + 4 * d), "GB/s")
    return out


def cpu_baseline(model_bytes: bytes, windows: np.ndarray, eot: int, lens: np.ndarray, threads: int,
                 n_tokens: int) -> dict:
    """The CPU oracle's fast path on `threads` windows of `n_tokens` tokens (one window per thread)."""
    from oracle import oracle as O

    om = O.Model(model_bytes)
    sample = windows[:threads, :n_tokens]
    fb = O.FastBatch(om, sample.shape[0], 0)
    slots, inputs, coded = window_rows(sample, eot)
    t0 = time.perf_counter()
    fb.run_coded(slots, inputs, np.zeros(slots.size, np.uint32), coded, 32, threads=threads)
    dt = time.perf_counter() - t0
    nbytes = int(lens[coded.astype(np.int64)].sum())
    return {"value": nbytes / dt / 1e6, "unit": "MB/s", "cores": threads, "kind": "port",
            "tokens_per_s": slots.size / dt,
            "sample": f"{sample.shape[0]} windows x {n_tokens} tokens (positions 0..{n_tokens - 1}), "
                      f"{nbytes} input bytes, {dt:.1f} s, one window per thread"}


def run_reference(args, world, rank):
    """--impl reference: the CPU oracle port of the reference CPU engine, timed on the host cores."""
    if rank != 0:
        return 0
    from taco_b200 import synth

    model = synth.gpt2_hsm(124)
    vocab = synth.vocabulary()
    lens = synth.token_lengths(vocab)
    threads = args.cpu_threads or os.cpu_count() or 1
    n_tok = 256
    wins = synth.zipf_windows(threads, n_tok, seed=1000)
    from oracle import oracle as O

    om = O.Model(model)
    slots, inputs, coded = window_rows(wins, synth.VOCAB - 1)
    nbytes = int(lens[coded.astype(np.int64)].sum())
    for _ in range(args.warmup):
        fb = O.FastBatch(om, threads, 0)
        fb.run_coded(slots, inputs, np.zeros(slots.size, np.uint32), coded, 32, threads=threads)
    times = []
    for _ in range(args.steps):
        fb = O.FastBatch(om, threads, 0)
        t0 = time.perf_counter()
        fb.run_coded(slots, inputs, np.zeros(slots.size, np.uint32), coded, 32, threads=threads)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = nbytes * args.steps / total / 1e6
    sample = f"{threads} windows x {n_tok} tokens per step ({nbytes} input bytes), one window per thread"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "MB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/int32/int64",
        "data": "synthetic", "config": {"workload": "fold throughput (configs[2]) sample on host cores",
                                         "model": "GPT-2 124M synthetic .hsm", "window": n_tok},
        "cpu_baseline": {"value": value, "unit": "MB/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "MB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "tokens_per_s": slots.size * args.steps / total,
        "note": "the reference is Rust (cargo absent, crates not vendored): its CPU engine runs as the C++ "
                "oracle port (oracle/), a restatement of crates/hardshell with the same chunked prefill",
    }
    print(json.dumps(line))
    return 0


def main():
    args = parse_args()
    world, rank, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, world, rank)

    import torch

    pg = False
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
        pg = True

    from taco_b200 import backend as B
    from taco_b200 import shard, synth

    model_bytes = synth.gpt2_hsm(124)
    vocab = synth.vocabulary()
    lens = synth.token_lengths(vocab)
    eot = synth.VOCAB - 1
    # The job: windows x world windows of seeded text, dealt round-robin to the GPUs (weak scaling:
    # each GPU gets `windows`); no collective touches them.
    n_total = args.windows * world
    all_windows = synth.zipf_windows(n_total, WINDOW, seed=1000)
    windows = all_windows[shard.deal(n_total, world, rank)]
    slots, inputs, coded = window_rows(windows, eot)
    kinds = np.zeros(slots.size, np.uint32)
    step_bytes = int(lens[coded.astype(np.int64)].sum())
    if args.only:
        dev = B.CudaDevice(local)
        model = B.CudaModel(dev, model_bytes)
        if args.only == "fold_dual":
            print(json.dumps({"fold_dual": fold_dual(B, model, windows, lens, eot, sample=args.windows)}))
        else:
            print(json.dumps({"fold_glue": fold_glue(B, model, model_bytes, vocab)}))
        model.close()
        dev.close()
        return 0

    peak = measured_int8_peak_tops(local) if rank == 0 and not args.no_peak else None
    dev = B.CudaDevice(local)
    model = B.CudaModel(dev, model_bytes)
    batch = B.CudaBatch(model, args.windows, args.max_rows)

    def step():
        for s in range(args.windows):
            batch.reset(s)
        return batch.run_coded(slots, inputs, kinds, coded, 32)

    # Warm-up; the first answers are checked for their symbols (the coded tokens).
    for i in range(args.warmup):
        ans = step()
    if not np.array_equal(ans["symbol"].astype(np.uint64), coded):
        raise SystemExit("the coder op answered the wrong symbols")

    def barrier():
        torch.cuda.synchronize(local)
        if pg:
            torch.distributed.barrier()

    barrier()
    clocks = ClockSampler(local)
    clocks.start()
    # The device time: K steps with per-op CUDA events on the batch stream.
    batch.set_profiling(True)
    launches0 = B.launch_count()
    for _ in range(args.steps):
        step()
    launches = B.launch_count() - launches0
    prof = batch.profile()
    batch.set_profiling(False)
    # End to end: K more steps through the C-ABI with host buffers, timed by the wall clock
    # without the profiling events.
    wall = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        wall.append(time.perf_counter() - t0)
    barrier()
    clk = clocks.stop()

    dev_s, wall_s = shard.max_over_ranks([prof["pass"]["ms"] / 1e3, sum(wall)], device=f"cuda:{local}")
    total_bytes = step_bytes * args.steps * world
    total_rows = slots.size * args.steps * world

    gemm_ops = sum(prof[k]["ops"] for k in prof if k.startswith("gemm"))
    gemm_ms = sum(prof[k]["ms"] for k in prof if k.startswith("gemm"))
    gemm_launches = sum(prof[k]["launches"] for k in prof if k.startswith("gemm"))
    achieved = gemm_ops / (gemm_ms * 1e-3) / 1e12 if gemm_ms else 0.0

    result = None
    if rank == 0:
        kernels = {k: {"ms": round(v["ms"], 3), "launches": v["launches"],
                       "share": round(v["ms"] / prof["pass"]["ms"], 4) if prof["pass"]["ms"] else None}
                   for k, v in prof.items() if k != "pass"}
        for k in kernels:
            if prof[k]["ops"] and prof[k]["ms"]:
                kernels[k]["tops"] = round(prof[k]["ops"] / (prof[k]["ms"] * 1e-3) / 1e12, 1)
        roofs = rooflines(prof, model.info, peak["tops"] if peak else None, measured_hbm_gbs(), read_traffic())
        dominant = max(roofs, key=lambda k: roofs[k]["share"])
        roof = dict(roofs[dominant], kernel=dominant)
        roof["peak_source"] = ((peak["how"] if peak else None) if roof["bound"] == "tensor"
                               else "MEASURED_PEAKS.json hbm_gbs (STREAM-style copy)")
        result = {
            "metric": METRIC, "value": total_bytes / dev_s / 1e6, "unit": "MB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * dev_s / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic",
            "config": {"workload": "fold throughput (BASELINE configs[2]): 512 windows x 1024 tokens per GPU, "
                                   "all positions in one forward pass per window, coder interval per row",
                       "model": "GPT-2 124M .hsm from seeded N(0,0.02) (taco_b200/synth.py)",
                       "windows_per_gpu": args.windows, "window_tokens": WINDOW, "max_rows_per_pass": args.max_rows,
                       "parallelism": f"{n_total} windows dealt round-robin to {world} GPU(s), no collective",
                       "l2": "inputs larger than L2: each step streams 124 MB of weights per pass and "
                             "9.7 GB of KV cache"},
            "tokens_per_s": total_rows / dev_s,
            "e2e": {"value": total_bytes / wall_s / 1e6, "unit": "MB/s",
                    "h2d_bytes_per_step": int(slots.size * 24), "d2h_bytes_per_step": int(slots.size * 24)},
            "roofline": roof,
            "rooflines": roofs,
            "gemm_frac_of_nominal_4500": achieved / NOMINAL_INT8_TOPS,
            "clocks": clk,
            "gpu_launches": launches,
            "kernels": kernels,
        }

    # Extras: the GEMM microbench and one unfold decode step.
    if rank == 0 and not args.no_extras:
        micro = {}
        for (K, N) in [(768, 2304), (768, 768), (768, 3072), (3072, 768), (768, 50257)]:
            n16 = (N + 15) // 16 * 16
            us = dev.linear_bench(8192, n16, K, seed=7, warmup=3, iters=20)
            tops = 2.0 * 8192 * N * K / (us * 1e-6) / 1e12
            micro[f"M8192_K{K}_N{N}"] = {"us": round(us, 2), "tops": round(tops, 1),
                                        "frac": round(tops / peak["tops"], 3) if peak else None}
        result["gemm_microbench"] = micro
        result["unfold"] = unfold_step(B, model, lens, eot, clock_note=None)
        result["unfold_blocks"] = unfold_blocks(B, model)
        result["fold_dual"] = fold_dual(B, model, windows, lens, eot)
        result["fold_glue"] = fold_glue(B, model, model_bytes, vocab)
    if rank == 0:
        if world == 1 and not args.no_cpu:
            threads = args.cpu_threads or os.cpu_count() or 1
            result["cpu_baseline"] = cpu_baseline(model_bytes, windows, eot, lens, threads, 1024)
        print(json.dumps(result))
    batch.close()
    model.close()
    dev.close()
    if pg:
        torch.distributed.destroy_process_group()
    return 0


def unfold_step(B, model, lens, eot, clock_note=None, streams: int = 1024, context: int = 512, steps: int = 16) -> dict:
    """1024 streams decoded token by token. The streams are filled to `context`
    positions (prefill, not timed), then `steps` decode steps (one row per stream, the coder
    op answering a decode query for each row: the symbol whose interval holds a seeded 32-bit
    target) are timed with the wall clock around the C-ABI calls (end to end, no profiling), and
    the next `steps` steps on the device (per-op CUDA events). The next input of a stream is the
    text's own next token, so the rows are those of a real unfold."""
    from taco_b200 import synth

    toks = synth.zipf_windows(streams, context + 2 * steps, seed=77)
    batch = B.CudaBatch(model, streams, 16384)
    slots, inputs, coded = window_rows(toks[:, :context], eot)
    batch.run_coded(slots, inputs, np.zeros(slots.size, np.uint32), coded, 32)
    sl = np.arange(streams, dtype=np.uint32)
    kinds = np.ones(streams, np.uint32)
    targets = np.random.default_rng(78).integers(0, 1 << 32, (2 * steps, streams), dtype=np.uint64)
    t0 = time.perf_counter()
    for i in range(steps):
        batch.run_coded(sl, toks[:, context + i - 1], kinds, targets[i], 32)
    wall = time.perf_counter() - t0
    batch.set_profiling(True)
    for i in range(steps, 2 * steps):
        batch.run_coded(sl, toks[:, context + i - 1], kinds, targets[i], 32)
    prof = batch.profile()
    batch.close()
    dev_s = prof["pass"]["ms"] / 1e3
    nbytes = int(lens[toks[:, context + steps:context + 2 * steps].astype(np.int64)].sum())
    kv_read = streams * steps * 2 * 12 * 768 * (context + 1.5 * steps)
    return {"streams": streams, "positions": f"{context}..{context + steps - 1} (end to end), "
            f"{context + steps}..{context + 2 * steps - 1} (device)", "steps": steps,
            "tokens_per_s": streams * steps / dev_s, "MB_per_s": nbytes / dev_s / 1e6,
            "e2e_tokens_per_s": streams * steps / wall,
            "kv_GB_per_s": kv_read / dev_s / 1e9,
            "attention_share": round(prof["attention"]["ms"] / prof["pass"]["ms"], 3),
            "kernels_ms_per_step": {k: round(v["ms"] / steps, 3) for k, v in prof.items() if v["launches"]}}


def unfold_blocks(B, model, streams: int = 1024, tokens: int = 256) -> dict:
    """configs[3] with the range decoder on the device: `streams` coded blocks of `tokens` tokens,
    unfolded from position 0 by one hs_batch_decode_blocks call (no host round trip per token),
    against the same rows driven step by step through run_coded with decode queries (one host
    round trip per step, the structure of the reference's unfold loop; its targets here are
    seeded, as a host decoder's would be). The payloads are seeded random bytes: the decoder turns
    any input into symbols, and the work of a step does not depend on the bytes. Both arms are
    timed by the wall clock around the C-ABI calls, the better of two runs each; the device time
    of the decoder arm comes from a third, profiled call."""
    rng = np.random.default_rng(79)
    payloads = [rng.integers(0, 256, 4 * tokens, dtype=np.uint8).tobytes() for _ in range(streams)]
    sl = np.arange(streams, dtype=np.uint32)
    batch = B.CudaBatch(model, streams, 4096)
    batch.decode_blocks(sl[:8], payloads[:8], [4] * 8, 32)  # warm-up
    wall = float("inf")
    for _ in range(2):  # the better of two calls, for each arm
        t0 = time.perf_counter()
        toks, status = batch.decode_blocks(sl, payloads, [tokens] * streams, 32)
        wall = min(wall, time.perf_counter() - t0)
    batch.set_profiling(True)
    batch.decode_blocks(sl, payloads, [tokens] * streams, 32)
    prof = batch.profile()
    batch.set_profiling(False)
    dev_ms = prof["pass"]["ms"] + prof.get("decoder", {"ms": 0.0})["ms"]
    # The host loop over run_coded, from position 0 as well.
    targets = rng.integers(0, 1 << 32, (tokens, streams), dtype=np.uint64)
    kinds = np.ones(streams, np.uint32)
    wall_host = float("inf")
    for _ in range(2):
        for s in range(streams):
            batch.reset(s)
        inp = np.full(streams, model.eot_token(), np.uint32)
        t0 = time.perf_counter()
        for j in range(tokens):
            iv = batch.run_coded(sl, inp, kinds, targets[j], 32)
            inp = iv["symbol"].astype(np.uint32)
        wall_host = min(wall_host, time.perf_counter() - t0)
    batch.close()
    n = streams * tokens
    return {"streams": streams, "tokens_per_block": tokens, "positions": f"0..{tokens - 1}",
            "e2e_tokens_per_s": n / wall, "device_tokens_per_s": n / (dev_ms / 1e3),
            "host_loop_e2e_tokens_per_s": n / wall_host, "failed_blocks": int(status.sum()),
            "decoder_ms": round(prof.get("decoder", {"ms": 0.0})["ms"], 3)}


def fold_dual(B, model, windows, lens, eot, sample: int = 64) -> dict:
    """The encoder op of the profile logs (run_coded_dual: the interval of each coded token in the
    table of GPT-2 alone and in the mixed table of a prediction) on `sample` fold windows, against
    run_coded on the same rows. The predictions are those of a stand-in match model (the token
    that followed the last earlier occurrence of the input token in the window); the host mixer is
    a Python callback (q from the agreement bit), called once per predicted row as the reference's
    is. Timed by the wall clock around the C-ABI calls (the better of two), with the per-op device
    time from a third, profiled call; a mixed pass includes its host step (the statistics read
    back, the mixer calls and the records upload) inside the pass time."""
    w = windows[:sample]
    slots, inputs, coded = window_rows(w, eot)
    preds = np.full(slots.size, B.MIX_NONE, np.uint32)
    for r in range(w.shape[0]):
        seen = {}
        base = r * w.shape[1]
        for j in range(w.shape[1]):
            i = base + j
            p = seen.get(int(inputs[i]))
            if p is not None:
                preds[i] = p
            seen[int(inputs[i])] = int(coded[i])
    kinds = np.zeros(slots.size, np.uint32)
    nbytes = int(lens[coded.astype(np.int64)].sum())

    def mixer(i, total, predicted, top):
        return 52000 if top == preds[i] else 13000

    batch = B.CudaBatch(model, sample, 16384)

    def run(dual: bool):
        for s in range(sample):
            batch.reset(s)
        if dual:
            return batch.run_coded_dual(slots, inputs, coded, preds, 32, mixer)
        return batch.run_coded(slots, inputs, kinds, coded, 32)

    plain, mixed = run(True)
    if not (np.array_equal(plain["symbol"], coded) and np.array_equal(mixed["symbol"], coded)):
        raise SystemExit("the dual coder op answered the wrong symbols")
    out = {"windows": sample, "rows": int(slots.size), "predicted_rows": int((preds != B.MIX_NONE).sum())}
    for name, dual in (("dual", True), ("plain", False)):
        wall = float("inf")
        for _ in range(2):
            t0 = time.perf_counter()
            run(dual)
            wall = min(wall, time.perf_counter() - t0)
        batch.set_profiling(True)
        run(dual)
        prof = batch.profile()
        batch.set_profiling(False)
        out[name] = {"e2e_MB_per_s": nbytes / wall / 1e6, "device_MB_per_s": nbytes / (prof["pass"]["ms"] / 1e3) / 1e6,
                     "pass_ms": round(prof["pass"]["ms"], 3), "coder_ms": round(prof["coder"]["ms"], 3),
                     "coder_launches": prof["coder"]["launches"]}
    batch.close()
    return out


def fold_glue(B, model, model_bytes, vocab, mb: int = 2) -> dict:
    """The fold and the unfold of the profile text end to end through the host library (hs_fold,
    hs_unfold: tokenizer, zstd level 19, the coder op on the GPU, range encoder, container) on `mb`
    MiB of seeded Zipf text (the bytes of the synthetic vocabulary's word tokens), default block
    size 16 KiB, one slot per block. The synthetic vocabulary has no merges, so the tokenizer gives
    one token per byte (about 4.6 times the rows of the bench's token windows per byte). Timed by
    the wall clock (the better of two); the device time of the fold's passes from a third,
    profiled call. A random-initialised model rarely beats zstd, so the unfold mostly decodes zstd
    frames: it measures the glue, not the coder."""
    from taco_b200 import synth

    w = synth.zipf_windows(256, 1024, seed=4242)
    text = b"".join(vocab[t] for t in w.reshape(-1).tolist())[: mb << 20]
    tok = B.Tokenizer(model_bytes)
    batch = B.CudaBatch(model, 256, 16384)
    B.fold(batch, tok, text[:20000])  # warm-up
    wall = float("inf")
    for _ in range(2):
        t0 = time.perf_counter()
        got, stats = B.fold(batch, tok, text)
        wall = min(wall, time.perf_counter() - t0)
    batch.set_profiling(True)
    B.fold(batch, tok, text)
    prof = batch.profile()
    batch.set_profiling(False)
    uwall = float("inf")
    for _ in range(2):
        t0 = time.perf_counter()
        back = B.unfold(batch, tok, got)
        uwall = min(uwall, time.perf_counter() - t0)
    if back != text:
        raise SystemExit("the unfold did not give the input back")
    batch.close()
    tok.close()
    return {"input_bytes": len(text), "blocks": stats["blocks"], "tokens": stats["tokens"],
            "coded_blocks": stats["coded_blocks"], "zstd_blocks": stats["zstd_blocks"],
            "container_bytes": stats["container_len"],
            "fold_e2e_MB_per_s": len(text) / wall / 1e6, "fold_device_ms": round(prof["pass"]["ms"], 3),
            "fold_wall_ms": round(wall * 1e3, 3), "fold_device_share": round(prof["pass"]["ms"] / (wall * 1e3), 3),
            "unfold_e2e_MB_per_s": len(text) / uwall / 1e6}


if __name__ == "__main__":
    sys.exit(main())
