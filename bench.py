"""Benchmark of the B200 HardShell backend: fold (prefill) throughput in input MB/s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload ("fold throughput"): the synthetic GPT-2 124M .hsm
(taco_b200/synth.py) and 512 independent 1024-token windows per GPU: consecutive runs of the tokens
of seeded Zipf text (the synthetic vocabulary is byte-level BPE with merges, so the tokens are what
the fold's tokenizer makes of the text, and the bytes a window codes are text bytes). All positions
of every window are scored in one forward pass of its slot, each row answered by the coder op (the
interval of the coded token in FreqTable::from_weights(weights, 32)). One step = one run_coded call
over the 512 windows (passes of --max-rows rows). Windows are dealt to GPUs (weak scaling: 512 per
GPU, no collective on the data path; torch.distributed only for barriers and the max over ranks of
the timings).

value  = input bytes of all ranks / max over ranks of the device time of the K steps (CUDA
         events around every pass on the batch stream, the token rows already on the device);
e2e    = the same bytes / wall time of K more C-ABI calls with host buffers, without the
         profiling events (row upload, planning, interval read back inside);
parity = rank 0 compares the intervals (symbol, start, freq) of windows spread evenly over the
         timed step (512 slots, passes of --max-rows rows; the first and the last window of the
         step among them, so the rows at both ends of a pass are checked) with the CPU oracle's,
         field by field; a mismatch fails the run;
roofline = the kernel with the largest share of the pass time: algorithmic int8 ops (tensor-bound
         kernels) or algorithmic bytes (HBM-bound kernels) per launch / its mean CUDA-event launch
         time, against the int8 tensor peak measured in this run (torch._int_mm, cuBLASLt) or the
         measured HBM copy bandwidth (MEASURED_PEAKS.json); `rooflines` has every kernel class;
cpu_baseline = the CPU oracle's fast path (a C++ restatement of the reference CPU engine) on the
         parity windows, one window per host thread, rank 0 at N = 1.
Extra fields: the GEMM microbench (configs[1], M = 1024, 8192, 65536, each shape checked exactly
once), the unfold decode step over contexts 1 to 1024, the unfold of coded blocks with
the range decoder on the device on every rank (unfold at N GPUs) next to the CPU unfold (the
oracle's lockstep lanes), the encoder op of the profile logs (run_coded_dual), the fold and unfold
of the host library end to end (hs_fold, hs_unfold), and the 256 MiB mixed input of configs[4]
folded by hs_fold_multi on all N GPUs (`large_input`, with its SHA-256).
`--only fold_dual|fold_glue|large_input` runs one of those alone (profiling cases).
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
PARITY_WINDOWS = 16
NOMINAL_INT8_TOPS = 4500.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--windows", type=int, default=WINDOWS)
    ap.add_argument("--max-rows", type=int, default=65536)
    ap.add_argument("--no-extras", action="store_true", help="skip the GEMM microbench and the unfold step")
    ap.add_argument("--cpu-threads", type=int, default=0)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline (profiling runs)")
    ap.add_argument("--no-peak", action="store_true", help="skip the int8 peak measurement (profiling runs)")
    ap.add_argument("--only", default="", choices=["", "fold_dual", "fold_glue", "large_input", "unfold"],
                    help="run one extra alone (profiling runs)")
    ap.add_argument("--large-mb", type=int, default=256, help="configs[4] input size in MiB (0 = skip)")
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
    """DRAM bytes (read + write) per launch of each kernel class at this benchmark's 65,536-row
    passes, from the committed ncu summary (a 16,384-row pass captured, scaled by the rows)."""
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


def oracle_windows(model_bytes: bytes, windows: np.ndarray, eot: int, lens: np.ndarray, threads: int) -> dict:
    """The CPU oracle's fast path on `windows` (one window per host thread at a time): its
    answers {symbol, start, freq} per row, and its speed (the bench's cpu_baseline)."""
    from oracle import oracle as O

    om = O.Model(model_bytes)
    fb = O.FastBatch(om, windows.shape[0], 0)
    slots, inputs, coded = window_rows(windows, eot)
    t0 = time.perf_counter()
    ans = fb.run_coded(slots, inputs, np.zeros(slots.size, np.uint32), coded, 32, threads=threads)
    dt = time.perf_counter() - t0
    nbytes = int(lens[coded.astype(np.int64)].sum())
    return {"answers": ans, "value": nbytes / dt / 1e6, "unit": "MB/s", "cores": threads, "kind": "port",
            "tokens_per_s": slots.size / dt,
            "sample": f"{windows.shape[0]} windows x {windows.shape[1]} tokens (positions 0..{windows.shape[1] - 1}), "
                      f"{nbytes} input bytes, {dt:.1f} s, one window per thread"}


def run_reference(args, world, rank):
    """--impl reference: the CPU oracle port of the reference CPU engine, timed on the host cores,
    on the bench's own configuration: the same text windows of 1024 tokens, all positions scored.
    A step is one window per host thread (the smallest sample that keeps every thread busy); the
    warm-up steps run one window of 64 tokens each. The windows are tokenized by the Python
    restatement of the BPE (taco_b200/synth.py tokenize_text), not this repository's engine."""
    if rank != 0:
        return 0
    from oracle import oracle as O
    from taco_b200 import synth

    model = synth.gpt2_hsm(124)
    vocab = synth.vocabulary()
    lens = synth.token_lengths(vocab)
    eot = synth.VOCAB - 1
    threads = args.cpu_threads or os.cpu_count() or 1
    wins = synth.text_windows(threads, WINDOW, seed=1000)
    om = O.Model(model)
    slots, inputs, coded = window_rows(wins, eot)
    nbytes = int(lens[coded.astype(np.int64)].sum())
    ws, wi, wc = window_rows(wins[:1, :64], eot)
    for _ in range(args.warmup):
        fb = O.FastBatch(om, 1, 0)
        fb.run_coded(ws, wi, np.zeros(ws.size, np.uint32), wc, 32, threads=1)
    times = []
    for _ in range(args.steps):
        fb = O.FastBatch(om, threads, 0)
        t0 = time.perf_counter()
        fb.run_coded(slots, inputs, np.zeros(slots.size, np.uint32), coded, 32, threads=threads)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = nbytes * args.steps / total / 1e6
    sample = (f"{threads} windows x {WINDOW} tokens per step ({nbytes} input bytes), one window per thread; "
              "warm-up steps: one window of 64 tokens")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "MB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8/int32/int64",
        "data": "synthetic",
        "config": {"workload": "fold throughput (BASELINE configs[2]): 1024-token windows of Zipf text, all "
                               "positions scored, coder interval per row; a step holds one window per host thread",
                   "model": "GPT-2 124M .hsm from seeded N(0,0.02) (taco_b200/synth.py)",
                   "window_tokens": WINDOW, "windows_per_step": threads, "same_config": True},
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
    all_windows = synth.text_windows(n_total, WINDOW, seed=1000)
    windows = all_windows[shard.deal(n_total, world, rank)]
    slots, inputs, coded = window_rows(windows, eot)
    kinds = np.zeros(slots.size, np.uint32)
    step_bytes = int(lens[coded.astype(np.int64)].sum())
    if args.only:
        if args.only == "large_input":
            print(json.dumps({"large_input": large_input(B, model_bytes, args.large_mb, [local], args.max_rows)}))
            return 0
        dev = B.CudaDevice(local)
        model = B.CudaModel(dev, model_bytes)
        if args.only == "fold_dual":
            print(json.dumps({"fold_dual": fold_dual(B, model, windows, lens, eot, sample=args.windows)}))
        elif args.only == "unfold":
            print(json.dumps({"unfold": unfold_sweep(B, model, lens, eot)}))
        else:
            print(json.dumps({"fold_glue": fold_glue(B, model, model_bytes, args.max_rows)}))
        model.close()
        dev.close()
        return 0

    peak = measured_int8_peak_tops(local) if rank == 0 and not args.no_peak else None
    dev = B.CudaDevice(local)
    model = B.CudaModel(dev, model_bytes)
    batch = B.CudaBatch(model, args.windows, args.max_rows)

    # The answers land in one host buffer for every step, as a caller coding batch after batch
    # keeps its output buffer.
    ans_buf = np.zeros(slots.size, dtype=B.INTERVAL_DTYPE)

    def step():
        for s in range(args.windows):
            batch.reset(s)
        return batch.run_coded(slots, inputs, kinds, coded, 32, out=ans_buf)

    # Warm-up; the answers of the last one are checked: the symbols here, the intervals of the
    # first windows against the oracle below.
    for i in range(args.warmup):
        ans = step()
    ans = ans.copy()  # the buffer is reused by the timed steps
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
    achieved = gemm_ops / (gemm_ms * 1e-3) / 1e12 if gemm_ms else 0.0

    # The unfold on every GPU at once (configs[3] at N GPUs): each rank decodes its own coded
    # blocks with the device range decoder, timed between barriers, the max over ranks.
    ub = ub_timed = None
    if not args.no_extras:
        ub = unfold_blocks(B, model, lens)
        ub_batch = B.CudaBatch(model, 1024, 4096)
        unfold_blocks(B, model, lens, timed_only=True, batch=ub_batch)  # warm
        barrier()
        t0 = time.perf_counter()
        ub_timed = unfold_blocks(B, model, lens, timed_only=True, batch=ub_batch)
        ub_wall = time.perf_counter() - t0
        barrier()
        ub_batch.close()
        (ub_max,) = shard.max_over_ranks([ub_wall], device=f"cuda:{local}")

    result = None
    failed = False
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
            "config": {"workload": "fold throughput (BASELINE configs[2]): 512 windows x 1024 tokens per GPU of "
                                   "tokenized Zipf text, all positions in one forward pass per window, coder "
                                   "interval per row",
                       "model": "GPT-2 124M .hsm from seeded N(0,0.02) with a byte-level BPE vocabulary and merges "
                                "(taco_b200/synth.py)",
                       "windows_per_gpu": args.windows, "window_tokens": WINDOW, "max_rows_per_pass": args.max_rows,
                       "bytes_per_token": round(step_bytes / slots.size, 3),
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
        if ub_timed:
            result["unfold_gpus"] = {
                "n_gpus": world, "streams_per_gpu": ub_timed["streams"], "tokens_per_block": ub_timed["tokens_per_block"],
                "e2e_tokens_per_s": world * ub_timed["tokens"] / ub_max,
                "e2e_MB_per_s": world * ub_timed["bytes"] / ub_max / 1e6,
                "timing": "wall clock of one hs_batch_decode_blocks call per rank (its batch made beforehand) between "
                          "barriers, max over ranks",
                "per_rank_first_call": {k: ub[k] for k in ("e2e_tokens_per_s", "device_tokens_per_s")}}
        # Parity on the bench's own shape: the intervals of windows spread evenly over the last
        # warm-up step (512 slots, passes of max_rows rows; the first and the last window among
        # them) against the oracle's, field by field.
        threads = args.cpu_threads or os.cpu_count() or 1
        n_par = max(PARITY_WINDOWS, threads) if world == 1 else PARITY_WINDOWS
        n_par = min(n_par, args.windows)
        pick = np.unique(np.linspace(0, args.windows - 1, n_par).round().astype(np.int64))
        n_par = pick.size
        ora = oracle_windows(model_bytes, windows[pick], eot, lens, threads)
        got = np.stack([ans["symbol"], ans["start"], ans["freq"]], 1).astype(np.uint64)
        got = got.reshape(args.windows, WINDOW, 3)[pick].reshape(-1, 3)
        bad = np.any(got != ora["answers"], axis=1)
        result["parity"] = {"windows": int(n_par), "rows": int(n_par * WINDOW), "pass_rows": args.max_rows,
                            "window_indices": [int(w) for w in pick],
                            "slots": args.windows, "fields": ["symbol", "start", "freq"],
                            "mismatches": int(bad.sum()),
                            "against": "CPU oracle fast path (oracle/), the same windows"}
        failed = bool(bad.any())
        if world == 1 and not args.no_cpu:
            result["cpu_baseline"] = {k: v for k, v in ora.items() if k != "answers"}

    # Extras: the GEMM microbench, the unfold sweep and the CPU unfold.
    if rank == 0 and not args.no_extras:
        result["gemm_microbench"] = gemm_microbench(dev, peak)
        result["unfold"] = unfold_sweep(B, model, lens, eot)
        result["unfold_blocks"] = ub
        threads = args.cpu_threads or os.cpu_count() or 1
        cpu_u = unfold_cpu(model_bytes, eot, threads)
        result["unfold_cpu_baseline"] = cpu_u
        result["unfold_ratio"] = {
            "e2e_device_decoder_vs_cpu": ub["e2e_tokens_per_s"] / cpu_u["tokens_per_s"],
            f"gpus_{world}_vs_cpu": result["unfold_gpus"]["e2e_tokens_per_s"] / cpu_u["tokens_per_s"],
            "note": "tokens/s of the device decoder (1,024 blocks x 256 tokens from position 0, wall clock) over the "
                    "CPU oracle's lockstep-lane decode from position 0 on all host threads"}
        result["fold_dual"] = fold_dual(B, model, windows, lens, eot)
        result["fold_glue"] = fold_glue(B, model, model_bytes, args.max_rows)
    batch.close()
    model.close()
    dev.close()
    # the large mixed input through hs_fold_multi on every GPU of the job, from rank 0
    # after every rank has freed its handles.
    if args.large_mb and not args.no_extras:
        if pg:
            torch.distributed.barrier()
        if rank == 0:
            result["large_input"] = large_input(B, model_bytes, args.large_mb, list(range(world)), args.max_rows)
        if pg:
            torch.distributed.barrier()
    if rank == 0:
        print(json.dumps(result))
    if pg:
        torch.distributed.destroy_process_group()
    if failed:
        print("parity: the GPU intervals differ from the oracle's", file=sys.stderr)
        return 1
    return 0


def gemm_microbench(dev, peak) -> dict:
    """the linear op on device-resident int8 operands (hs_op_linear_bench, CUDA events
    over 20 launches after 3) at M = 1024, 8192 and 65536 for the five GPT-2 shapes (N rounded up
    to 16). Each shape is also checked exactly once at M = 1024 through the host-buffer op: the
    int32 accumulators against A . W^T (float64 BLAS, exact below 2^53) and the requantised int8
    against the rule of ops.rs:434 (LinearOut::Act)."""
    micro = {}
    rng = np.random.default_rng(12)
    for (K, N) in [(768, 2304), (768, 768), (768, 3072), (3072, 768), (768, 50257)]:
        n16 = (N + 15) // 16 * 16
        for M in (1024, 8192, 65536):
            us = dev.linear_bench(M, n16, K, seed=7, warmup=3, iters=20)
            tops = 2.0 * M * N * K / (us * 1e-6) / 1e12
            micro[f"M{M}_K{K}_N{N}"] = {"us": round(us, 2), "tops": round(tops, 1),
                                        "frac": round(tops / peak["tops"], 3) if peak else None}
        A = rng.integers(-127, 128, (1024, K), dtype=np.int8)
        W = rng.integers(-127, 128, (n16, K), dtype=np.int8)
        b = rng.integers(-2**20, 2**20, n16).astype(np.int32)
        m = rng.integers(1 << 30, 1 << 31, n16).astype(np.int32)
        sh = 38
        raw = dev.matmul_raw(A, W)
        want = A.astype(np.float64) @ W.astype(np.float64).T
        exact_raw = bool(np.array_equal(raw.astype(np.float64), want))
        y = dev.linear_act(A, W, b, m, sh)
        p = (want.astype(np.int64) + b.astype(np.int64)) * m.astype(np.int64)
        yw = np.clip((p >> sh) + ((p >> (sh - 1)) & 1), -127, 127).astype(np.int8)
        micro[f"exact_K{K}_N{N}"] = {"M": 1024, "int32": exact_raw, "requant_int8": bool(np.array_equal(y, yw))}
        if not (exact_raw and np.array_equal(y, yw)):
            raise SystemExit(f"the GEMM microbench shape K={K} N={N} is not exact")
    return micro


def unfold_sweep(B, model, lens, eot, streams: int = 1024, steps: int = 8,
                 points=(0, 128, 256, 384, 512, 640, 768, 896, 1008)) -> dict:
    """1024 streams decoded token by token with the context growing from 1 to 1024.
    The streams are filled (prefill, not timed) to each point p, then `steps` decode steps (one row
    per stream, a decode query with a seeded 32-bit target each) are timed end to end (the wall
    clock around the C-ABI calls), and the next `steps` on the device (per-op CUDA events). Each
    stream's next input is its text's own next token, so the rows are those of a real unfold.
    The KV cache read per step is streams x 2 x L x d bytes per context position."""
    from taco_b200 import synth

    toks = synth.text_windows(streams, 1024, seed=77)
    info = model.info
    batch = B.CudaBatch(model, streams, 16384)
    sl = np.arange(streams, dtype=np.uint32)
    kinds = np.ones(streams, np.uint32)
    rng = np.random.default_rng(78)
    pos, out = 0, []

    def inputs_at(j):
        return np.full(streams, eot, np.uint32) if j == 0 else toks[:, j - 1]

    for p in points:
        if p > pos:  # prefill rows pos .. p - 1 of every stream, slot-major
            cols = np.arange(pos, p)
            inp = np.stack([inputs_at(j) for j in cols], 1).reshape(-1)
            s = np.repeat(sl, cols.size)
            batch.run_coded(s, inp, np.zeros(s.size, np.uint32), toks[:, pos:p].reshape(-1).astype(np.uint64), 32)
        t0 = time.perf_counter()
        for j in range(p, p + steps):
            batch.run_coded(sl, inputs_at(j), kinds, rng.integers(0, 1 << 32, streams, dtype=np.uint64), 32)
        wall = time.perf_counter() - t0
        batch.set_profiling(True)
        for j in range(p + steps, p + 2 * steps):
            batch.run_coded(sl, inputs_at(j), kinds, rng.integers(0, 1 << 32, streams, dtype=np.uint64), 32)
        prof = batch.profile()
        batch.set_profiling(False)
        pos = p + 2 * steps
        dev_s = prof["pass"]["ms"] / 1e3
        kv = streams * steps * 2 * info.n_layer * info.d_model * (p + steps + (steps + 1) / 2)
        out.append({"context": f"{p + steps + 1}..{p + 2 * steps}", "tokens_per_s": streams * steps / dev_s,
                    "e2e_tokens_per_s": streams * steps / wall, "kv_GB_per_s": kv / dev_s / 1e9,
                    "ms_per_step": round(1000 * dev_s / steps, 3),
                    "attention_share": round(prof["attention"]["ms"] / prof["pass"]["ms"], 3),
                    "ops_ms_per_step": {k: round(v["ms"] / steps, 4) for k, v in prof.items()
                                        if k != "pass" and v["ms"] > 0}})
    batch.close()
    return {"streams": streams, "steps_per_point": steps, "points": out}


def unfold_blocks(B, model, lens, streams: int = 1024, tokens: int = 256, timed_only: bool = False,
                  batch=None) -> dict:
    """configs[3] with the range decoder on the device: `streams` coded blocks of `tokens` tokens,
    unfolded from position 0 by one hs_batch_decode_blocks call (no host round trip per token).
    The payloads are seeded random bytes: the decoder turns any input into symbols, and the work of
    a step does not depend on the bytes. Timed by the wall clock around the C-ABI call, the better
    of two, with the device time from a third, profiled call; then the same rows driven step by
    step through run_coded with decode queries (one host round trip per step, the structure of the
    reference's GPU unfold loop). `timed_only`: one call on the given batch (made beforehand, so
    its allocation is outside the timing), its symbols and bytes, nothing else."""
    rng = np.random.default_rng(79)
    payloads = [rng.integers(0, 256, 4 * tokens, dtype=np.uint8).tobytes() for _ in range(streams)]
    sl = np.arange(streams, dtype=np.uint32)
    if timed_only:
        toks, status = batch.decode_blocks(sl, payloads, [tokens] * streams, 32)
        return {"streams": streams, "tokens_per_block": tokens, "tokens": streams * tokens,
                "bytes": int(lens[np.concatenate(toks).astype(np.int64)].sum())}
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
    nbytes = int(lens[np.concatenate(toks).astype(np.int64)].sum())
    return {"streams": streams, "tokens_per_block": tokens, "positions": f"0..{tokens - 1}",
            "e2e_tokens_per_s": n / wall, "device_tokens_per_s": n / (dev_ms / 1e3),
            "e2e_MB_per_s": nbytes / wall / 1e6,
            "host_loop_e2e_tokens_per_s": n / wall_host, "failed_blocks": int(status.sum()),
            "decoder_ms": round(prof.get("decoder", {"ms": 0.0})["ms"], 3)}


def unfold_cpu(model_bytes: bytes, eot: int, threads: int, steps: int = 24) -> dict:
    """The CPU unfold of the reference (crates/taco/src/unfold.rs:215-246): blocks decode in
    lockstep lanes of up to 8 per thread, every thread busy: 8 x threads streams decoded from
    position 0 for `steps` steps (one row per stream and step, a decode query with a seeded target
    each) by the CPU oracle's fast path with lanes, timed by the wall clock."""
    from oracle import oracle as O

    om = O.Model(model_bytes)
    streams = 8 * threads
    fb = O.FastBatch(om, streams, 0)
    rng = np.random.default_rng(80)
    sl = np.arange(streams, dtype=np.uint32)
    kinds = np.ones(streams, np.uint32)
    inp = np.full(streams, eot, np.uint32)
    t0 = time.perf_counter()
    for _ in range(steps):
        ans = fb.run_coded(sl, inp, kinds, rng.integers(0, 1 << 32, streams, dtype=np.uint64), 32, threads=threads,
                           lanes=True)
        inp = ans[:, 0].astype(np.uint32)
    dt = time.perf_counter() - t0
    return {"tokens_per_s": streams * steps / dt, "cores": threads, "kind": "port",
            "sample": f"{streams} streams (8 lanes per thread) x {steps} decode steps from position 0, {dt:.1f} s"}


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


def fold_glue(B, model, model_bytes, max_rows: int, mb: int = 2) -> dict:
    """The fold and the unfold of the profile text end to end through the host library (hs_fold,
    hs_unfold: tokenizer, zstd level 19, the coder op on the GPU, range encoder, container) on `mb`
    MiB of seeded Zipf text, default block size 16 KiB. Timed by the wall clock (the better of
    two); the device time of the fold's passes from a third, profiled call. A random-initialised
    model rarely beats zstd, so the encoders of most blocks stop before their last windows (which
    then never run) and the unfold mostly decodes zstd frames."""
    from taco_b200 import synth

    text = synth.zipf_text(mb << 20, seed=4242)[: mb << 20]
    tok = B.Tokenizer(model_bytes)
    batch = B.CudaBatch(model, 512, max_rows)
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
            "gpu_rows": stats["gpu_rows"], "coded_blocks": stats["coded_blocks"], "zstd_blocks": stats["zstd_blocks"],
            "container_bytes": stats["container_len"],
            "fold_e2e_MB_per_s": len(text) / wall / 1e6, "fold_device_ms": round(prof["pass"]["ms"], 3),
            "fold_wall_ms": round(wall * 1e3, 3), "fold_device_share": round(prof["pass"]["ms"] / (wall * 1e3), 3),
            "stages_ms": {k: round(stats[k], 1) for k in ("prep_ms", "gpu_ms", "finish_ms")},
            "unfold_e2e_MB_per_s": len(text) / uwall / 1e6}


def large_input(B, model_bytes: bytes, mb: int, ordinals: list[int], max_rows: int) -> dict:
    """`mb` MiB of the seeded mixed stream (70 % Zipf text, 20 % JSON key/number
    records, 10 % uniform random bytes, in 64 KiB pieces; synth.mixed_stream) folded by
    hs_fold_multi on the GPUs `ordinals` (two host threads each; 512 slots, passes of max_rows) and
    unfolded by hs_unfold_multi on the same GPUs (each worker opens its device and loads the model
    inside the timed call, as the fold's do); wall clock, the container's SHA-256, the stage times of the
    fold. The same bytes on every GPU count (tests/test_gpu_fold.py, tests/test_gpu_large_input.py
    check the equality with one GPU and with the CPU path on samples)."""
    import hashlib

    from taco_b200 import synth

    data = synth.mixed_stream(mb << 20)
    tok = B.Tokenizer(model_bytes)
    t0 = time.perf_counter()
    got, stats = B.fold_multi(ordinals, model_bytes, tok, data, slots=512, max_rows=max_rows)
    fold_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    back = B.unfold_multi(ordinals, model_bytes, tok, got, slots=256, max_rows=max_rows)
    unfold_s = time.perf_counter() - t0
    ok = back == data
    tok.close()
    if not ok:
        raise SystemExit("the large input did not unfold to itself")
    return {"input_MiB": mb, "gpus": len(ordinals), "blocks": stats["blocks"], "tokens": stats["tokens"],
            "gpu_rows": stats["gpu_rows"], "coded_blocks": stats["coded_blocks"], "zstd_blocks": stats["zstd_blocks"],
            "raw_blocks": stats["blocks"] - stats["coded_blocks"] - stats["zstd_blocks"],
            "container_bytes": stats["container_len"], "sha256": hashlib.sha256(got).hexdigest(),
            "fold_wall_s": round(fold_s, 3), "fold_MB_per_s": len(data) / fold_s / 1e6,
            "fold_stages_ms": {k: round(stats[k], 1) for k in ("prep_ms", "gpu_ms", "finish_ms")},
            "unfold_wall_s": round(unfold_s, 3), "unfold_MB_per_s": len(data) / unfold_s / 1e6,
            "gpus_failed": stats["gpus_failed"], "host_cores": os.cpu_count(),
            "workers_per_gpu": int(os.environ.get("HS_FOLD_WORKERS_PER_GPU", "2"))}


if __name__ == "__main__":
    sys.exit(main())
