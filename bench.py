# SPDX-License-Identifier: MIT
"""Benchmark of the fused decode on BASELINE configs[1]:
bf16 logits [B=64, T=128, K=8, V=32000] = N(0, 2) + Zipf(s=1.1) per-token bias, from_logits,
eos=2, length-penalty alpha=1.0 -- decoded through the engine's C ABI (dbs_cuda_decode_ex2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload c1|c2|c3|c4|c5|search]

One JSON line on rank 0. `value` is whole-job candidates/s (B*T*K*V per decode, all ranks)
with inputs resident in HBM; `e2e` is the same metric through the same C-ABI call with the
inputs in pinned host memory, copied in and the outputs copied out inside the timed region
(in chunks of examples, each chunk's copy overlapping the previous chunk's decode). Under
torchrun the config's 64 examples are split contiguously over the ranks (strong scaling, no
collective on the data path; the outputs stay sharded by example); `--scaling weak` gives every
rank a batch of its own instead. `--impl reference` times the reference's own CPU
implementation (libdbs, oracle/_ref/libdbs.so) with every host thread on the same config.

`--workload c1` / `--workload c3` time BASELINE configs[0] / configs[2] (decode only; the median
of per-decode CUDA events with L2 flushed between decodes).

`--workload c4` benchmarks BASELINE configs C4: bf16 log-probs [256,256,4,50257] with variable steps,
the decode plus the dense bf16 input gradient of a minimum-risk loss (dbs_cuda_backward_dense), per GPU
(weak scaling under torchrun).

`--workload c5` benchmarks BASELINE configs C5 instead: fp32 logits [16,32,64,256000] of the
same recipe, eos=1, alpha=0.6, the vocabulary lane-interleaved over the N ranks
(beamgrad_b200.vocab_sharding; strong scaling: N GPUs decode the same problem).
"""

from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

B, T, K, V = 64, 128, 8, 32000
EOS, ALPHA = 2, 1.0
METRIC = "beam candidates/s (B·T·K·V) and HBM GB/s vs roofline at 1/2/4/8 B200"


def workload() -> str:
    tag = "C2" if (B, T) == (64, 128) else "C2-shaped (reduced, profiling only)"
    return f"{tag}: bf16 logits [{B},{T},{K},{V}] N(0,2)+Zipf(1.1) bias, from_logits, eos={EOS}, alpha={ALPHA}"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own GPU engine (C2 at N=1)")
    ap.add_argument("--with-backward", action="store_true",
                    help="C2: also time the dense bf16 input gradient of the decode (a stage of its own)")
    ap.add_argument("--with-pool", type=int, default=0, metavar="M",
                    help="C2: also time the relaxed pool of the decode (P = K x M candidates per step and "
                         "their relaxed top-K weights, dbs_cuda_relaxed_pool)")
    ap.add_argument("--c5-path", default="sharded", choices=["sharded", "chained"],
                    help="C5 on one GPU: the vocabulary-shard stages (default) or the single-GPU chained decode")
    ap.add_argument("--batch", type=int, default=None,
                    help="C2: examples of the whole job (64); C4: examples per GPU (256); smaller only for profiling")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="C2 on N GPUs: strong = the config's batch split over the ranks (default); "
                         "weak = every rank decodes a batch of its own")
    ap.add_argument("--seq", type=int, default=128, help="decode steps T (C2: 128); smaller only for profiling")
    ap.add_argument("--workload", default="c2", choices=["c1", "c2", "c3", "c4", "c5", "search"])
    args = ap.parse_args()
    global B, T, C4, C5
    if args.workload == "c4" and args.batch is not None:
        C4 = (args.batch,) + C4[1:]
    if args.workload == "c5" and args.batch is not None:
        C5 = (args.batch,) + C5[1:]
    if args.workload in ("c1", "c3") and args.batch is not None:
        spec = SPECS[args.workload]
        spec.shape = (args.batch,) + spec.shape[1:]
        spec.name += "-shaped (reduced batch, profiling only)"
    if args.workload in ("c1", "c3", "c4", "c5", "search"):
        return args
    B, T = args.batch if args.batch is not None else 64, args.seq
    return args


def measured_traffic():
    """DRAM bytes (read + written) of one decode launch of this workload, from the committed
    one-pass ncu capture in profiles/; None for reduced (profiling) workloads."""
    if (B, T, K, V) != (64, 128, 8, 32000):
        return None
    path = Path(__file__).resolve().parent / "profiles" / "decode_chain_kernel.c2.traffic.json"
    try:
        d = json.loads(path.read_text())
    except (OSError, ValueError):
        return None
    return d["dram_bytes_read"] + d["dram_bytes_write"]


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# FP32 lane operations per logit entry of the bit-exact logsumexp, counted by ncu on the C2
# decode (profiles/decode_chain_kernel.c2_pipes.md): 11.0 packed FFMA2 instructions per entry
# (two lane operations each: the subtraction of the row maximum, the Cephes exp_nonpositive's
# range reduction and degree-5 polynomial, the lane add) and 1.0 scalar FADD (the
# round-toward-minus-infinity floor) -- 23 operations on the FMA pipes.
FP32_OPS_PER_ENTRY = 23


def fp32_roofline(entries: int, seconds: float, clocks: dict) -> dict:
    """The FP32-issue bound of a from-logits decode: entries x ops per entry against one FP32
    operation per lane per clock (148 SMs x 128 lanes) at the SM clock seen under load."""
    mhz = clocks.get("sm_mhz") or clocks.get("sm_max_mhz") or 1965.0
    peak = 148 * 128 * mhz * 1e6 / 1e12  # Tops/s
    achieved = entries * FP32_OPS_PER_ENTRY / seconds / 1e12
    return {"bound": "fp32_issue", "achieved": achieved, "peak": peak, "unit": "Tops/s", "frac": achieved / peak,
            "ops_per_entry": FP32_OPS_PER_ENTRY, "entries": entries, "sm_mhz": mhz}


class ClockSampler:
    """nvidia-smi samples of SM clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: str):
        self.index = index
        self.rows: list[tuple[float, list[str]]] = []
        self.proc = None
        self.window = (0.0, 0.0)
        self.extended = False

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "20"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            deadline = time.monotonic() + 5.0  # start timing only once samples flow
            while not self.rows and time.monotonic() < deadline:
                time.sleep(0.01)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.monotonic(), [c.strip() for c in line.split(",")]))

    def start(self):
        self.window = (time.monotonic(), float("inf"))

    def stop(self):
        self.window = (self.window[0], time.monotonic())

    def in_window(self) -> list[list[str]]:
        t0, t1 = self.window
        return [r for t, r in self.rows if t0 <= t <= t1]

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = self.in_window()
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if len(r) > 2 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) > 2 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in rows:
            for i, n in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower().startswith("active"):
                    reasons.add(n)
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
               "reasons": sorted(reasons), "samples": len(rows)}
        if self.extended:
            out["window"] = "timed region plus untimed decodes after it (the timed region was shorter than a sample)"
        return out


def make_inputs(torch, seed: int, device, examples=None):
    """Examples `examples` (default: all B) of the C2 input, bf16 [len(examples), T, K, V].

    Example b is drawn from its own seed, so a rank that holds examples [start, stop) of the
    batch gets the same bits as the whole-batch input has there, whatever the rank count."""
    examples = range(B) if examples is None else examples
    g = torch.Generator(device=device).manual_seed(seed)
    bias = -1.1 * torch.log(torch.randperm(V, generator=g, device=device).float() + 1.0)
    x = torch.empty((len(examples), T, K, V), dtype=torch.bfloat16, device=device)
    for i, b in enumerate(examples):  # one example at a time: keeps the float32 temporary small
        g.manual_seed(seed * 1009 + 1 + b)
        x[i] = (torch.randn((T, K, V), generator=g, device=device) * 2.0 + bias).to(torch.bfloat16)
    return x


def rows_read(tokens, parents, from_logprob, raw) -> int:
    """Rows the search read: 1 per example at t = 0, then the live, unfinished slots of step t-1."""
    live = (parents[:, :-1] >= 0) & (from_logprob[:, :-1] == 1) & (tokens[:, :-1] != EOS) & np.isfinite(raw[:, :-1])
    return int(tokens.shape[0] + live.sum())


def cpu_reference(x_host_bits: np.ndarray, threads: int, min_seconds: float = 10.0, max_reps: int = 5):
    """The reference CPU decoder (libdbs, every host thread) on the whole workload; seconds per decode."""
    from oracle import oracle
    from beamgrad_b200 import _abi as A

    pb = oracle.Problem(x_host_bits, dtype=A.DTYPE_BF16, from_logits=True, eos=EOS, alpha=ALPHA)
    times = []
    with oracle.RefDecoder(pb) as d:
        start = time.perf_counter()
        while len(times) < max_reps and (time.perf_counter() - start < min_seconds or len(times) < 1):
            t0 = time.perf_counter()
            d.decode(threads=threads)
            times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times)


def reference_gpu(torch, x, dtype: int, from_logits: bool, a, ours: dict, steps: int, dev, stream):
    """beamgrad 2.3.0's own GPU engine (cuda/dbs_cuda.cu built for sm_100a, oracle/_ref) on the
    same device-resident input and arguments `a` through the same C ABI call
    (dbs_cuda_decode_ex2): candidates/s from the median of per-decode CUDA events, and whether
    its outputs equal this engine's (`ours`, host copies of the decode outputs)."""
    from oracle import oracle
    from beamgrad_b200 import _abi as A

    if not oracle.ref_cuda_available():
        return {"unavailable": "oracle/_ref/libdbs_cuda_ref.so was not built"}
    lib = oracle.ref_cuda_lib()
    fields = {name for name, _ in A.DecodeOutputs._fields_}
    ours = {k: v for k, v in ours.items() if k in fields}
    out = {k: torch.empty(v.shape, dtype=torch.from_numpy(v).dtype, device=dev) for k, v in ours.items()}
    o = A.DecodeOutputs()
    for k, v in out.items():
        setattr(o, k, v.data_ptr())
    nb = lib.dbs_cuda_decode_workspace_size(C.byref(a))
    ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)

    def decode():
        A.check(lib.dbs_cuda_decode_ex2(C.c_void_p(x.data_ptr()), dtype, int(from_logits), C.byref(a), None,
                                        C.byref(o), None, C.c_void_p(ws.data_ptr()), nb,
                                        C.c_void_p(stream.cuda_stream)), "reference decode")

    decode()
    torch.cuda.synchronize(dev)
    same = all(out[k].cpu().numpy().tobytes() == ours[k].tobytes() for k in ours)
    times = []
    for _ in range(max(3, min(steps, 10))):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        decode()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        times.append(e0.elapsed_time(e1) / 1e3)
    sec = statistics.median(times)
    cand = a.batch_size * a.steps * a.beam_size * a.vocab_size
    return {"value": cand / sec, "unit": "candidates/s", "ms_per_step": sec * 1e3,
            "kind": "beamgrad 2.3.0 cuda/dbs_cuda.cu, unmodified, built for sm_100a (oracle/Makefile)",
            "matches_this_engine": same, "decodes_timed": len(times)}


def run_reference_arm(args, rank: int, world: int):
    if rank != 0:
        return
    import torch
    from oracle import oracle

    if not oracle.ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libdbs.so was not built"}))
        return
    threads = oracle.cpu_count()
    x = make_inputs(torch, 1000, "cuda" if torch.cuda.is_available() else "cpu")
    bits = x.view(torch.int16).cpu().numpy().view(np.uint16)
    del x
    per_step = []
    for i in range(args.warmup + args.steps):
        sec, _ = cpu_reference(bits, threads, min_seconds=0.0, max_reps=1)
        if i >= args.warmup:
            per_step.append(sec)
    sec = statistics.median(per_step)
    cand = B * T * K * V
    value = cand / sec
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "candidates/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": workload(), "global_batch": B, "seq_len": T, "beam": K, "vocab": V,
                   "parallelism": "host threads"},
        "cpu_baseline": {"value": value, "unit": "candidates/s", "cores": threads, "kind": "reference",
                         "sample": f"full workload ({B} examples) per step, libdbs dbs_decode_batch_into_ex"},
        "e2e": {"value": value, "unit": "candidates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------- C4
C4 = (256, 256, 4, 50257)
C4_EOS, C4_ALPHA = 50256, 0.0


def c4_workload() -> str:
    B4, T4, K4, V4 = C4
    tag = "C4" if B4 == 256 else "C4-shaped (reduced batch, profiling only)"
    return (f"{tag}: bf16 log-probs [{B4},{T4},{K4},{V4}] = log_softmax(N(0,2)+Zipf(1.1) bias), steps per example "
            f"U{{16..{T4}}}, eos={C4_EOS}, alpha={C4_ALPHA}; decode + dense input gradient (bf16) of the mean "
            f"minimum-risk loss, costs U[0,1]")


def c4_inputs(torch, seed: int, device, n: int | None = None):
    """The first n examples (all by default) of the C4 input: bf16 [n, T, K, V], steps [n] int32,
    costs [n, K] float32."""
    B4, T4, K4, V4 = C4
    n = B4 if n is None else n
    g = torch.Generator(device=device).manual_seed(seed)
    bias = -1.1 * torch.log(torch.randperm(V4, generator=g, device=device).float() + 1.0)
    steps = torch.randint(16, T4 + 1, (B4,), generator=g, device=device, dtype=torch.int32)[:n].contiguous()
    costs = torch.rand((B4, K4), generator=g, device=device)[:n].contiguous()
    x = torch.empty((n, T4, K4, V4), dtype=torch.bfloat16, device=device)
    for b in range(n):
        x[b] = torch.log_softmax(torch.randn((T4, K4, V4), generator=g, device=device) * 2.0 + bias, -1).to(x.dtype)
    return x, steps, costs


def minimum_risk_grad(torch, final_scores, costs):
    """d/d final_scores of mean_b sum_k softmax(final_scores[b])_k * costs[b, k] over live beams
    (python/beamgrad/losses.py:139-169 of beamgrad 2.3.0, temperature 1), and the loss."""
    live = torch.isfinite(final_scores)
    any_live = live.any(-1, keepdim=True)
    logits = torch.where(live, final_scores, float("-inf"))
    logits = torch.where(any_live, logits, torch.zeros_like(logits))
    p = torch.softmax(logits, -1)
    c = torch.where(live, costs, 0.0)
    expected = (p * c).sum(-1, keepdim=True)
    B = final_scores.shape[0]
    g = torch.where(any_live, p * (c - expected) / B, 0.0)
    return g.contiguous(), (expected[:, 0] * any_live[:, 0]).mean()


def c4_cpu_reference(torch, threads: int, n_examples: int = 8):
    """The reference CPU library (libdbs: dbs_decode_batch_into_ex, then dbs_backward_batch_into_ex into a
    zeroed float32 gradient) on the first n_examples of C4; candidates/s and the sample."""
    from oracle import oracle
    from beamgrad_b200 import _abi as A

    B4, T4, K4, V4 = C4
    x, steps, costs = c4_inputs(torch, 4000, "cuda" if torch.cuda.is_available() else "cpu", n_examples)
    bits = x.view(torch.int16).cpu().numpy().view(np.uint16)
    steps_h = steps.cpu().numpy()
    costs_t = costs.cpu()
    del x
    pb = oracle.Problem(bits, dtype=A.DTYPE_BF16, from_logits=False, eos=C4_EOS, alpha=C4_ALPHA, steps=steps_h)
    times = []
    with oracle.RefDecoder(pb) as d:
        for _ in range(3):
            t0 = time.perf_counter()
            trace = d.decode(threads=threads)
            g, _ = minimum_risk_grad(torch, torch.from_numpy(trace["final_scores"]), costs_t)
            d.backward(trace, {"final_scores": g.numpy()}, threads=threads)
            times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    return (n_examples * T4 * K4 * V4 / sec,
            f"{n_examples} of the {B4} examples of C4 (decode + dense float32 backward), median of 3 runs")


def write_ceiling(torch, buf, stream, reps: int = 5) -> float | None:
    """GB/s of cudaMemsetAsync over `buf` on this GPU: the speed of a pure write stream, which
    the copy-based HBM peak understates (a copy also reads)."""
    try:
        cudart = C.CDLL("libcudart.so.12")  # the runtime the engine library already loaded
    except OSError:
        return None
    nbytes = buf.numel() * buf.element_size()
    fn = cudart.cudaMemsetAsync
    fn.argtypes = [C.c_void_p, C.c_int, C.c_size_t, C.c_void_p]
    fn.restype = C.c_int
    sp = C.c_void_p(stream.cuda_stream)
    for _ in range(2):
        if fn(C.c_void_p(buf.data_ptr()), 0, nbytes, sp) != 0:
            return None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        fn(C.c_void_p(buf.data_ptr()), 0, nbytes, sp)
    e1.record(stream)
    e1.synchronize()
    return nbytes * reps / (e0.elapsed_time(e1) / 1e3) / 1e9


def run_c4(args, rank: int, world: int, local: int):
    import torch

    from oracle import oracle

    B4, T4, K4, V4 = C4
    cand = B4 * T4 * K4 * V4
    if args.impl == "reference":
        if rank != 0:
            return
        if not oracle.ref_available():
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libdbs.so was not built"}))
            return
        threads = oracle.cpu_count()
        per = []
        for i in range(args.warmup + args.steps):
            value, sample = c4_cpu_reference(torch, threads, n_examples=2)
            if i >= args.warmup:
                per.append(value)
        value = statistics.median(per)
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": value, "unit": "candidates/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": cand / value * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": c4_workload(), "global_batch": B4, "seq_len": T4, "beam": K4, "vocab": V4,
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": "candidates/s", "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": value, "unit": "candidates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return

    from beamgrad_b200 import _abi as A

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    lib = A.load()
    dev = torch.device("cuda", local)
    x, steps, costs = c4_inputs(torch, 4000 + rank, dev)
    f32, i32, u8 = torch.float32, torch.int32, torch.uint8
    out = {
        "final_scores": torch.empty((B4, K4), dtype=f32, device=dev),
        "final_raw_scores": torch.empty((B4, K4), dtype=f32, device=dev),
        "final_lengths": torch.empty((B4, K4), dtype=i32, device=dev),
        "tokens": torch.empty((B4, T4, K4), dtype=i32, device=dev),
        "parents": torch.empty((B4, T4, K4), dtype=i32, device=dev),
        "lengths": torch.empty((B4, T4, K4), dtype=i32, device=dev),
        "scores": torch.empty((B4, T4, K4), dtype=f32, device=dev),
        "raw_scores": torch.empty((B4, T4, K4), dtype=f32, device=dev),
        "from_logprob": torch.empty((B4, T4, K4), dtype=u8, device=dev),
        "invalid_input": torch.empty((B4,), dtype=u8, device=dev),
    }
    o = A.DecodeOutputs()
    for k, v in out.items():
        setattr(o, k, v.data_ptr())
    a = A.DecodeArgs()
    a.batch_size, a.steps, a.beam_size, a.vocab_size = B4, T4, K4, V4
    a.eos_token, a.length_penalty_alpha, a.repetition_penalty = C4_EOS, C4_ALPHA, 1.0
    a.steps_per_example = steps.data_ptr()
    ws_bytes = max(lib.dbs_cuda_decode_workspace_size(C.byref(a)), lib.dbs_cuda_backward_workspace_size(C.byref(a)))
    ws = torch.empty(ws_bytes, dtype=u8, device=dev)
    grad = torch.empty((B4, T4, K4, V4), dtype=torch.bfloat16, device=dev)
    bi = A.BackwardInputs()
    bi.parents, bi.tokens = out["parents"].data_ptr(), out["tokens"].data_ptr()
    bi.lengths, bi.from_logprob = out["lengths"].data_ptr(), out["from_logprob"].data_ptr()
    stream = torch.cuda.current_stream(dev)
    sp = C.c_void_p(stream.cuda_stream)
    loss_h = torch.empty((), dtype=f32, pin_memory=True)

    def step(inp, ev=None):
        if ev:
            ev[0].record(stream)
        A.check(lib.dbs_cuda_decode_ex2(C.c_void_p(inp.data_ptr()), A.DTYPE_BF16, 0, C.byref(a), None, C.byref(o),
                                        None, C.c_void_p(ws.data_ptr()), ws_bytes, sp), "decode")
        g, loss = minimum_risk_grad(torch, out["final_scores"], costs)
        bi.grad_final_scores = g.data_ptr()
        if ev:
            ev[1].record(stream)
        A.check(lib.dbs_cuda_backward_dense(C.byref(a), C.byref(bi), C.c_void_p(grad.data_ptr()), A.DTYPE_BF16,
                                            C.c_void_p(ws.data_ptr()), ws_bytes, sp), "backward")
        if ev:
            ev[2].record(stream)
        return g, loss

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        step(x)
    barrier()
    try:
        gpu_id = f"GPU-{torch.cuda.get_device_properties(dev).uuid}"
    except (AttributeError, RuntimeError):
        gpu_id = str(local)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    evs = []
    with ClockSampler(gpu_id) as clocks:
        barrier()
        clocks.start()
        start.record(stream)
        for _ in range(args.steps):
            ev = tuple(torch.cuda.Event(enable_timing=True) for _ in range(3))
            step(x, ev)
            evs.append(ev)
        stop.record(stream)
        barrier()
        clocks.stop()
        if clocks.proc is not None and not clocks.in_window():
            clocks.extended = True
            deadline = time.monotonic() + 2.0
            while not clocks.in_window() and time.monotonic() < deadline:
                step(x)
                torch.cuda.synchronize(dev)
                clocks.stop()
    elapsed = start.elapsed_time(stop) / 1e3
    t_all = torch.tensor([elapsed], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t_all, op=dist.ReduceOp.MAX)
    elapsed = float(t_all.item())
    fwd_s = statistics.mean(e[0].elapsed_time(e[1]) for e in evs) / 1e3
    bwd_s = statistics.mean(e[1].elapsed_time(e[2]) for e in evs) / 1e3

    write_gbs = write_ceiling(torch, grad, stream)

    host = {k: v.cpu().numpy() for k, v in out.items()}
    ref_gpu = None
    if world == 1 and not args.no_reference_gpu:
        # The reference engine's decode of the same input (its backward is not timed here).
        ref_gpu = reference_gpu(torch, x, A.DTYPE_BF16, False, a, host, args.steps, dev, stream)
    live = ((host["parents"][:, :-1] >= 0) & (host["from_logprob"][:, :-1] == 1) &
            (host["tokens"][:, :-1] != C4_EOS) & np.isfinite(host["raw_scores"][:, :-1]))
    n_rows = int(B4 + live.sum())
    slots = B4 * T4 * K4
    fwd_bytes = n_rows * V4 * 2 + slots * (4 * 5 + 1) + B4 * K4 * 12
    bwd_bytes = slots * V4 * 2 + slots * (4 * 4 + 1)  # gradient written once; trace + draws read
    peak, peak_kind = peaks()
    fwd_gbs, bwd_gbs = fwd_bytes / fwd_s / 1e9, bwd_bytes / bwd_s / 1e9
    dominant = ("dbs_cuda_backward_dense (gradient memset + backward_kernel + scatter_dense_kernel)", bwd_bytes,
                bwd_gbs) \
        if bwd_s >= fwd_s else ("dbs_cuda_decode_ex2 (decode_chain_warp_kernel)", fwd_bytes, fwd_gbs)

    # End to end: the input from pinned host memory, the decode + backward, the loss back to the host
    # (the gradient stays on the device, where the model's backward consumes it).
    e2e = None
    if not args.no_e2e:
        xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        xh.copy_(x)
        xd = torch.empty_like(x)
        n_e2e = max(2, min(args.steps, 3))

        def e2e_step():
            xd.copy_(xh, non_blocking=True)
            _, loss = step(xd)
            loss_h.copy_(loss, non_blocking=True)

        e2e_step()
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        s1.record(stream)
        barrier()
        e2e_t = torch.tensor([s0.elapsed_time(s1) / 1e3 / n_e2e], device=dev, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
        e2e = {"value": world * cand / float(e2e_t.item()), "unit": "candidates/s",
               "h2d_bytes_per_step": xh.numel() * xh.element_size(), "d2h_bytes_per_step": 4}
        del xh, xd

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and oracle.ref_available():
        threads = oracle.cpu_count()
        value, sample = c4_cpu_reference(torch, threads)
        cpu = {"value": value, "unit": "candidates/s", "cores": threads, "kind": "reference", "sample": sample}

    if dist is not None:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": world * cand / elapsed * args.steps,
            "unit": "candidates/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": elapsed / args.steps * 1e3,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": c4_workload(), "global_batch": world * B4, "seq_len": T4, "beam": K4,
                       "vocab": V4, "parallelism": f"batch x{world}" if world > 1 else "single GPU",
                       "candidates": "nominal B*T_max*K*V per step",
                       "l2": f"inputs ({x.numel() * 2 / 1e9:.1f} GB per GPU) larger than L2 (126 MB)",
                       "stage_ms": {"decode_and_loss": round(fwd_s * 1e3, 4), "backward_dense": round(bwd_s * 1e3, 4)},
                       "rows_read": n_rows},
            "roofline": {"bound": "hbm", "achieved": dominant[2], "peak": peak, "unit": "GB/s",
                         "frac": dominant[2] / peak, "traffic": None, "peak_kind": peak_kind, "kernel": dominant[0],
                         "alg_bytes_per_launch": dominant[1]},
            "roofline_stages": {"decode": {"achieved": fwd_gbs, "frac": fwd_gbs / peak, "alg_bytes": fwd_bytes},
                                "backward_dense": {"achieved": bwd_gbs, "frac": bwd_gbs / peak,
                                                   "write_stream_gbs": write_gbs,
                                                   "frac_of_write_stream": bwd_gbs / write_gbs if write_gbs else None,
                                                   "alg_bytes": bwd_bytes}},
            "cpu_baseline": cpu,
            "reference_gpu": ref_gpu,
            "e2e": e2e,
            "gpu_launches": args.steps * 4,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------- C1, C3
class Spec:
    """A decode-only BASELINE config: shape, dtype, inputs and search options."""

    def __init__(self, name, shape, dtype, from_logits, eos, alpha, min_length=0, banned_frac=0.0, rep=1.0, ngram=0,
                 sample=1):
        self.name, self.shape, self.dtype, self.from_logits = name, shape, dtype, from_logits
        self.eos, self.alpha, self.min_length = eos, alpha, min_length
        self.banned_frac, self.rep, self.ngram, self.sample = banned_frac, rep, ngram, sample

    def workload(self) -> str:
        B_, T_, K_, V_ = self.shape
        kind = "logits" if self.from_logits else "log-probs"
        extra = ""
        if self.banned_frac:
            extra += f", banned {self.banned_frac:.0%} of V, repetition penalty {self.rep}, no_repeat_ngram {self.ngram}"
        return (f"{self.name}: {self.dtype} {kind} [{B_},{T_},{K_},{V_}], eos={self.eos}, alpha={self.alpha}, "
                f"min_length={self.min_length}{extra}")


SPECS = {
    # fp32 log_softmax(3*N(0,1)) [8,32,4,1000], eos=2, alpha=0.6, min_length=4.
    "c1": Spec("C1", (8, 32, 4, 1000), "f32", False, 2, 0.6, min_length=4, sample=8),
    # fp16 logits N(0,2)+Zipf(1.1) [32,64,8,151936], banned 1%, rep 1.2, 3-gram, EOS suppressed.
    "c3": Spec("C3", (32, 64, 8, 151936), "f16", True, -1, 0.0, banned_frac=0.01, rep=1.2, ngram=3, sample=2),
}


def spec_inputs(torch, spec: Spec, seed: int, device, n: int | None = None):
    """The first n examples (all by default) of the config's input, and its banned-token mask."""
    B_, T_, K_, V_ = spec.shape
    n = B_ if n is None else n
    g = torch.Generator(device=device).manual_seed(seed)
    if spec.name == "C1":
        x = torch.log_softmax(3.0 * torch.randn((B_, T_, K_, V_), generator=g, device=device), -1)[:n].contiguous()
        return x, None
    bias = -1.1 * torch.log(torch.randperm(V_, generator=g, device=device).float() + 1.0)
    banned = torch.zeros(V_, dtype=torch.uint8, device=device)
    banned[torch.randperm(V_, generator=g, device=device)[: int(spec.banned_frac * V_)]] = 1
    x = torch.empty((n, T_, K_, V_), dtype=torch.float16, device=device)
    for b in range(n):
        x[b] = (torch.randn((T_, K_, V_), generator=g, device=device) * 2.0 + bias).half()
    return x, banned


def spec_cpu_reference(torch, spec: Spec, threads: int):
    """The reference CPU library on the first spec.sample examples; candidates/s and the sample."""
    from oracle import oracle
    from beamgrad_b200 import _abi as A

    B_, T_, K_, V_ = spec.shape
    x, banned = spec_inputs(torch, spec, 100, "cuda" if torch.cuda.is_available() else "cpu", spec.sample)
    xh = x.cpu().numpy() if spec.dtype == "f32" else x.view(torch.int16).cpu().numpy().view(np.uint16)
    dt = A.DTYPE_F32 if spec.dtype == "f32" else A.DTYPE_F16
    pb = oracle.Problem(xh, dtype=dt, from_logits=spec.from_logits, eos=spec.eos, alpha=spec.alpha,
                        min_length=spec.min_length, ngram=spec.ngram, rep_penalty=spec.rep,
                        banned=None if banned is None else banned.cpu().numpy())
    times = []
    with oracle.RefDecoder(pb) as d:
        for _ in range(3):
            t0 = time.perf_counter()
            d.decode(threads=threads)
            times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    return spec.sample * T_ * K_ * V_ / sec, f"{spec.sample} of the {B_} examples, median of 3 runs of libdbs"


def run_decode_only(args, rank: int, world: int, local: int, spec: Spec):
    """A decode-only config through dbs_cuda_decode_ex2, per GPU (weak scaling under torchrun)."""
    import torch

    from oracle import oracle

    B_, T_, K_, V_ = spec.shape
    cand = B_ * T_ * K_ * V_
    if args.impl == "reference":
        if rank != 0:
            return
        if not oracle.ref_available():
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libdbs.so was not built"}))
            return
        threads = oracle.cpu_count()
        per = [spec_cpu_reference(torch, spec, threads) for _ in range(args.warmup + args.steps)][args.warmup:]
        value = statistics.median(v for v, _ in per)
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": value, "unit": "candidates/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": cand / value * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": spec.dtype, "data": "synthetic",
            "config": {"workload": spec.workload(), "global_batch": B_, "seq_len": T_, "beam": K_, "vocab": V_,
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": "candidates/s", "cores": threads, "kind": "reference",
                             "sample": per[0][1]},
            "e2e": {"value": value, "unit": "candidates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return

    from beamgrad_b200 import _abi as A

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    lib = A.load()
    dev = torch.device("cuda", local)
    x, banned = spec_inputs(torch, spec, 100 + rank, dev)
    f32, i32, u8 = torch.float32, torch.int32, torch.uint8
    out = {n: torch.empty(sh, dtype=dt, device=dev) for n, sh, dt in (
        ("final_scores", (B_, K_), f32), ("final_raw_scores", (B_, K_), f32), ("final_lengths", (B_, K_), i32),
        ("tokens", (B_, T_, K_), i32), ("parents", (B_, T_, K_), i32), ("lengths", (B_, T_, K_), i32),
        ("scores", (B_, T_, K_), f32), ("raw_scores", (B_, T_, K_), f32), ("from_logprob", (B_, T_, K_), u8),
        ("invalid_input", (B_,), u8))}
    o = A.DecodeOutputs()
    for k, v in out.items():
        setattr(o, k, v.data_ptr())
    a = A.DecodeArgs()
    a.batch_size, a.steps, a.beam_size, a.vocab_size = B_, T_, K_, V_
    a.eos_token, a.length_penalty_alpha, a.min_length = spec.eos, spec.alpha, spec.min_length
    a.repetition_penalty, a.no_repeat_ngram_size = spec.rep, spec.ngram
    if banned is not None:
        a.banned_tokens = banned.data_ptr()
    dt = A.DTYPE_F32 if spec.dtype == "f32" else A.DTYPE_F16
    row_lse = torch.empty((B_, T_, K_), dtype=f32, device=dev)
    ws_bytes = lib.dbs_cuda_decode_workspace_size(C.byref(a))
    ws = torch.empty(ws_bytes, dtype=u8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = C.c_void_p(stream.cuda_stream)

    def decode(inp):
        A.check(lib.dbs_cuda_decode_ex2(C.c_void_p(inp.data_ptr()), dt, int(spec.from_logits), C.byref(a), None,
                                        C.byref(o), C.c_void_p(row_lse.data_ptr()), C.c_void_p(ws.data_ptr()),
                                        ws_bytes, sp), "decode")

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        decode(x)
    barrier()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 256 MB > L2: flushed between decodes
    try:
        gpu_id = f"GPU-{torch.cuda.get_device_properties(dev).uuid}"
    except (AttributeError, RuntimeError):
        gpu_id = str(local)
    evs = []
    with ClockSampler(gpu_id) as clocks:
        barrier()
        clocks.start()
        deadline = time.monotonic() + 0.5
        while True:  # at least `steps` decodes and half a second, so the clock sampler sees the load
            for _ in range(args.steps):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                decode(x)
                e1.record(stream)
                evs.append((e0, e1))
            barrier()
            if time.monotonic() > deadline:
                break
        clocks.stop()
    per = statistics.median(e0.elapsed_time(e1) for e0, e1 in evs) / 1e3
    t_all = torch.tensor([per], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t_all, op=dist.ReduceOp.MAX)
    per = float(t_all.item())
    host = {k: v.cpu().numpy() for k, v in out.items()}
    live = ((host["parents"][:, :-1] >= 0) & (host["from_logprob"][:, :-1] == 1) &
            (host["tokens"][:, :-1] != spec.eos) & np.isfinite(host["raw_scores"][:, :-1]))
    n_rows = int(B_ + live.sum())
    elem = 4 if spec.dtype == "f32" else 2
    alg_bytes = n_rows * V_ * elem + B_ * T_ * K_ * 21 + B_ * K_ * 12
    peak, peak_kind = peaks()
    achieved = alg_bytes / per / 1e9

    e2e = None
    if not args.no_e2e:
        xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        xh.copy_(x)
        xd = torch.empty_like(x)
        outs_h = {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in out.items()}
        n_e2e = max(2, min(args.steps, 5))

        def e2e_step():
            xd.copy_(xh, non_blocking=True)
            decode(xd)
            for k, v in out.items():
                outs_h[k].copy_(v, non_blocking=True)

        e2e_step()
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        s1.record(stream)
        barrier()
        e2e_t = torch.tensor([s0.elapsed_time(s1) / 1e3 / n_e2e], device=dev, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
        e2e = {"value": world * cand / float(e2e_t.item()), "unit": "candidates/s",
               "h2d_bytes_per_step": xh.numel() * xh.element_size(),
               "d2h_bytes_per_step": sum(v.numel() * v.element_size() for v in outs_h.values())}

    ref_gpu = None
    if world == 1 and not args.no_reference_gpu:
        ref_gpu = reference_gpu(torch, x, dt, spec.from_logits, a, host, args.steps, dev, stream)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and oracle.ref_available():
        threads = oracle.cpu_count()
        value, sample = spec_cpu_reference(torch, spec, threads)
        cpu = {"value": value, "unit": "candidates/s", "cores": threads, "kind": "reference", "sample": sample}
    if dist is not None:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": world * cand / per, "unit": "candidates/s", "n_gpus": world,
            "steps": len(evs), "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": spec.dtype, "data": "synthetic",
            "config": {"workload": spec.workload(), "global_batch": world * B_, "seq_len": T_, "beam": K_,
                       "vocab": V_, "parallelism": f"batch x{world}" if world > 1 else "single GPU",
                       "l2": "256 MB buffer written between timed decodes (L2 flushed)",
                       "timing": "median of per-decode CUDA events", "rows_read": n_rows},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "peak_kind": peak_kind, "alg_bytes_per_launch": alg_bytes},
            "cpu_baseline": cpu,
            "reference_gpu": ref_gpu,
            "e2e": e2e,
            "gpu_launches": 2 * len(evs),
            "clocks": clocks.summary(),
        }
        if spec.from_logits:
            line["roofline_fp32"] = fp32_roofline(n_rows * V_, per, clocks.summary())
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


# ---------------------------------------------------------------------------- search loop
def run_search(args, rank: int, world: int, local: int):
    """beamgrad's step-by-step search loop (python/beamgrad/_search.py:330-467) on C2's shape
    with bf16 log-prob rows fed one step at a time: the loop as beamgrad writes it over
    torch.ops.beamgrad.decode_step (per step: float32 copy of the rows, state clones, the
    validation read-back and the active.any() check, sequences by gather + cat), against
    beamgrad_b200.search.DeviceSearch eager (live flag read every step, as beamgrad stops) and
    the same search captured in one CUDA graph. Each step's "model" is a copy of that step's
    rows into a fixed buffer. Per GPU; rank 0 prints."""
    import torch

    from beamgrad_b200 import ops
    from beamgrad_b200 import search as S

    Bs, Ts, Ks, Vs = 64, 128, 8, 32000
    cand = Bs * Ts * Ks * Vs
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the search loop workload has no CPU arm: "
                              "beamgrad's loop is the 'loop_reference_style' figure of our line"}))
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    ops.load()
    g = torch.Generator(device=dev).manual_seed(7000 + rank)
    bias = -1.1 * torch.log(torch.randperm(Vs, generator=g, device=dev).float() + 1.0)
    x = torch.empty((Ts, Bs, Ks, Vs), dtype=torch.bfloat16, device=dev)  # step-major: each step contiguous
    for t in range(Ts):
        x[t] = torch.log_softmax(torch.randn((Bs, Ks, Vs), generator=g, device=dev) * 2.0 + bias, -1).to(x.dtype)
    rows = torch.empty((Bs, Ks, Vs), dtype=torch.bfloat16, device=dev)
    eos, alpha = 2, 1.0
    stream = torch.cuda.current_stream(dev)

    def reference_loop():
        raw = torch.full((Bs, Ks), float("-inf"), device=dev)
        raw[:, 0] = 0.0
        lengths = torch.zeros((Bs, Ks), dtype=torch.int32, device=dev)
        finished = torch.zeros((Bs, Ks), dtype=torch.uint8, device=dev)
        sequences = torch.empty((Bs, Ks, 0), dtype=torch.int64, device=dev)
        for t in range(Ts):
            active = torch.isfinite(raw) & (finished == 0)
            if t > 0 and not bool(active.any()):
                break
            rows.copy_(x[t])
            tok, par, lengths, scores, raw, flp, finished, final = torch.ops.beamgrad.decode_step(
                rows.to(torch.float32).contiguous(), raw, lengths, finished, sequences.to(torch.int32), eos, 0, alpha,
                None, 0, 1.0, True, [])
            parents, tokens = par.long(), tok.long()
            source = parents.clamp(min=0)[..., None].expand(Bs, Ks, t)
            emitted = torch.where(flp.bool(), tokens, -1)
            sequences = torch.cat([sequences.gather(1, source), emitted[..., None]], dim=2)
            sequences = torch.where((parents >= 0)[..., None], sequences, -1)
        return sequences

    search = S.DeviceSearch(Bs, Ks, Vs, Ts, dtype=torch.bfloat16, eos_token=eos, length_penalty_alpha=alpha,
                            device=dev)

    def device_loop(check_every: int):
        search.reset()
        for t in range(Ts):
            if t > 0 and t % check_every == 0 and not search.live_after(t - 1):
                break
            rows.copy_(x[t])
            search.step(rows)

    def graph_body():
        search.reset()
        for t in range(Ts):
            rows.copy_(x[t])
            search.step(rows)

    def timed(fn, reps):
        fn()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / 1e3 / reps

    reps = max(1, args.steps)
    for _ in range(max(0, args.warmup - 1)):
        device_loop(1)
    try:
        gpu_id = f"GPU-{torch.cuda.get_device_properties(dev).uuid}"
    except (AttributeError, RuntimeError):
        gpu_id = str(local)
    with ClockSampler(gpu_id) as clocks:
        clocks.start()
        t_ref = timed(reference_loop, reps)
        t_dev1 = timed(lambda: device_loop(1), reps)
        t_devT = timed(lambda: device_loop(Ts), reps)
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            graph_body()
        stream.wait_stream(side)
        torch.cuda.synchronize(dev)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            graph_body()
        t_graph = timed(graph.replay, reps)
        clocks.stop()
    steps_run = int(search.result().trace.steps[0])
    same = torch.equal(search.result().sequences[..., :steps_run], reference_loop()[..., :steps_run].long())
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": cand / t_dev1, "unit": "candidates/s", "n_gpus": world, "steps": reps,
            "warmup": args.warmup, "ms_per_step": t_dev1 * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"search loop: bf16 log-prob rows [{Bs},{Ks},{Vs}] per step, {Ts} steps "
                                   f"(C2's shape, log_softmax(N(0,2)+Zipf(1.1))), eos={eos}, alpha={alpha}",
                       "global_batch": Bs, "seq_len": Ts, "beam": Ks, "vocab": Vs, "steps_run": steps_run,
                       "step": "one whole search (Ts model steps: a 32.8 MB row copy + one search step)"},
            "loops_ms": {"loop_reference_style": t_ref * 1e3, "device_search_check_every_step": t_dev1 * 1e3,
                         "device_search_no_host_sync": t_devT * 1e3, "device_search_cuda_graph": t_graph * 1e3},
            "speedup_vs_reference_style": t_ref / t_dev1,
            "sequences_match_reference_style": bool(same),
            "roofline": None, "cpu_baseline": None, "e2e": None,
            "gpu_launches": None, "clocks": clocks.summary(),
        }), flush=True)


# ---------------------------------------------------------------------------- C5
C5 = (16, 32, 64, 256000)
C5_EOS, C5_ALPHA = 1, 0.6


def c5_workload() -> str:
    B5, T5, K5, V5 = C5
    tag = "C5" if B5 == 16 else "C5-shaped (reduced batch, profiling only)"
    return (f"{tag}: fp32 logits [{B5},{T5},{K5},{V5}] N(0,2)+Zipf(1.1) bias, from_logits, eos={C5_EOS}, "
            f"alpha={C5_ALPHA}, vocabulary lane-interleaved over the ranks")


def c5_example(torch, device, b: int):
    """Example b of the C5 input, full vocabulary [T, K, V] float32 (the same on every rank)."""
    B5, T5, K5, V5 = C5
    g = torch.Generator(device=device).manual_seed(5000)
    bias = -1.1 * torch.log(torch.randperm(V5, generator=g, device=device).float() + 1.0)
    g.manual_seed(5001 + b)
    return torch.randn((T5, K5, V5), generator=g, device=device) * 2.0 + bias


def c5_shard(torch, world: int, rank: int, device):
    from beamgrad_b200 import vocab_sharding as vs

    B5, T5, K5, V5 = C5
    cols = vs.shard_tokens(V5, world, rank, device)
    x = torch.empty((B5, T5, K5, cols.numel()), dtype=torch.float32, device=device)
    for b in range(B5):
        x[b] = c5_example(torch, device, b).index_select(-1, cols)
    return x


def c5_cpu_reference(torch, device, threads: int, n_examples: int = 1):
    """The reference CPU decoder on the first n_examples of C5 (full vocabulary); candidates/s."""
    from oracle import oracle
    from beamgrad_b200 import _abi as A

    B5, T5, K5, V5 = C5
    x = np.stack([c5_example(torch, device, b).cpu().numpy() for b in range(n_examples)])
    pb = oracle.Problem(x, dtype=A.DTYPE_F32, from_logits=True, eos=C5_EOS, alpha=C5_ALPHA)
    times = []
    with oracle.RefDecoder(pb) as d:
        for _ in range(3):
            t0 = time.perf_counter()
            d.decode(threads=threads)
            times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    return n_examples * T5 * K5 * V5 / sec, f"{n_examples} example(s) of C5 (full vocabulary), median of 3 runs"


def run_c5_chained(args, world: int, local: int):
    """C5 on one GPU through dbs_cuda_decode_ex2 (the chained decode for beams above 16,
    decode_chain_wide_kernel): median of per-decode CUDA events."""
    import torch

    from beamgrad_b200 import _abi as A

    if world != 1:
        raise SystemExit("--c5-path chained runs on one GPU")
    B5, T5, K5, V5 = C5
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lib = A.load()
    x = c5_shard(torch, 1, 0, dev)  # one shard: the whole vocabulary in token order
    f32, i32, u8 = torch.float32, torch.int32, torch.uint8
    out = {n: torch.empty(sh, dtype=dt, device=dev) for n, sh, dt in (
        ("final_scores", (B5, K5), f32), ("final_raw_scores", (B5, K5), f32), ("final_lengths", (B5, K5), i32),
        ("tokens", (B5, T5, K5), i32), ("parents", (B5, T5, K5), i32), ("lengths", (B5, T5, K5), i32),
        ("scores", (B5, T5, K5), f32), ("raw_scores", (B5, T5, K5), f32), ("from_logprob", (B5, T5, K5), u8),
        ("invalid_input", (B5,), u8))}
    o = A.DecodeOutputs()
    for k, v in out.items():
        setattr(o, k, v.data_ptr())
    a = A.DecodeArgs()
    a.batch_size, a.steps, a.beam_size, a.vocab_size = B5, T5, K5, V5
    a.eos_token, a.length_penalty_alpha, a.repetition_penalty = C5_EOS, C5_ALPHA, 1.0
    nb = lib.dbs_cuda_decode_workspace_size(C.byref(a))
    ws = torch.empty(nb, dtype=u8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def decode():
        A.check(lib.dbs_cuda_decode_ex2(C.c_void_p(x.data_ptr()), A.DTYPE_F32, 1, C.byref(a), None, C.byref(o), None,
                                        C.c_void_p(ws.data_ptr()), nb, C.c_void_p(stream.cuda_stream)), "decode")

    for _ in range(args.warmup):
        decode()
    torch.cuda.synchronize(dev)
    times = []
    for _ in range(args.steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        decode()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        times.append(e0.elapsed_time(e1) / 1e3)
    sec = statistics.median(times)
    cand = B5 * T5 * K5 * V5
    print(json.dumps({
        "metric": METRIC, "value": cand / sec, "unit": "candidates/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": c5_workload() + "; one GPU, chained decode (decode_chain_wide_kernel)",
                   "global_batch": B5, "seq_len": T5, "beam": K5, "vocab": V5, "parallelism": "single GPU",
                   "timing": "median of per-decode CUDA events"},
        "gpu_launches": 2 * args.steps,
    }), flush=True)


def run_c5(args, rank: int, world: int, local: int):
    import torch

    from oracle import oracle

    B5, T5, K5, V5 = C5
    cand = B5 * T5 * K5 * V5
    if args.impl == "reference":
        if rank != 0:
            return
        if not oracle.ref_available():
            print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libdbs.so was not built"}))
            return
        threads = oracle.cpu_count()
        dev = "cuda" if torch.cuda.is_available() else "cpu"
        per = []
        for i in range(args.warmup + args.steps):
            value, sample = c5_cpu_reference(torch, dev, threads)
            if i >= args.warmup:
                per.append(value)
        value = statistics.median(per)
        print(json.dumps({
            "impl": "reference", "metric": METRIC, "value": value, "unit": "candidates/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": cand / value * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": c5_workload(), "global_batch": B5, "seq_len": T5, "beam": K5, "vocab": V5,
                       "parallelism": "host threads"},
            "cpu_baseline": {"value": value, "unit": "candidates/s", "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": value, "unit": "candidates/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }), flush=True)
        return

    from beamgrad_b200 import vocab_sharding as vs

    if args.c5_path == "chained":
        return run_c5_chained(args, world, local)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    dev = torch.device("cuda", local)
    x = c5_shard(torch, world, rank, dev)
    d = vs.ShardDecode(x, V5, True, world, rank, eos_token=C5_EOS, length_penalty_alpha=C5_ALPHA)
    stream = torch.cuda.current_stream(dev)

    def decode():
        vs.decode_vocab_sharded(d)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        decode()
    barrier()
    try:
        gpu_id = f"GPU-{torch.cuda.get_device_properties(dev).uuid}"
    except (AttributeError, RuntimeError):
        gpu_id = str(local)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(gpu_id) as clocks:
        barrier()
        clocks.start()
        start.record(stream)
        for _ in range(args.steps):
            decode()
        stop.record(stream)
        barrier()
        clocks.stop()
        if clocks.proc is not None and not clocks.in_window():
            clocks.extended = True
            deadline = time.monotonic() + 2.0
            while not clocks.in_window() and time.monotonic() < deadline:
                decode()
                torch.cuda.synchronize(dev)
                clocks.stop()
    elapsed = start.elapsed_time(stop) / 1e3
    t_all = torch.tensor([elapsed], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t_all, op=dist.ReduceOp.MAX)
    elapsed = float(t_all.item())

    # Stage times of one more (untimed) decode; the scan is the dominant kernel.
    d.timings = {}
    decode()
    stage = d.stage_ms()
    d.timings = None
    # Every rank's stage times (the collectives included), gathered to rank 0.
    stage_keys = ("scan", "allreduce_max", "lanes", "allgather", "merge", "select", "rescan", "allgather_rescan")
    mine = torch.tensor([stage.get(k, 0.0) for k in stage_keys], dtype=torch.float64, device=dev)
    per_rank = [mine.cpu().tolist()]
    if dist is not None:
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        per_rank = [t.cpu().tolist() for t in parts]
    stage_per_rank = [{k: round(v, 4) for k, v in zip(stage_keys, r) if k in stage} for r in per_rank]
    Vr = d.plan.shard_vocab
    scan_rows = B5 * (1 + (T5 - 1) * K5)  # rows the search may read: the scan's
    scan_bytes = scan_rows * Vr * 4 + scan_rows * d.plan.row_words * 8
    peak, peak_kind = peaks()
    achieved = scan_bytes / (stage["scan"] / 1e3) / 1e9

    # End to end: this rank's shard from pinned host memory, the decode, the outputs back.
    e2e = None
    shard_bytes = x.numel() * x.element_size()
    if not args.no_e2e and shard_bytes <= (8 << 30):
        xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        xh.copy_(x)
        outs_h = {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in d.out.items()}
        d2h = sum(v.numel() * v.element_size() for v in outs_h.values())
        n_e2e = max(2, min(args.steps, 3))

        def e2e_step():
            d.shard.copy_(xh, non_blocking=True)
            vs.decode_vocab_sharded(d)
            for k, v in d.out.items():
                outs_h[k].copy_(v, non_blocking=True)

        e2e_step()
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        s1.record(stream)
        barrier()
        e2e_t = torch.tensor([s0.elapsed_time(s1) / 1e3 / n_e2e], device=dev, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
        e2e = {"value": cand / float(e2e_t.item()), "unit": "candidates/s", "h2d_bytes_per_step": shard_bytes,
               "d2h_bytes_per_step": d2h}
        del xh

    ref_gpu = None
    if world == 1 and not args.no_reference_gpu:
        # One shard is the whole vocabulary in token order: the reference engine decodes it as is.
        from beamgrad_b200 import _abi as A

        a = A.DecodeArgs()
        a.batch_size, a.steps, a.beam_size, a.vocab_size = B5, T5, K5, V5
        a.eos_token, a.length_penalty_alpha, a.repetition_penalty = C5_EOS, C5_ALPHA, 1.0
        host = {("invalid_input" if k == "invalid" else k): v.cpu().numpy() for k, v in d.out.items()}
        ref_gpu = reference_gpu(torch, x, A.DTYPE_F32, True, a, host, args.steps, dev, stream)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and oracle.ref_available():
        threads = oracle.cpu_count()
        value, sample = c5_cpu_reference(torch, dev, threads)
        cpu = {"value": value, "unit": "candidates/s", "cores": threads, "kind": "reference", "sample": sample}

    if dist is not None:
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC,
            "value": cand / elapsed * args.steps,
            "unit": "candidates/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": elapsed / args.steps * 1e3,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": c5_workload(), "global_batch": B5, "seq_len": T5, "beam": K5, "vocab": V5,
                       "parallelism": f"vocab x{world}" if world > 1 else "single GPU (vocab-shard path, one shard)",
                       "l2": f"inputs ({shard_bytes / 1e9:.2f} GB per GPU) larger than L2 (126 MB)",
                       "stage_ms": {k: round(v, 4) for k, v in stage.items()}, "rescan_rounds": d.rounds,
                       "stage_ms_per_rank": stage_per_rank},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": None, "peak_kind": peak_kind, "kernel": "vs_scan_kernel",
                         "alg_bytes_per_launch": scan_bytes},
            "cpu_baseline": cpu,
            "reference_gpu": ref_gpu,
            "e2e": e2e,
            "gpu_launches": args.steps * (5 + d.rounds * 2),
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload == "c5":
        return run_c5(args, rank, world, local)
    if args.workload == "c4":
        return run_c4(args, rank, world, local)
    if args.workload in ("c1", "c3"):
        return run_decode_only(args, rank, world, local, SPECS[args.workload])
    if args.workload == "search":
        return run_search(args, rank, world, local)
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)

    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    from beamgrad_b200 import _abi as A

    lib = A.load()
    dev = torch.device("cuda", local)
    strong = args.scaling == "strong"
    # Strong scaling: rank r decodes examples [start, stop) of the one C2 batch (contiguous,
    # beamgrad_b200.sharding.shard_range); weak: every rank its own whole batch.
    if strong:
        from beamgrad_b200.sharding import shard_range

        start, stop = shard_range(B, rank, world)
        x = make_inputs(torch, 1000, dev, range(start, stop))
    else:
        start, stop = 0, B
        x = make_inputs(torch, 1000 + rank, dev)
    Bl = stop - start  # examples on this rank
    global_batch = B if strong else world * B

    # Outputs and workspace allocated once. The outputs are views of one flat byte buffer, so
    # that under strong scaling one all_gather_into_tensor per decode (inside the timed
    # region) leaves the whole batch's outputs on every rank, as one GPU would have them.
    f32, i32, u8 = torch.float32, torch.int32, torch.uint8
    most = max(b1 - b0 for b0, b1 in (shard_range(B, r, world) for r in range(world))) if strong else Bl
    layout = [("final_scores", (K,), f32), ("final_raw_scores", (K,), f32), ("final_lengths", (K,), i32),
              ("tokens", (T, K), i32), ("parents", (T, K), i32), ("lengths", (T, K), i32), ("scores", (T, K), f32),
              ("raw_scores", (T, K), f32), ("from_logprob", (T, K), u8), ("invalid_input", (), u8)]
    offsets, flat_bytes = {}, 0
    for name, shape, dt in layout:
        offsets[name] = flat_bytes
        n = most * (int(np.prod(shape)) if shape else 1) * torch.empty((), dtype=dt).element_size()
        flat_bytes += (n + 15) // 16 * 16
    flat = torch.zeros(flat_bytes, dtype=u8, device=dev)
    out = {}
    for name, shape, dt in layout:
        n = Bl * (int(np.prod(shape)) if shape else 1) * torch.empty((), dtype=dt).element_size()
        out[name] = flat[offsets[name]: offsets[name] + n].view(dt).view((Bl,) + shape)
    gathered = torch.empty(world * flat_bytes, dtype=u8, device=dev) if strong and world > 1 else None

    def gather_outputs():
        if gathered is not None:
            dist.all_gather_into_tensor(gathered, flat)
    row_lse = torch.empty((Bl, T, K), dtype=f32, device=dev)
    o = A.DecodeOutputs()
    for k, v in out.items():
        setattr(o, k, v.data_ptr())
    a = A.DecodeArgs()
    a.batch_size, a.steps, a.beam_size, a.vocab_size = Bl, T, K, V
    a.eos_token, a.length_penalty_alpha, a.repetition_penalty = EOS, ALPHA, 1.0
    ws_bytes = lib.dbs_cuda_decode_workspace_size(C.byref(a))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def decode(inp) -> None:
        rc = lib.dbs_cuda_decode_ex2(C.c_void_p(inp.data_ptr()), A.DTYPE_BF16, 1, C.byref(a), None, C.byref(o),
                                     C.c_void_p(row_lse.data_ptr()), C.c_void_p(ws.data_ptr()), ws_bytes,
                                     C.c_void_p(stream.cuda_stream))
        A.check(rc, "decode")

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(args.warmup):
        decode(x)
        gather_outputs()
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launch_ms = []
    try:  # nvidia-smi names the GPU by UUID, whatever CUDA_VISIBLE_DEVICES maps it to
        gpu_id = f"GPU-{torch.cuda.get_device_properties(dev).uuid}"
    except (AttributeError, RuntimeError):
        gpu_id = str(local)
    with ClockSampler(gpu_id) as clocks:
        barrier()
        clocks.start()
        start.record(stream)
        for _ in range(args.steps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            decode(x)
            e1.record(stream)
            launch_ms.append((e0, e1))
            gather_outputs()
        stop.record(stream)
        barrier()
        clocks.stop()
        if clocks.proc is not None and not clocks.in_window():
            # The timed region fell between two samples: keep the GPU on the same work
            # (untimed) until one arrives, and say so in the line.
            clocks.extended = True
            deadline = time.monotonic() + 2.0
            while not clocks.in_window() and time.monotonic() < deadline:
                decode(x)
                torch.cuda.synchronize(dev)
                clocks.stop()
    elapsed = start.elapsed_time(stop) / 1e3
    per_launch = statistics.mean(e0.elapsed_time(e1) for e0, e1 in launch_ms) / 1e3
    t_all = torch.tensor([elapsed], device=dev, dtype=torch.float64)
    if dist is not None:
        dist.all_reduce(t_all, op=dist.ReduceOp.MAX)
    elapsed = float(t_all.item())

    # Algorithmic bytes of one decode: every row the search read (V bf16 entries) + trace/state writes.
    host = {k: v.cpu().numpy() for k, v in out.items()}
    n_rows = rows_read(host["tokens"], host["parents"], host["from_logprob"], host["raw_scores"])
    trace_bytes = Bl * T * K * (4 * 5 + 1) + Bl * T * K * 4 + Bl * K * 12
    alg_bytes = n_rows * V * 2 + trace_bytes
    peak, peak_kind = peaks()
    achieved = alg_bytes / per_launch / 1e9

    # --with-backward: the dense bf16 input gradient of the decode, written once by
    # dbs_cuda_backward_dense (from logits: every row with a path gradient gets its softmax
    # correction, every other entry 0), upstream gradient linspace(-1, 1) over the beams.
    backward = None
    if args.with_backward:
        g_final = torch.linspace(-1.0, 1.0, K, device=dev).repeat(Bl, 1).contiguous()
        bi = A.BackwardInputs()
        bi.parents, bi.tokens = out["parents"].data_ptr(), out["tokens"].data_ptr()
        bi.lengths, bi.from_logprob = out["lengths"].data_ptr(), out["from_logprob"].data_ptr()
        bi.grad_final_scores = g_final.data_ptr()
        bi.logits, bi.logits_type, bi.row_lse = x.data_ptr(), A.DTYPE_BF16, row_lse.data_ptr()
        bws = lib.dbs_cuda_backward_workspace_size(C.byref(a))
        bw = torch.empty(max(bws, 1), dtype=torch.uint8, device=dev)
        grad = torch.empty_like(x)

        def backward_dense():
            A.check(lib.dbs_cuda_backward_dense(C.byref(a), C.byref(bi), C.c_void_p(grad.data_ptr()), A.DTYPE_BF16,
                                                C.c_void_p(bw.data_ptr()), bws, C.c_void_p(stream.cuda_stream)),
                    "backward")

        for _ in range(2):
            backward_dense()
        bt = []
        for _ in range(max(3, min(args.steps, 10))):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            backward_dense()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            bt.append(e0.elapsed_time(e1) / 1e3)
        bsec = statistics.median(bt)
        # Written: the whole gradient; read: the logits rows with a path gradient, i.e. the rows
        # (b, t, parent) along the final beams' backtracked paths (beams share prefixes).
        par, flp = host["parents"], host["from_logprob"]
        grad_rows = set()
        for b in range(Bl):
            slots = list(range(K))
            for t in range(T - 1, -1, -1):
                nxt = []
                for k in slots:
                    pk = int(par[b, t, k])
                    if pk < 0:
                        continue
                    if flp[b, t, k]:  # a token read from row (b, t, parent); carried-forward slots read none
                        grad_rows.add((b, t, pk))
                    nxt.append(pk)
                slots = sorted(set(nxt))
        bbytes = grad.numel() * grad.element_size() + len(grad_rows) * V * 2
        backward = {"ms": bsec * 1e3, "alg_bytes": bbytes, "rows_with_path_gradient": len(grad_rows),
                    "achieved_gbs": bbytes / bsec / 1e9, "frac": bbytes / bsec / 1e9 / peak,
                    "kernel": "backward_kernel + dense_grad_kernel (dbs_cuda_backward_dense, bf16)"}
        del grad
        # The reference-compatible form: += into a zeroed float32 gradient (dbs_cuda_backward_ex:
        # backward_kernel, then logit_correction_kernel over the rows with a path gradient).
        g32 = torch.zeros(x.shape, dtype=torch.float32, device=dev)
        ex_t = []
        for i in range(4):
            g32.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            A.check(lib.dbs_cuda_backward_ex(C.byref(a), C.byref(bi), C.c_void_p(g32.data_ptr()),
                                             C.c_void_p(bw.data_ptr()), bws, C.c_void_p(stream.cuda_stream)),
                    "backward_ex")
            e1.record(stream)
            torch.cuda.synchronize(dev)
            if i:
                ex_t.append(e0.elapsed_time(e1) / 1e3)
        backward["backward_ex_f32_ms"] = statistics.median(ex_t) * 1e3
        del g32

    # --with-pool M: the relaxed pool of the decode (one CTA per (example, step) re-reads the
    # step's rows), with its relaxed top-K weights (temperature 0.5, tolerance 1e-4, 50 iterations).
    pool = None
    if args.with_pool > 0:
        P = K * args.with_pool
        pl = {k: torch.empty((Bl, T, P), dtype=dt, device=dev)
              for k, dt in (("parents", torch.int32), ("tokens", torch.int32), ("lengths", torch.int32),
                            ("scores", torch.float32), ("raw_scores", torch.float32), ("from_logprob", torch.uint8),
                            ("relaxed_weights", torch.float32))}
        po = A.PoolOutputs()
        for k, v in pl.items():
            setattr(po, k, v.data_ptr())
        tr = A.DecodeOutputs()
        for k in ("parents", "tokens", "lengths", "raw_scores", "from_logprob"):
            setattr(tr, k, out[k].data_ptr())

        def relaxed_pool():
            A.check(lib.dbs_cuda_relaxed_pool(C.c_void_p(x.data_ptr()), A.DTYPE_BF16, 1, C.byref(a), C.byref(tr),
                                              C.c_void_p(row_lse.data_ptr()), P, 0.5, 1e-4, 50, C.byref(po),
                                              C.c_void_p(stream.cuda_stream)), "relaxed_pool")

        for _ in range(2):
            relaxed_pool()
        pt = []
        for _ in range(max(3, min(args.steps, 10))):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            relaxed_pool()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            pt.append(e0.elapsed_time(e1) / 1e3)
        psec = statistics.median(pt)
        # Read: the rows the decode read (the pool's scanned candidates come from the same rows)
        # and the trace; written: the seven [B, T, P] pool arrays.
        pbytes = n_rows * V * 2 + Bl * T * K * 17 + Bl * T * P * 25
        pool = {"ms": psec * 1e3, "multiplier": args.with_pool, "pool_size": P, "alg_bytes": pbytes,
                "achieved_gbs": pbytes / psec / 1e9, "frac": pbytes / psec / 1e9 / peak,
                "kernel": "pool_kernel (dbs_cuda_relaxed_pool, relaxed weights on)"}
        del pl

    # End to end through the same C-ABI call: pinned host input -> device, decode, outputs -> host.
    # The rank's examples go in chunks: chunk c's copy (on a copy stream) overlaps the decode of
    # chunk c - 1 (dbs_cuda_decode_ex2 on that chunk's slices of the inputs and outputs).
    e2e = None
    if not args.no_e2e:
        from beamgrad_b200.sharding import shard_range

        xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        xh.copy_(x)
        xd = torch.empty_like(x)
        outs_h = {k: torch.empty(v.shape, dtype=v.dtype, pin_memory=True) for k, v in out.items()}
        h2d = xh.numel() * xh.element_size()
        d2h = sum(v.numel() * v.element_size() for v in outs_h.values())
        e2e_steps = max(2, min(args.steps, 5))
        n_chunks = min(Bl, 8)
        chunks = [shard_range(Bl, c, n_chunks) for c in range(n_chunks)]
        calls = []
        for c0, c1 in chunks:
            ac = A.DecodeArgs()
            ac.batch_size, ac.steps, ac.beam_size, ac.vocab_size = c1 - c0, T, K, V
            ac.eos_token, ac.length_penalty_alpha, ac.repetition_penalty = EOS, ALPHA, 1.0
            oc = A.DecodeOutputs()
            for k, v in out.items():
                setattr(oc, k, v[c0:c1].data_ptr())
            calls.append((c0, c1, ac, oc, lib.dbs_cuda_decode_workspace_size(C.byref(ac))))
        ws_c = torch.empty(max(c[4] for c in calls), dtype=torch.uint8, device=dev)
        copy_stream = torch.cuda.Stream(dev)
        copied = [torch.cuda.Event() for _ in chunks]
        consumed = [torch.cuda.Event() for _ in chunks]
        for ev in consumed:
            ev.record(stream)

        def e2e_step():
            for i, (c0, c1, ac, oc, nb) in enumerate(calls):
                copy_stream.wait_event(consumed[i])  # the previous step's decode of this chunk is done
                with torch.cuda.stream(copy_stream):
                    xd[c0:c1].copy_(xh[c0:c1], non_blocking=True)
                copied[i].record(copy_stream)
                stream.wait_event(copied[i])
                rc = lib.dbs_cuda_decode_ex2(C.c_void_p(xd[c0:c1].data_ptr()), A.DTYPE_BF16, 1, C.byref(ac), None,
                                             C.byref(oc), C.c_void_p(row_lse[c0:c1].data_ptr()),
                                             C.c_void_p(ws_c.data_ptr()), nb, C.c_void_p(stream.cuda_stream))
                A.check(rc, "decode")
                consumed[i].record(stream)
            for k, v in out.items():
                outs_h[k].copy_(v, non_blocking=True)

        e2e_step()
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        copy_stream.wait_event(s0)
        for _ in range(e2e_steps):
            e2e_step()
        s1.record(stream)
        barrier()
        e2e_t = torch.tensor([s0.elapsed_time(s1) / 1e3 / e2e_steps], device=dev, dtype=torch.float64)
        if dist is not None:
            dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
        # Decoding in chunks gives the same outputs as the whole-shard decode (examples are independent).
        for k, v in outs_h.items():
            if v.numpy().tobytes() != host[k].tobytes():
                raise RuntimeError(f"e2e: chunked decode output {k} differs from the whole-shard decode")
        e2e = {"value": global_batch * T * K * V / float(e2e_t.item()), "unit": "candidates/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "chunks": n_chunks}
        del xh, xd

    ref_gpu = None
    if world == 1 and not args.no_reference_gpu:
        ref_gpu = reference_gpu(torch, x, A.DTYPE_BF16, True, a, host, args.steps, dev, stream)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle

        if oracle.ref_available():
            bits = x.view(torch.int16).cpu().numpy().view(np.uint16)
            threads = oracle.cpu_count()
            sec, reps = cpu_reference(bits, threads)
            cpu = {"value": B * T * K * V / sec, "unit": "candidates/s", "cores": threads, "kind": "reference",
                   "sample": f"the full workload ({B} examples), {reps} run(s) of libdbs dbs_decode_batch_into_ex"}

    if dist is not None:
        dist.barrier()
    if rank == 0:
        cand = global_batch * T * K * V
        line = {
            "metric": METRIC,
            "value": cand / elapsed * args.steps,
            "unit": "candidates/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": elapsed / args.steps * 1e3,
            "higher_is_better": True,
            "scaling": "strong" if strong else "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": workload(), "global_batch": global_batch, "seq_len": T, "beam": K, "vocab": V,
                       "parallelism": (f"batch-sharded over {world} GPUs, {Bl} examples on rank 0, outputs "
                                       f"all-gathered to every rank in the timed region" if strong else
                                       f"batch x{world}, {B} examples per GPU") if world > 1 else "single GPU",
                       "l2": f"inputs ({Bl * T * K * V * 2 / 1e9:.2f} GB on rank 0) larger than L2 (126 MB)"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": measured_traffic(), "peak_kind": peak_kind,
                         "alg_bytes_per_launch": alg_bytes, "rows_read": n_rows},
            "roofline_fp32": fp32_roofline(n_rows * V, per_launch, clocks.summary()),
            "cpu_baseline": cpu,
            "reference_gpu": ref_gpu,
            "backward": backward,
            "pool": pool,
            "e2e": e2e,
            "gpu_launches": 2 * args.steps,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
