#!/usr/bin/env python
"""Headline benchmark: Qwen2.5-0.5B-shape int8 greedy decode, batch 1 per GPU.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    (N > 1: launched by torch.distributed.run, one rank per GPU)

Workload (BASELINE.json config 3's model at the north star's batch-1 decode):
a seeded random-init Qwen2.5-0.5B-shape int8 .ecm (24 layers, E 896, 14/2
heads, I 4864, V 151936, tied fp16 lm_head), a 64-token uniform-random prompt
prefilled once, then greedy decode.  A step is one decode token of the stream.
Positions cycle through [64, 64+256): every 256 steps a new 256-token
continuation of the cached prompt starts, so the context stays that of a
64-prompt / 256-decode run however many steps are timed.

Our arm: `value` times K steps of the device-resident decode loop (CUDA-graph
step, greedy argmax on the device) with CUDA events on the model stream, max
over ranks; `e2e` times the reference-facing call gpt2_forward with host
token/position arrays and host logits (608 KB per step) -- the same contract
the reference runtime times for its tokens_per_sec (decode forward only,
sampling excluded).  Independent replicas per GPU: weak scaling, no collective
on the data path.

Reference arm (--impl reference): the reference's own C implementation
(oracle/_ref/libecref.so, built from its sources) on the host cores, rank 0
only, same model, prompt and metric.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from edgecore_b200 import synth  # noqa: E402

METRIC = "Qwen2.5-0.5B-shape int8 decode tok/s @1/2/4/8 B200; GEMV % of HBM peak"
CONFIG_KEY = "c3_qwen05b_int8"
PROMPT = 64
PERIOD = 256
PROFILE_STEPS = 24


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4096)
    ap.add_argument("--warmup", type=int, default=32)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=512)
    ap.add_argument("--cpu-seconds", type=float, default=15.0,
                    help="minimum timed seconds of the reference CPU decode (both the reference arm and the "
                         "cpu_baseline leg, which runs the reference arm in a child process)")
    ap.add_argument("--op-sweep", action="store_true",
                    help="instead of the decode benchmark: BASELINE config 1's int8 operator sweep "
                         "(M in 1/8/64/512 and the 16384 prefill rows of config 3, Qwen2.5-0.5B (N,K) shapes), "
                         "one JSON line per shape")
    ap.add_argument("--config", default="c3", choices=["c3", "c4", "c0", "c2", "c3b"],
                    help="c3 (default): the headline, Qwen2.5-0.5B-shape int8 batch-1 decode, one stream per GPU; "
                         "c4: BASELINE config 4, Qwen2.5-1.5B-shape int8, --streams independent streams split over "
                         "the GPUs, lm_head column-split with an NCCL argmax combine")
    ap.add_argument("--streams", type=int, default=1024, help="--config c4: streams over all GPUs")
    ap.add_argument("--prompt", type=int, default=128, help="--config c4: prompt tokens per stream")
    ap.add_argument("--decode", type=int, default=128, help="--config c4: timed greedy steps per stream")
    ap.add_argument("--no-extras", action="store_true",
                    help="default line without the config 0/2 decode, operator sweep, batch sweep and config-3 "
                         "batched sub-measurements")
    ap.add_argument("--no-c4", action="store_true",
                    help="default run: skip the config-4 sub-measurement (\"c4\" in the JSON line)")
    ap.add_argument("--sweep-m", type=int, default=0, help="--op-sweep: only this M")
    ap.add_argument("--sweep-n", type=int, default=0, help="--op-sweep: only this N")
    return ap.parse_args()


def host_cores() -> int:
    return len(os.sched_getaffinity(0))


def config_dict(world: int) -> dict:
    spec = synth.CONFIGS[CONFIG_KEY]
    return {"workload": "qwen2.5-0.5b-shape int8 (W8A8 linears, fp16 tied lm_head) batch-1 greedy decode, "
                        "64-token prompt, positions cycling 64..319",
            "config": CONFIG_KEY, "n_layer": spec.n_layer, "n_embd": spec.n_embd, "n_head": spec.n_head,
            "n_kv_head": spec.n_kv_head, "intermediate": spec.intermediate, "vocab": spec.vocab,
            "prompt": PROMPT, "decode_period": PERIOD, "streams_per_gpu": 1,
            "global_batch": world, "parallelism": f"replicas{world}",
            "l2": "inputs larger than L2 (631.6 MB of weights streamed per step vs 126 MB L2)"}


# ---- clocks -------------------------------------------------------------------

class ClockSampler:
    """SM clocks and throttle reasons sampled during the timed region: NVML
    polled every 10 ms from a thread (one sample is always taken at start and
    at stop, so even a timed region of a few ms has a record); nvidia-smi at
    its 20 ms floor where NVML is missing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    PERIOD_S = 0.010
    # NVML clock-event reason bits
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, gpu_index: int):
        import threading
        self.rows: list[tuple[float, float, float, int]] = []
        self.p = None
        self.nv = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self._nvml_index(gpu_index))
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
        except Exception:
            self.nv = None
        if self.nv is not None:
            self.stop_ev = threading.Event()
            self._sample()
            self.th = threading.Thread(target=self._loop, daemon=True)
            self.th.start()
            return
        self.tmp = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-i", str(gpu_index), "-lms", "20"], stdout=self.tmp,
                                      stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    @staticmethod
    def _nvml_index(local: int) -> int:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            try:
                return int(vis.split(",")[local])
            except (ValueError, IndexError):
                pass
        return local

    def _sample(self) -> None:
        nv = self.nv
        try:
            sm = float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
            pw = nv.nvmlDeviceGetPowerUsage(self.h) / 1000.0
            rs = int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
            self.rows.append((time.perf_counter(), sm, pw, rs))
        except Exception:
            pass

    def _loop(self) -> None:
        while not self.stop_ev.wait(self.PERIOD_S):
            self._sample()

    def stop(self) -> dict:
        if self.nv is not None:
            self.stop_ev.set()
            self.th.join(timeout=5)
            self._sample()
            try:
                self.nv.nvmlShutdown()
            except Exception:
                pass
            if not self.rows:
                return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": "nvml"}
            sm = [r[1] for r in self.rows]
            reasons = sorted({n for r in self.rows for n, b in self.BITS.items() if r[3] & b})
            return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": self.max_mhz, "reasons": reasons,
                    "samples": len(self.rows), "power_w_max": max(r[2] for r in self.rows),
                    "source": f"nvml every {1e3 * self.PERIOD_S:.0f} ms"}
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.p.kill()
        self.tmp.flush()
        rows = [r.split(",") for r in Path(self.tmp.name).read_text().splitlines() if r.count(",") >= 8]
        os.unlink(self.tmp.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if "Active" in v and "Not" not in v})
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows),
                "source": "nvidia-smi -lms 20"}


# ---- CPU reference ------------------------------------------------------------

def run_reference_decode(path: Path, steps: int, warmup: int, min_s: float, threads: int, cap_s: float = 120.0,
                         key: str = CONFIG_KEY, prompt: int = PROMPT, period: int = PERIOD):
    """Reference CPU decode (oracle/_ref, built from the reference sources;
    the restatement if that is absent): `warmup` untimed steps, then timed
    steps until at least `steps` steps and `min_s` seconds are done (at most
    `cap_s` seconds).  Returns (tok/s, steps timed, kind)."""
    from oracle import oracle
    try:
        R = oracle.Reference(threads=threads)
        kind = "reference"
    except FileNotFoundError:
        R = oracle.Restatement()
        kind = "port"
    spec = synth.CONFIGS[key]
    m = R.open(path, batch_cap=1, max_ctx=prompt + period)
    m.reset()
    toks = synth.prompt_ids(spec.vocab, prompt)
    lg = m.forward(toks, np.arange(prompt, dtype=np.int32), np.zeros(prompt, np.int32))
    cur = int(np.argmax(lg[-1]))
    pos = prompt
    total, done = 0.0, 0
    i = 0
    while True:
        t0 = time.perf_counter()
        lg = m.forward(np.array([cur], np.int32), np.array([pos], np.int32))
        dt = time.perf_counter() - t0
        cur = int(np.argmax(lg[0]))
        pos = pos + 1 if pos + 1 < prompt + period else prompt
        if i >= warmup:
            total += dt
            done += 1
            if (done >= steps and total >= min_s) or total >= cap_s:
                break
        i += 1
    m.close()
    return done / total, done, kind


def reference_arm(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    name = args.config if args.config in DECODE_CONFIGS else "c3"
    key, prompt, period, metric = DECODE_CONFIGS[name]
    spec = synth.CONFIGS[key]
    path = synth.ensure_model(spec)
    threads = host_cores()
    warm = max(args.warmup, 3)
    tps, done, kind = run_reference_decode(path, args.steps, warm, args.cpu_seconds, threads,
                                           key=key, prompt=prompt, period=period)
    sample = (f"{done} timed decode steps (at least --steps {args.steps} and {args.cpu_seconds:.0f} s, at most "
              f"120 s) after a {prompt}-token prefill and {warm} warm-up steps, {threads} threads, "
              f"gpt2_forward per step as the reference runtime times it")
    line = {"impl": "reference", "metric": metric, "value": tps, "unit": "tok/s", "n_gpus": world,
            "steps": done, "warmup": warm, "ms_per_step": 1000.0 / tps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8" if spec.precision == "int8" else spec.precision,
            "data": "synthetic (seeded random-init weights)",
            "config": config_dict(1) if name == "c3" else decode_config(name),
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


DECODE_CONFIGS = {   # BASELINE configs 0, 2 and 3 at batch 1: (model, prompt tokens, decode tokens, metric)
    "c0": ("c0_gpt2_small_int8", 16, 128, "GPT-2-small-shape int8 batch-1 greedy decode tok/s"),
    "c2": ("c2_qwen05b_fp16", 64, 256, "Qwen2.5-0.5B-shape fp16 batch-1 greedy decode tok/s"),
    "c3": (CONFIG_KEY, PROMPT, PERIOD, METRIC),
}


def decode_config(name: str) -> dict:
    key, prompt, period, _ = DECODE_CONFIGS[name]
    spec = synth.CONFIGS[key]
    return {"workload": f"{key}: batch-1 greedy decode, {prompt}-token prompt, positions cycling "
                        f"{prompt}..{prompt + period - 1} ({period}-token continuations)",
            "config": key, "arch": spec.arch, "precision": spec.precision, "n_layer": spec.n_layer,
            "n_embd": spec.n_embd, "n_head": spec.n_head, "n_kv_head": spec.n_kv_head,
            "intermediate": spec.intermediate, "vocab": spec.vocab, "prompt": prompt, "decode_period": period,
            "streams_per_gpu": 1, "global_batch": 1, "parallelism": "replicas1",
            "l2": "weights streamed per step larger than L2"}


# ---- our arm ------------------------------------------------------------------

def measured_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def committed_traffic() -> dict:
    p = ROOT / "profiles" / "traffic.json"
    return json.loads(p.read_text()) if p.exists() else {}


def ours_arm(args, rank: int, world: int, local: int) -> None:
    import torch
    import torch.distributed as dist

    import edgecore_b200 as ec

    torch.cuda.set_device(local)
    spec = synth.CONFIGS[CONFIG_KEY]
    if rank == 0:
        path = synth.ensure_model(spec)
    if world > 1:
        dist.barrier()
    path = synth.ensure_model(spec)

    max_ctx = PROMPT + PERIOD
    # cold start as the reference CLI reports it (load_time_ms,
    # src/runtime_main.c:651-656): gpt2_load = parse + device upload + repack
    t_load = time.perf_counter()
    m = ec.Model(path, batch_cap=1, max_ctx=max_ctx)
    torch.cuda.synchronize()
    load_ms = (time.perf_counter() - t_load) * 1e3
    stream = torch.cuda.Stream()
    m.set_stream(stream.cuda_stream)
    toks = synth.prompt_ids(spec.vocab, PROMPT)
    lg = m.forward(toks, np.arange(PROMPT), np.zeros(PROMPT, np.int32))
    first = int(np.argmax(lg[-1]))
    d_tok = torch.tensor([first], dtype=torch.int32, device="cuda")

    # warm-up: W steps of the same cycling loop (captures the graph)
    m.decode_greedy_cycle(d_tok, PROMPT, PERIOD, max(args.warmup, 3))
    torch.cuda.synchronize()

    # timed region: exactly K steps, barrier + synchronize on both sides
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    m.decode_greedy_cycle(d_tok, PROMPT, PERIOD, args.steps)
    end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = world * args.steps / (ms_max / 1000.0)

    # e2e: the reference-facing gpt2_forward, host arrays in and host logits out
    e2e_steps = min(args.e2e_steps, args.steps)
    m.set_stream(None)
    cur = first
    lg = m.forward(toks, np.arange(PROMPT), np.zeros(PROMPT, np.int32))
    pos = PROMPT
    tok_h = np.empty(1, np.int32)
    pos_h = np.empty(1, np.int32)
    for _ in range(3):
        tok_h[0], pos_h[0] = cur, pos
        m.forward(tok_h, pos_h)
    if world > 1:
        dist.barrier()
    # One logits buffer for the whole loop, as the reference runtime keeps
    # one; each timed call is the bare C-ABI gpt2_forward on host pointers.
    out = np.empty((1, spec.vocab), np.float32)
    tok_p, pos_p, out_p = (ctypes.c_void_p(a.ctypes.data) for a in (tok_h, pos_h, out))
    fwd = m.lib.gpt2_forward
    e2e_s = 0.0
    for i in range(e2e_steps):
        tok_h[0], pos_h[0] = cur, pos
        t0 = time.perf_counter()
        fwd(m.h, tok_p, pos_p, None, 1, out_p)
        e2e_s += time.perf_counter() - t0
        cur = int(np.argmax(out[0]))
        pos = pos + 1 if pos + 1 < PROMPT + PERIOD else PROMPT
    te = torch.tensor([e2e_s], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = world * e2e_steps / float(te.item())

    # roofline of the dominant kernel, the persistent decode kernel: its one
    # launch in the timed region ran all K steps, so achieved = algorithmic
    # bytes of those K steps / the CUDA-event time of the timed region
    m.set_stream(stream.cuda_stream)
    prof = m.decode_profile(d_tok, PROMPT, PROFILE_STEPS)
    torch.cuda.synchronize()
    classes = {k: v for k, v in prof.items() if k != "steps"}
    dom = max(classes, key=lambda k: classes[k]["ms"])
    peak, peak_kind = measured_peaks()
    kv_per_pos = m.n_layer * 2 * m.n_kv_embd * 2            # K and V fp16 bytes per cached position

    def kv_bytes(p: int) -> float:                           # step at position p: read p+1 rows, write 1
        return float(kv_per_pos * (p + 2))
    prof_pos = [PROMPT + i for i in range(prof["steps"])]
    fixed = (sum(v["bytes"] for v in classes.values()) - sum(kv_bytes(p) for p in prof_pos)) / prof["steps"]
    timed_pos = [PROMPT + (i % PERIOD) for i in range(args.steps)]
    timed_bytes = args.steps * fixed + sum(kv_bytes(p) for p in timed_pos)
    achieved = timed_bytes / (ms_max / 1e3) / 1e9
    traffic_rec = committed_traffic().get("k_decode")
    traffic = traffic_rec["bytes_per_step"] * args.steps if traffic_rec else None
    roofline = {"bound": "hbm", "kernel": f"k_decode<int8,fp16,M=1> (persistent, 1 launch = {args.steps} steps)",
                "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "peak_source": (f"measured hbm_gbs (MEASURED_PEAKS.json), burst copy" if peak_kind == "measured"
                                else "fallback 6.65 TB/s"),
                "traffic": traffic,
                "traffic_source": traffic_rec["source"] if traffic_rec else None,
                "bytes_per_step": timed_bytes / args.steps,
                "method": "algorithmic bytes of the timed steps (weights, scales, biases, norm vectors, fp16 "
                          "lm_head, KV reads and writes) / CUDA-event time of the timed region on the "
                          "kernel's stream",
                "profile_us_per_step": {k: 1e3 * v["ms"] / prof["steps"] for k, v in classes.items() if v["launches"]},
                "profile_method": f"{prof['steps']} more steps, one launch each, CUDA events around every launch"}
    launches = 1   # the timed region is one launch of the persistent decode kernel
    gemv = gemv_lm_head(stream) if rank == 0 else None
    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_baseline_leg(args)
    m.close()
    extras = {}
    if rank == 0 and world == 1 and not args.no_extras:
        extras["batch_sweep"] = batch_sweep(args, stream, value)
        extras["c3_batched"] = c3_batched(args, stream)
        extras["c0"] = decode_line(args, "c0", stream)
        extras["c2"] = decode_line(args, "c2", stream)
        extras["op_sweep"] = list(op_sweep_results(args, cpu_seconds=0.25))
    c4 = None if args.no_c4 else c4_arm(args, rank, world, local)
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "int8",
                "data": "synthetic (seeded random-init weights, uniform-random prompt ids)",
                "config": config_dict(world), "clocks": clk,
                "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": 12,
                        "d2h_bytes_per_step": 4 * spec.vocab, "steps": e2e_steps,
                        "api": "gpt2_forward (host tokens/positions, host logits [1][151936])"},
                "gpu_launches": launches,
                "roofline": roofline, "cpu_baseline": cpu, "gemv_lm_head": gemv,
                "load_time_ms": load_ms, **extras, "c4": c4}
        print(json.dumps(line), flush=True)


def cpu_baseline_leg(args) -> dict:
    """The reference arm run in a child process (same code, same conditions as
    `--impl reference`: no CUDA context or torch threads in the process that
    times the CPU)."""
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
           "--warmup", str(max(args.warmup, 3)), "--cpu-seconds", str(args.cpu_seconds)]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=600)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if r.returncode != 0 or not lines:
        return {"value": None, "unit": "tok/s", "cores": host_cores(), "kind": "reference",
                "sample": f"reference arm failed: rc {r.returncode}: {r.stderr[-300:]}"}
    ref = json.loads(lines[-1])
    out = dict(ref["cpu_baseline"])
    out["sample"] = "child process `bench.py --impl reference`: " + out["sample"]
    return out


SWEEP_SHAPES = ((1152, 896), (896, 896), (4864, 896), (896, 4864), (151936, 896))


def time_op(launch, nbuf: int, reps: int, warmup: int, stream, graph: bool = True) -> float:
    """Mean µs per launch of `launch(i)` (i selects one of `nbuf` rotating
    operand sets whose total exceeds L2, so every launch reads HBM), CUDA
    events on `stream` around `reps` back-to-back launches.  With `graph`
    the launches are captured once into a CUDA graph and the graph replay is
    timed, so the figure is device time (kernels back to back) rather than
    the host cost of `reps` library calls."""
    import torch
    with torch.cuda.stream(stream):
        for i in range(warmup):
            launch(i % nbuf)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream, capture_error_mode="relaxed"):
            for i in range(reps):
                launch(i % nbuf)
        with torch.cuda.stream(stream):   # a graph replays on the current stream
            g.replay()
            torch.cuda.synchronize()
            start.record(stream)
            g.replay()
            end.record(stream)
        torch.cuda.synchronize()
        del g
        return start.elapsed_time(end) * 1e3 / reps
    with torch.cuda.stream(stream):
        start.record(stream)
        for i in range(reps):
            launch(i % nbuf)
        end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) * 1e3 / reps


def gemv_lm_head(stream, reps: int = 20, warmup: int = 3) -> dict:
    """The metric's "GEMV % of HBM peak": gemm_fp16_fp32 at M = 1 on the
    Qwen2.5-0.5B lm_head (151936 x 896 fp16, 272 MB, larger than L2) through
    ec_gemm_async, CUDA events around back-to-back launches."""
    import torch

    import edgecore_b200 as ec
    N, K, M = 151936, 896, 1
    g = torch.Generator(device="cuda").manual_seed(0)
    W = (torch.randn((N, K), device="cuda", generator=g) * 0.02).half()
    X = torch.randn((M, K), device="cuda", generator=g)
    out = torch.empty((M, N), device="cuda")
    us = time_op(lambda i: ec.gemm_async(1, out, X, None, W.view(torch.int16), stream=stream.cuda_stream),
                 1, reps, warmup, stream)
    assert ec.device_error_take(stream.cuda_stream) == 0
    peak, kind = measured_peaks()
    algo = N * K * 2 + M * K * 4 + M * N * 4
    del W
    return {"op": "gemm_fp16_fp32", "M": M, "N": N, "K": K, "us": us, "achieved_gbs": algo / us / 1e3,
            "frac": algo / us / 1e3 / peak, "peak": peak, "peak_source": kind,
            "kernel": "k_gemv<fp16,M=1> (weight streaming)", "algorithmic_bytes": algo}


# ---- sub-measurements of the default line (1 GPU) ------------------------------

def child_reference(args, config: str, cpu_seconds: float) -> dict | None:
    """`bench.py --impl reference --config <config>` in a child process (no CUDA
    context or torch threads in the process that times the CPU); its line."""
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--config", config, "--steps", "1",
           "--warmup", str(max(args.warmup, 3)), "--cpu-seconds", str(cpu_seconds)]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=900)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if r.returncode != 0 or not lines:
        return {"value": None, "cores": host_cores(), "kind": "reference",
                "sample": f"reference arm failed: rc {r.returncode}: {r.stderr[-300:]}"}
    return json.loads(lines[-1])


def decode_line(args, name: str, stream, steps: int | None = None, cpu: bool = True) -> dict:
    """Batch-1 greedy decode of BASELINE config 0 / 2 / 3: the device-resident
    loop timed with CUDA events (value), the reference-facing gpt2_forward
    with host arrays (e2e), the algorithmic bytes of the timed steps over the
    measured time (roofline), and the reference CPU path on the host cores."""
    import torch

    import edgecore_b200 as ec
    key, prompt, period, metric = DECODE_CONFIGS[name]
    spec = synth.CONFIGS[key]
    path = synth.ensure_model(spec)
    steps = steps or 4 * period
    t_load = time.perf_counter()
    m = ec.Model(path, batch_cap=1, max_ctx=prompt + period)
    torch.cuda.synchronize()
    load_ms = (time.perf_counter() - t_load) * 1e3
    m.set_stream(stream.cuda_stream)
    toks = synth.prompt_ids(spec.vocab, prompt)
    lg = m.forward(toks, np.arange(prompt), np.zeros(prompt, np.int32))
    first = int(np.argmax(lg[-1]))
    d_tok = torch.tensor([first], dtype=torch.int32, device="cuda")
    m.decode_greedy_cycle(d_tok, prompt, period, max(args.warmup, 3))
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(torch.cuda.current_device())
    start.record(stream)
    m.decode_greedy_cycle(d_tok, prompt, period, steps)
    end.record(stream)
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms = start.elapsed_time(end)
    prof = m.decode_profile(d_tok, prompt, 8)
    torch.cuda.synchronize()
    classes = {k: v for k, v in prof.items() if k != "steps"}
    kv_per_pos = m.n_layer * 2 * m.n_kv_embd * 2
    fixed = (sum(v["bytes"] for v in classes.values())
             - sum(kv_per_pos * (prompt + i + 2) for i in range(prof["steps"]))) / prof["steps"]
    timed_bytes = steps * fixed + sum(kv_per_pos * (prompt + (i % period) + 2) for i in range(steps))
    peak, peak_kind = measured_peaks()
    achieved = timed_bytes / (ms / 1e3) / 1e9
    # e2e: gpt2_forward on host arrays, host logits
    m.set_stream(None)
    m.forward(toks, np.arange(prompt), np.zeros(prompt, np.int32))
    tok_h, pos_h = np.empty(1, np.int32), np.empty(1, np.int32)
    out = np.empty((1, spec.vocab), np.float32)
    tok_p, pos_p, out_p = (ctypes.c_void_p(a.ctypes.data) for a in (tok_h, pos_h, out))
    fwd = m.lib.gpt2_forward
    cur, pos, e2e_s, n_e2e = first, prompt, 0.0, min(128, period)
    for i in range(n_e2e + 3):
        tok_h[0], pos_h[0] = cur, pos
        t0 = time.perf_counter()
        fwd(m.h, tok_p, pos_p, None, 1, out_p)
        if i >= 3:
            e2e_s += time.perf_counter() - t0
        cur = int(np.argmax(out[0]))
        pos = pos + 1 if pos + 1 < prompt + period else prompt
    m.close()
    line = {"metric": metric, "value": steps / (ms / 1e3), "unit": "tok/s", "n_gpus": 1, "steps": steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms / steps, "higher_is_better": True,
            "dtype": spec.precision, "config": decode_config(name), "clocks": clk,
            "e2e": {"value": n_e2e / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": 4 * spec.vocab, "steps": n_e2e,
                    "api": f"gpt2_forward (host tokens/positions, host logits [1][{spec.vocab}])"},
            "gpu_launches": 1,
            "roofline": {"bound": "hbm", "kernel": f"k_decode (persistent, 1 launch = {steps} steps)",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": peak_kind, "bytes_per_step": timed_bytes / steps, "traffic": None,
                         "method": "algorithmic bytes of the timed steps / CUDA-event time of the timed launch"},
            "load_time_ms": load_ms, "cpu_baseline": None}
    if cpu:
        ref = child_reference(args, name, min(args.cpu_seconds, 5.0))
        line["cpu_baseline"] = ref.get("cpu_baseline", ref) if ref else None
    return line


def batch_sweep(args, stream, m1_value: float) -> list:
    """Batched greedy decode of the config-3 model over M independent streams
    (each a distinct 64-token prompt in its own KV slot): M = 1 is the
    headline loop; M = 8, 32, 128 run ec_decode_batch (the persistent decode
    kernel up to 7 streams; from 8, one CUDA graph of the per-layer kernels
    per step with tensor-core GEMMs)."""
    import torch

    import edgecore_b200 as ec
    spec = synth.CONFIGS[CONFIG_KEY]
    path = synth.ensure_model(spec)
    out = [{"M": 1, "tok_s": m1_value, "path": "k_decode (persistent)"}]
    steps = 64
    for M in (8, 32, 128):
        m = ec.Model(path, batch_cap=M, max_ctx=PROMPT + 2 * steps + 8)
        m.set_stream(stream.cuda_stream)
        t = np.concatenate([synth.prompt_ids(spec.vocab, PROMPT, seed=100 + b) for b in range(M)]).astype(np.int32)
        p = np.tile(np.arange(PROMPT, dtype=np.int32), M)
        sl = np.repeat(np.arange(M, dtype=np.int32), PROMPT)
        ids, _ = m.forward_argmax(t, p, sl)
        d_tok = torch.from_numpy(ids.reshape(M, PROMPT)[:, -1].copy()).cuda()
        d_pos = torch.full((M,), PROMPT, dtype=torch.int32, device="cuda")
        wt, wp = d_tok.clone(), d_pos.clone()
        torch.cuda.synchronize()       # the library's stream starts after torch's default stream
        m.decode_batch(wt, wp, max(args.warmup, 3))
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        m.decode_batch(d_tok, d_pos, steps)
        end.record(stream)
        torch.cuda.synchronize()
        assert ec.device_error_take(stream.cuda_stream) == 0
        ms = start.elapsed_time(end)
        out.append({"M": M, "tok_s": M * steps / (ms / 1e3), "ms_per_step": ms / steps, "steps": steps,
                    "path": "ec_decode_batch: " + ("k_decode (persistent, one launch for all steps)" if M < 8 else
                                                   "one CUDA graph of per-layer kernels per step, tcgen05 GEMMs"),
                    "graph_kernels_per_step": m.batch_graph_kernels(0) if M > 8 else 0})
        m.close()
    return out


C3B_SEQ, C3B_LEN, C3B_DEC = 32, 512, 128


def c3_batched(args, stream) -> dict:
    """32 sequences x 512 distinct uniform-random prompt
    tokens prefilled in one gpt2_forward-shaped call (rows carry their own
    positions and KV slots, reference src/edgecore.h:249-260), then 128
    greedy decode steps of the 32 streams (ec_decode_batch).  The prefill's
    tensor work is the int8 linears (2 * rows * int8 weights) plus the fp16
    lm_head over every row, the counts BASELINE quotes (1.17e13 + 4.46e12)."""
    import torch

    import edgecore_b200 as ec
    spec = synth.CONFIGS[CONFIG_KEY]
    path = synth.ensure_model(spec)
    S, P, D = C3B_SEQ, C3B_LEN, C3B_DEC
    m = ec.Model(path, batch_cap=S, max_ctx=P + D + 8)
    m.set_stream(stream.cuda_stream)
    t = np.concatenate([synth.prompt_ids(spec.vocab, P, seed=300 + b) for b in range(S)]).astype(np.int32)
    p = np.tile(np.arange(P, dtype=np.int32), S)
    sl = np.repeat(np.arange(S, dtype=np.int32), P)
    m.forward_argmax(t, p, sl)                      # workspaces and tensor maps for S*P rows
    torch.cuda.synchronize()
    reps, best = 3, 1e30
    for _ in range(reps):
        t0 = time.perf_counter()
        ids, _ = m.forward_argmax(t, p, sl)
        torch.cuda.synchronize()
        best = min(best, time.perf_counter() - t0)
    rows = S * P
    L, E, I, V, kv = spec.n_layer, spec.n_embd, spec.intermediate, spec.vocab, spec.kv_embd
    w_int8 = L * ((E + 2 * kv) * E + E * E + 2 * I * E + E * I)
    int8_ops = 2.0 * rows * w_int8
    fp16_flops = 2.0 * rows * V * E
    d_tok = torch.from_numpy(ids.reshape(S, P)[:, -1].copy()).cuda()
    d_pos = torch.full((S,), P, dtype=torch.int32, device="cuda")
    wt, wp = d_tok.clone(), d_pos.clone()
    torch.cuda.synchronize()           # the library's stream starts after torch's default stream
    m.decode_batch(wt, wp, max(args.warmup, 3))
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    m.decode_batch(d_tok, d_pos, D)
    end.record(stream)
    torch.cuda.synchronize()
    assert ec.device_error_take(stream.cuda_stream) == 0
    dms = start.elapsed_time(end)
    m.close()
    line = {"metric": "Qwen2.5-0.5B-shape int8: 32x512 distinct-prompt prefill, then 128 batched greedy steps",
            "prefill_tok_s": rows / best, "prefill_ms": best * 1e3, "prefill_rows": rows,
            "prefill_int8_tops": int8_ops / best / 1e12, "prefill_fp16_tflops": fp16_flops / best / 1e12,
            "prefill_tensor_ops": {"int8": int8_ops, "fp16": fp16_flops},
            "prefill_timing": f"best of {reps} host-timed forward_argmax calls of {rows} rows (synchronised)",
            "decode_tok_s": S * D / (dms / 1e3), "decode_ms_per_step": dms / D, "decode_steps": D,
            "decode_timing": "CUDA events around ec_decode_batch of 128 steps",
            "kv": "paged arena: 64-position pages per slot, mapped as the prefill and the decode steps reach them"}
    ref = child_reference(args, "c3b", 0.0)
    line["cpu_baseline"] = ref.get("cpu_baseline", ref) if ref else None
    return line


def c3b_reference_arm(args, rank: int) -> None:
    """The reference's own C path on a bounded sample of config 3: a prefill of
    2 x 128 distinct-prompt rows in one gpt2_forward call, then 3 batched
    steps of 32 streams."""
    if rank != 0:
        return
    from oracle import oracle
    try:
        R, kind = oracle.Reference(threads=host_cores()), "reference"
    except FileNotFoundError:
        R, kind = oracle.Restatement(), "port"
    spec = synth.CONFIGS[CONFIG_KEY]
    path = synth.ensure_model(spec)
    n, plen = 2, 128
    # the reference's workspaces hold max(max_ctx, batch_cap) rows per call (src/gpt2.c:319-351)
    m = R.open(path, batch_cap=C3B_SEQ, max_ctx=n * plen + 8)
    m.reset()
    t = np.concatenate([synth.prompt_ids(spec.vocab, plen, seed=300 + b) for b in range(n)]).astype(np.int32)
    t0 = time.perf_counter()
    m.forward(t, np.tile(np.arange(plen, dtype=np.int32), n), np.repeat(np.arange(n, dtype=np.int32), plen))
    pre = n * plen / (time.perf_counter() - t0)
    cur = synth.prompt_ids(spec.vocab, C3B_SEQ, seed=7).astype(np.int32)
    slots = np.arange(C3B_SEQ, dtype=np.int32)
    pos = np.full(C3B_SEQ, plen, np.int32)
    m.forward(cur, pos, slots)
    t0 = time.perf_counter()
    for s in range(3):
        lg = m.forward(cur, pos + 1 + s, slots)
        cur = np.argmax(lg, axis=1).astype(np.int32)
    dec = 3 * C3B_SEQ / (time.perf_counter() - t0)
    m.close()
    sample = (f"prefill of {n} x {plen} rows in one gpt2_forward call ({pre:.1f} tok/s), then 3 batched steps "
              f"of {C3B_SEQ} streams ({dec:.1f} tok/s), {host_cores()} threads")
    line = {"impl": "reference", "metric": "config 3 batched decode tok/s (CPU sample)", "value": dec,
            "unit": "tok/s", "prefill_tok_s": pre,
            "cpu_baseline": {"value": dec, "unit": "tok/s", "prefill_tok_s": pre, "cores": host_cores(),
                             "kind": kind, "sample": sample},
            "e2e": {"value": dec, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- config 4: many independent streams, column-split lm_head --------------

C4_KEY = "c4_qwen15b_int8"
C4_METRIC = "Qwen2.5-1.5B-shape int8 batched greedy decode tok/s (1024 streams, column-split lm_head)"


def c4_config(args, world: int) -> dict:
    spec = synth.CONFIGS[C4_KEY]
    return {"workload": f"qwen2.5-1.5b-shape int8 (W8A8 linears, fp16 tied lm_head): {args.streams} independent "
                        f"streams, {args.prompt}-token uniform-random prompts prefilled untimed, then {args.decode} "
                        f"greedy decode steps per stream; streams split data-parallel over the GPUs, lm_head "
                        f"column-split with one NCCL all_gather of hidden rows and one all_reduce(MAX) of int64 "
                        f"argmax keys per step",
            "config": C4_KEY, "n_layer": spec.n_layer, "n_embd": spec.n_embd, "n_head": spec.n_head,
            "n_kv_head": spec.n_kv_head, "intermediate": spec.intermediate, "vocab": spec.vocab,
            "streams": args.streams, "streams_per_gpu": args.streams // world, "prompt": args.prompt,
            "decode_steps": args.decode, "global_batch": args.streams,
            "parallelism": f"dp{world} streams + lm_head column split x{world}",
            "l2": "inputs larger than L2 (1.78 GB of int8 layer weights streamed per step vs 126 MB L2)"}


def c4_prompts(spec, g0: int, n: int, plen: int) -> np.ndarray:
    return np.stack([synth.prompt_ids(spec.vocab, plen, seed=100_000 + g0 + j) for j in range(n)])


def c4_reference_decode(args, threads: int, steps: int = 3, rows: int = 8, plen: int = 8):
    """The reference's CPU batched decode of the config-4 model on a bounded
    sample: `rows` streams with `plen`-token prompts (shorter than the GPU
    run's: the CPU time is in the GEMMs, not the short-context attention),
    then `steps` batched gpt2_forward calls of `rows` rows."""
    from oracle import oracle
    # the reference's loader holds 512 tensor entries (src/gpt2.c:180-181) and
    # this 28-layer model with q/k/v biases has 534: the restatement of the
    # reference numerics (same algorithm, its own C, OpenMP GEMMs) stands in
    R = oracle.Restatement()
    kind = "port"
    spec = synth.CONFIGS[C4_KEY]
    m = R.open(synth.ensure_model(spec), batch_cap=rows, max_ctx=plen + steps + 1)
    m.reset()
    pr = c4_prompts(spec, 0, rows, plen)
    lg = m.forward(pr.reshape(-1), np.tile(np.arange(plen, dtype=np.int32), rows),
                   np.repeat(np.arange(rows, dtype=np.int32), plen))
    cur = np.argmax(lg.reshape(rows, plen, -1)[:, -1], axis=1).astype(np.int32)
    pos = np.full(rows, plen, np.int32)
    t0 = time.perf_counter()
    for _ in range(steps):
        lg = m.forward(cur, pos, np.arange(rows, dtype=np.int32))
        cur = np.argmax(lg, axis=1).astype(np.int32)
        pos += 1
    dt = time.perf_counter() - t0
    m.close()
    return rows * steps / dt, kind, (f"{steps} batched forward steps of {rows} streams after {plen}-token "
                                     f"prompts, {threads} threads, the C restatement of the reference numerics "
                                     f"(the reference cannot load this model: 534 tensors > its 512-entry table)")


def c4_reference_arm(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    threads = host_cores()
    tps, kind, sample = c4_reference_decode(args, threads)
    line = {"impl": "reference", "metric": C4_METRIC, "value": tps, "unit": "tok/s", "n_gpus": world,
            "steps": 3, "warmup": 0, "ms_per_step": 1000.0 * 8 / tps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic (seeded random-init weights)",
            "config": c4_config(args, 1),
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": threads, "kind": kind, "sample": sample},
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def c4_arm(args, rank: int, world: int, local: int) -> None:
    import torch
    import torch.distributed as dist

    import edgecore_b200 as ec
    from edgecore_b200.vocab_shard import ShardedBatchDecoder

    torch.cuda.set_device(local)
    if args.streams % world:
        raise SystemExit(f"--streams {args.streams} must be a multiple of the GPU count {world}")
    spec = synth.CONFIGS[C4_KEY]
    if rank == 0:
        synth.ensure_model(spec)
    if world > 1:
        dist.barrier()
    path = synth.ensure_model(spec)
    mloc = args.streams // world
    e2e_steps = 4
    ctx = args.prompt + args.decode + e2e_steps + 1
    m = ec.Model(path, batch_cap=mloc, max_ctx=ctx)
    stream = torch.cuda.current_stream()   # the decoder runs on its own stream and orders itself with this one

    # untimed prefill of this rank's streams (full lm_head): first greedy ids
    g0 = rank * mloc
    first = np.empty(mloc, np.int32)
    per = max(1, 8192 // args.prompt)
    for j0 in range(0, mloc, per):
        n = min(per, mloc - j0)
        pr = c4_prompts(spec, g0 + j0, n, args.prompt)
        ids, _ = m.forward_argmax(pr.reshape(-1), np.tile(np.arange(args.prompt, dtype=np.int32), n),
                                  np.repeat(np.arange(j0, j0 + n, dtype=np.int32), args.prompt))
        first[j0:j0 + n] = ids.reshape(n, args.prompt)[:, -1]
    tok = torch.from_numpy(first).cuda()
    pos = torch.full((mloc,), args.prompt, dtype=torch.int32, device="cuda")

    dec = ShardedBatchDecoder(m, rank, world, mloc, spec.n_embd, spec.vocab, device=torch.device("cuda", local))
    # warm-up on a copy of the state: same shapes (graph capture, tensor maps), untimed
    wt, wp = tok.clone(), pos.clone()
    for s in range(max(args.warmup, 3)):
        dec.step(wt, wp, args.prompt + s + 1)
    torch.cuda.synchronize()

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler(local) if rank == 0 else None
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for s in range(args.decode):
        dec.step(tok, pos, args.prompt + s + 1)
    end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    t = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    value = args.streams * args.decode / (ms / 1e3)

    # kernels per timed step: the captured layer graph, then the lm_head
    # block (activation split + tensor-core GEMM), the row argmax (2), the key
    # packing and the key -> token advance; NCCL kernels not counted
    launches = args.decode * (m.batch_graph_kernels(1) + 6)

    # e2e through the reference-facing gpt2_forward: host token / position
    # arrays of this rank's streams, host logits [mloc][vocab] of the full
    # lm_head, each call synchronous (the reference runtime's contract)
    m.set_vocab_shard(0, spec.vocab)
    cur = tok.cpu().numpy()
    p_h = pos.cpu().numpy()
    slots = np.arange(mloc, dtype=np.int32)
    out = np.empty((mloc, spec.vocab), np.float32)
    m.forward(cur, p_h, slots, out=out)       # first call: full-vocab workspaces
    cur = np.argmax(out, axis=1).astype(np.int32)
    p_h = p_h + 1
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps - 1):
        m.forward(cur, p_h, slots, out=out)
        cur = np.argmax(out, axis=1).astype(np.int32)
        p_h = p_h + 1
    te = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e = args.streams * (e2e_steps - 1) / float(te.item())

    # roofline of a decode step: HBM bytes that must move per step (every int8
    # layer weight, scales, this GPU's lm_head block, the KV rows read and
    # written) and the tensor work (int8 linears + fp16 lm_head over all rows)
    peak, peak_kind = measured_peaks()
    L, E, I, V = spec.n_layer, spec.n_embd, spec.intermediate, spec.vocab
    kv = spec.kv_embd
    w_int8 = L * ((E + 2 * kv) * E + E * E + 2 * I * E + E * I)
    lm_bytes = V * E * 2 / world
    mean_ctx = args.prompt + (args.decode + 1) / 2
    kv_bytes = mloc * L * 2 * kv * 2 * (mean_ctx + 1)
    step_bytes = w_int8 * (1 + 4 / E) + lm_bytes + kv_bytes
    step_s = ms / 1e3 / args.decode
    flops = 2.0 * mloc * w_int8 + 2.0 * args.streams * V * E / world
    roofline = {"bound": "hbm", "achieved": step_bytes / step_s / 1e9, "peak": peak, "unit": "GB/s",
                "frac": step_bytes / step_s / 1e9 / peak, "traffic": None,
                "peak_source": "measured hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured" else "fallback",
                "bytes_per_step": step_bytes, "tensor_ops_per_step": flops,
                "tensor_tops": flops / step_s / 1e12,
                "method": "algorithmic bytes per step (int8 layer weights + scales, this GPU's fp16 lm_head block, "
                          "KV rows read and written at the mean context) / CUDA-event time per step, per GPU"}
    cpu = None
    if rank == 0 and world == 1:
        tps, kind, sample = c4_reference_decode(args, host_cores())
        cpu = {"value": tps, "unit": "tok/s", "cores": host_cores(), "kind": kind, "sample": sample}
    line = None
    if rank == 0:
        line = {"metric": C4_METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.decode,
                "warmup": max(args.warmup, 3), "ms_per_step": ms / args.decode, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "int8",
                "data": "synthetic (seeded random-init weights, uniform-random prompt ids)",
                "config": c4_config(args, world), "clocks": clk,
                "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 12 * mloc,
                        "d2h_bytes_per_step": 4 * mloc * spec.vocab, "steps": e2e_steps - 1,
                        "api": f"gpt2_forward per rank ({mloc} host token/position/slot rows, host logits "
                               f"[{mloc}][{spec.vocab}])"},
                "gpu_launches": launches, "roofline": roofline, "cpu_baseline": cpu}
    del dec
    m.close()
    return line


def op_sweep(args) -> None:
    for line in op_sweep_results(args, cpu_seconds=min(args.cpu_seconds, 2.0)):
        print(json.dumps(line), flush=True)


def op_sweep_results(args, cpu_seconds: float):
    """BASELINE config 1's int8 operator sweep plus the fp16 lm_head, through
    ec_gemm_async with device operands: X int8 [M][K] (the A2 quantisation
    output) with a_scale, W int8 [N][K] with per-row scales (or fp16 W and
    fp32 X).  Kernel time = CUDA events around back-to-back launches that
    rotate through weight copies totalling >= 256 MB (> 126 MB L2).  One
    JSON line per shape, with the reference CPU gemm on a bounded sample."""
    import torch

    import edgecore_b200 as ec
    torch.manual_seed(0)
    stream = torch.cuda.Stream()
    peak, peak_kind = measured_peaks()
    ref = None
    if cpu_seconds > 0:
        try:
            from oracle import oracle
            ref = oracle.Reference(threads=host_cores())
        except FileNotFoundError:
            ref = None
    cases = [("int8", M, N, K) for M in (1, 8, 64, 512) for N, K in SWEEP_SHAPES]
    cases += [("fp16", M, 151936, 896) for M in (1, 8, 64, 512)]
    for wt_name, M, N, K in cases:
        if (args.sweep_m and M != args.sweep_m) or (args.sweep_n and N != args.sweep_n):
            continue
        wt = 0 if wt_name == "int8" else 1
        elt = 1 if wt == 0 else 2
        wbytes = N * K * elt
        nbuf = max(1, -(-(256 << 20) // wbytes))
        if wt == 0:
            Ws = [torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda") for _ in range(nbuf)]
            A = torch.randint(-127, 128, (M, K), dtype=torch.int8, device="cuda")
            a_s = torch.rand(M, device="cuda") * 1e-2 + 1e-3
        else:
            Ws = [(torch.randn((N, K), device="cuda") * 0.02).half().view(torch.int16) for _ in range(nbuf)]
            A = torch.randn((M, K), device="cuda")
            a_s = None
        w_s = torch.rand(N, device="cuda") * 1.9e-2 + 1e-3 if wt == 0 else None
        out = torch.empty((M, N), device="cuda")
        us = time_op(lambda i: ec.gemm_async(wt, out, A, a_s, Ws[i], w_s, stream=stream.cuda_stream),
                     nbuf, max(10, 2 * nbuf), max(args.warmup, 3), stream)
        assert ec.device_error_take(stream.cuda_stream) == 0
        algo = wbytes + (4 * N if wt == 0 else 0) + M * K * (1 if wt == 0 else 4) + (4 * M if wt == 0 else 0) + 4 * M * N
        flops = 2.0 * M * N * K
        line = {"op_sweep": "gemm_int8" if wt == 0 else "gemm_fp16_fp32", "M": M, "N": N, "K": K,
                "us_per_call": us, "algorithmic_bytes": algo, "achieved_gbs": algo / us / 1e3,
                "hbm_frac": algo / us / 1e3 / peak, "hbm_peak_gbs": peak, "peak_source": peak_kind,
                "tops" if wt == 0 else "tflops": flops / us / 1e6,
                "path": "weight-streaming GEMV" if M < 8 else "tcgen05",
                "timing": f"CUDA events around one replay of a CUDA graph of {max(10, 2 * nbuf)} back-to-back "
                          f"launches rotating {nbuf} weight copies ({nbuf * wbytes / 2**20:.0f} MiB > L2)"}
        if ref is not None and M * N * K <= 2e10:
            Ah = A.cpu().numpy()
            Wh = Ws[0].cpu().numpy()
            t0 = time.perf_counter()
            n = 0
            while True:
                if wt == 0:
                    ref.gemm_int8(Ah, a_s.cpu().numpy(), Wh, w_s.cpu().numpy())
                else:
                    ref.gemm_fp16(Ah, Wh.view(np.uint16))
                n += 1
                if time.perf_counter() - t0 >= cpu_seconds:
                    break
            cpu_us = (time.perf_counter() - t0) / n * 1e6
            line["cpu_baseline"] = {"value": cpu_us, "unit": "us_per_call", "cores": host_cores(),
                                    "kind": "reference", "sample": f"{n} calls of the reference "
                                    f"{'gemm_int8' if wt == 0 else 'gemm_fp16_fp32'} on host operands"}
        else:
            line["cpu_baseline"] = None
        del Ws, A, out
        yield line


def main():
    args = parse()
    if args.op_sweep:
        op_sweep(args)
        return
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        if args.config == "c4":
            c4_reference_arm(args, rank, world)
        elif args.config == "c3b":
            c3b_reference_arm(args, rank)
        else:
            reference_arm(args, rank, world)
        return
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
                                device_id=torch.device("cuda", local))
    try:
        if args.config == "c4":
            line = c4_arm(args, rank, world, local)
            if rank == 0:
                print(json.dumps(line), flush=True)
        elif args.config in ("c0", "c2") and rank == 0:
            print(json.dumps(decode_line(args, args.config, torch.cuda.Stream(), steps=args.steps)), flush=True)
        elif args.config == "c3b" and rank == 0:
            print(json.dumps(c3_batched(args, torch.cuda.Stream())), flush=True)
        elif args.config in ("c3",):
            ours_arm(args, rank, world, local)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
