#!/usr/bin/env python
"""Benchmark of the quantized-matmul hot path.

Default workload: the large-image Q8_0 GEMM, activations
M=16384 x K=3072 fp32 N(0,1), weights N=12288 x K=3072 Q8_0 encoded from
N(0, 0.02) floats.  One step = the activation quantize + the tensor-core
GEMM, inputs resident in HBM; L2 is flushed (256 MB write) between timed
steps, outside the timed events.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload q8_0_large|q8_0_gemm|q5k_gemm|q6k_gemm|dit|decode|decode_gated|decode_shapes|attention]

Multi-GPU (torchrun, one rank per GPU): the same whole problem N-sharded by
output column (weight rows) over the ranks -- rank r holds weight rows
[r*N/G, (r+1)*N/G) -- through libpxq's communicator (NCCL inside libpxq):
one step = every rank quantizes the replicated activation, its GEMM
epilogue stores its columns into every rank's Y over NVLink, with a device
barrier before and after, so every rank ends with the full Y ("scaling":
"strong"; value = whole-problem ops / max over ranks of the step time).  The
NCCL all-gather + re-layout variant is reported beside it.

At N=1 the line also carries the other BASELINE figures ("extras"): the
Q5_K GEMM, the Q8_0 GEMM, the Q5_K decode matvec
(configs[3], ms per token and HBM fraction at M=1/4/8) and the activation
quantize kernels (HBM GB/s), and a parity figure: the whole timed output
against the reference's own cpu_quant_matmul (the cpu_baseline run).

`--impl reference` times Pixelina's own CPU cpu_quant_matmul (built from the
reference sources into oracle/_ref) on the host cores, same metric/config.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Q8_0/Q5_K GEMM TOPS & matvec HBM GB/s at 1/2/4/8 B200, % of roofline"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
L2_FLUSH_BYTES = 256 << 20

Q8_0, Q5_K, Q6_K = 8, 13, 14

GEMM_WORKLOADS = {
    "q5k_gemm": dict(wtype=Q5_K, M=4096, N=10240, K=3840, name="Q5_K GEMM (BASELINE configs[1])"),
    "q8_0_gemm": dict(wtype=Q8_0, M=4096, N=3840, K=3840, name="Q8_0 GEMM (BASELINE configs[0])"),
    "q8_0_large": dict(wtype=Q8_0, M=16384, N=12288, K=3072, name="large-image Q8_0 GEMM (BASELINE configs[4])"),
    "q6k_gemm": dict(wtype=Q6_K, M=4096, N=10240, K=3840, name="Q6_K GEMM at the configs[1] shape"),
}
TYPE_NAMES = {Q8_0: "Q8_0", Q5_K: "Q5_K", Q6_K: "Q6_K"}
DIT = dict(hidden=3072, ffn=12288, blocks=60, M=4352, qkv=9216)
DECODE = dict(hidden=3584, ffn=18944, layers=28, qkv=4608)


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured"
    except Exception:  # noqa: BLE001
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def gemm_peak(wtype, bf16, peak_src):
    """The roofline peak of a GEMM line.  Q8_0 is held to the int8 tensor
    rate (2x the measured bf16 dense peak on this part: the kind::i8 and
    kind::f16 MMA rates were measured in the ratio 2.00), whichever MMA kind
    its operand kind issues; the K-quant kernels issue kind::f16 MMAs (the
    bf16 peak)."""
    if wtype == Q8_0:
        kind = os.environ.get("PXQ_Q8_0_MMA", "f16s")
        mma = "kind::i8 MMAs" if kind in ("i8", "i8s") else "kind::f16 MMAs on exact fp16 copies of the int8 quants"
        return {"peak": 2 * bf16, "unit": "TFLOP/s",
                "peak_source": f"{peak_src} bf16 dense (burst) x 2, the int8 rate; the block dots are {mma}"}
    return {"peak": bf16, "unit": "TFLOP/s",
            "peak_source": f"{peak_src} bf16 dense (burst); the GEMM issues kind::f16 MMAs on exact integer values"}


def committed_traffic(kernel_key):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(kernel_key)
    except Exception:  # noqa: BLE001
        return None


# ------------------------------------------------------------------ clocks ---

class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.lines = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.device)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:  # noqa: BLE001
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        # the sampler is running before the caller's timed region starts
        t0 = time.perf_counter()
        while not self.lines and time.perf_counter() - t0 < 3.0:
            time.sleep(0.02)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- distributed ---

class Dist:
    def __init__(self, gpus: int):
        self.world = env_int("WORLD_SIZE", 1)
        self.rank = env_int("RANK", 0)
        self.local = env_int("LOCAL_RANK", 0)
        self.pg = False
        if gpus > 1 and self.world == 1:
            print(f"--gpus {gpus} needs torchrun (WORLD_SIZE is 1); running one rank", file=sys.stderr)

    def init(self):
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(self.local)
        if self.world > 1:
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.pg = True

    def barrier(self):
        if self.pg:
            import torch.distributed as dist

            dist.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        import torch.distributed as dist

        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        import torch.distributed as dist

        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg:
            import torch.distributed as dist

            dist.destroy_process_group()


# --------------------------------------------------------- synthetic data ---

def gpu_random_q8_0(rows: int, inner: int, gen):
    """Random valid Q8_0 rows on the GPU: int8 quants in [-127,127] and fp16
    scales of N(0, 0.02) block maxima (for multi-GB stacks)."""
    import torch

    nb = inner // 32
    q = torch.randint(-127, 128, (rows, nb, 32), dtype=torch.int8, device="cuda", generator=gen)
    d = (torch.rand((rows, nb), device="cuda", generator=gen) * 0.02 + 0.04) / 127
    out = torch.empty((rows, nb, 34), dtype=torch.uint8, device="cuda")
    out[:, :, 0:2] = d.to(torch.float16).view(torch.uint8).view(rows, nb, 2)
    out[:, :, 2:] = q.view(torch.uint8)
    return out.view(rows, nb * 34)


def gpu_random_q5_K(rows: int, inner: int, gen):
    """Random valid Q5_K rows on the GPU (every field drawn independently)."""
    import torch

    nsb = inner // 256
    raw = torch.randint(0, 256, (rows, nsb, 176), dtype=torch.uint8, device="cuda", generator=gen)
    d = torch.rand((rows, nsb, 2), device="cuda", generator=gen) * 4e-5 + 2e-5
    raw[:, :, 0:4] = d.to(torch.float16).view(torch.uint8).view(rows, nsb, 4)
    return raw.view(rows, nsb * 176)


def gpu_random_q6_K(rows: int, inner: int, gen):
    """Random valid Q6_K rows on the GPU: random quants and int8 scales, small fp16 d."""
    import torch

    nsb = inner // 256
    raw = torch.randint(0, 256, (rows, nsb, 210), dtype=torch.uint8, device="cuda", generator=gen)
    d = torch.rand((rows, nsb, 1), device="cuda", generator=gen) * 1e-5 + 5e-6
    raw[:, :, 208:210] = d.to(torch.float16).view(torch.uint8).view(rows, nsb, 2)
    return raw.view(rows, nsb * 210)


# ------------------------------------------------------------------ our arm ---

def time_steps(step, steps: int, warmup: int, flush, soak_s: float, sampler: ClockSampler, dist: Dist):
    """Warm up, soak ~soak_s seconds (clock settling, sampled), then time
    exactly `steps` steps with per-step CUDA events; flush L2 between steps
    outside the events.  Returns (per-step ms list, per-step kernel ms dict)."""
    import torch

    for _ in range(warmup):
        step(None)
    torch.cuda.synchronize()
    sampler.start()
    if soak_s > 0:
        # the same number of soak steps on every rank (steps may hold collectives)
        t0 = time.perf_counter()
        step(None)
        torch.cuda.synchronize()
        n_soak = int(dist.max(soak_s / max(time.perf_counter() - t0, 1e-6)))
        for _ in range(n_soak):
            step(None)
            torch.cuda.synchronize()
    events = []
    dist.barrier()
    torch.cuda.synchronize()
    for _ in range(steps):
        flush()
        ev = {}
        step(ev)
        events.append(ev)
    torch.cuda.synchronize()
    dist.barrier()
    clocks = sampler.stop()
    step_ms, kernel_ms = [], {}
    for ev in events:
        step_ms.append(ev["start"].elapsed_time(ev["end"]))
        for k, (a, b) in ev.get("kernels", {}).items():
            kernel_ms.setdefault(k, []).append(a.elapsed_time(b))
    return step_ms, kernel_ms, clocks


def ev_pair():
    import torch

    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def run_gemm_workload(args, dist: Dist, wl: dict):
    import torch

    from pixelina_b200 import pxq, synth

    pxq.init(dist.local)
    M, N, K, wtype = wl["M"], wl["N"], wl["K"], wl["wtype"]
    # weights: identical on every rank (seed 1); activations: per rank
    wbytes = synth.weights_for(wtype, N, K, seed=1)
    x_host = synth.activations(M, K, seed=100 + dist.rank)
    W = pxq.Weight(wbytes, wtype, K, N, key=f"bench:{wtype}:{N}:{K}")
    x = torch.from_numpy(x_host).cuda()
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")

    def flush():
        flush_buf.zero_()

    def step(ev):
        if ev is not None:
            ev["start"], ev["end"] = ev_pair()
            q0, q1 = ev_pair()
            g0, g1 = ev_pair()
            ev["kernels"] = {"quantize": (q0, q1), "gemm": (g0, g1)}
            ev["start"].record()
            q0.record()
        a = pxq.Activation(wtype, x)
        if ev is not None:
            q1.record()
            g0.record()
        pxq.matmul_quantized(W, a, out=y)
        if ev is not None:
            g1.record()
            ev["end"].record()
        a.release()

    sampler = ClockSampler(dist.local)
    launches0 = pxq.kernel_launches()
    step_ms, kernel_ms, clocks = time_steps(step, args.steps, args.warmup, flush, args.soak, sampler, dist)
    pxq.synchronize()
    # launches inside the timed steps only (2 per step: quantize + GEMM)
    launches_per_step = 2
    ops = 2.0 * M * N * K
    mean_step = statistics.mean(step_ms)
    job_ms = dist.max(mean_step)
    value = ops / (job_ms * 1e-3) / 1e12
    gemm_ms = dist.max(statistics.mean(kernel_ms["gemm"]))
    quant_ms = dist.max(statistics.mean(kernel_ms["quantize"]))
    hbm, bf16, bf16_sus, peak_src = measured_peaks()
    achieved = ops / (gemm_ms * 1e-3) / 1e12
    traffic = committed_traffic(args.workload)
    result = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "TOPS",
        "n_gpus": dist.world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(job_ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "i8xi8->f32",
        "data": "synthetic (seeded N(0,1) activations; " + ("weights with uniformly random Q6_K fields)" if wtype == Q6_K
                                                            else "weights encoded from N(0,0.02))"),
        "config": {"workload": f"{args.workload}: {wl['name']}", "M": M, "N": N, "K": K,
                   "weight_type": TYPE_NAMES[wtype],
                   "activation_quant": "Q8_0" if wtype == Q8_0 else "Q8_K",
                   "parallelism": "one GPU (N>1: the same problem N-sharded)",
                   "l2": "flushed between timed steps (256 MB write, outside the events)"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), **gemm_peak(wtype, bf16, peak_src),
                     "frac": round(achieved / gemm_peak(wtype, bf16, peak_src)["peak"], 4),
                     "int8_peak_equiv": 2 * bf16, "int8_frac": round(achieved / (2 * bf16), 4),
                     "bf16_frac": round(achieved / bf16, 4),
                     "kernel": "k_gemm_q8s" if wtype == Q8_0 else "k_gemm", "kernel_ms": round(gemm_ms, 4),
                     "quantize_ms": round(quant_ms, 4),
                     "traffic": traffic},
        "clocks": clocks,
        "gpu_launches": launches_per_step * args.steps,
        "library_launch_counter": pxq.kernel_launches() - launches0,
    }
    # end to end through the host-buffer C-ABI drop-in (cpu_quant_matmul)
    result["e2e"] = e2e_host(args, dist, wbytes, wtype, x_host, N, ops)
    if dist.world == 1 and dist.rank == 0 and not args.no_cpu_baseline:
        # the reference on a bounded sample of weight rows; its outputs check the timed Y
        result["cpu_baseline"], result["parity"] = cpu_baseline(wbytes, wtype, x_host, N, ops, y_dev=y)
    W.release()
    del y
    if dist.world == 1 and not args.no_extras:
        result["extras"] = run_extras(args, dist)
    return result


def e2e_host(args, dist: Dist, wbytes, wtype, x_host, rows, ops):
    """pxq_quant_matmul on pinned host buffers: H2D of X and D2H of Y inside."""
    import torch

    from pixelina_b200 import pxq

    M, K = x_host.shape
    xin = torch.from_numpy(x_host).pin_memory()
    yout = torch.empty((M, rows), dtype=torch.float32).pin_memory()
    w = np.ascontiguousarray(wbytes)
    call = lambda: pxq.quant_matmul_ptr(w.ctypes.data, wtype, xin.data_ptr(), yout.data_ptr(), rows, M, K)  # noqa: E731
    for _ in range(2):
        assert call() == 0, pxq.last_error()
    n = max(3, min(args.steps, 10))
    dist.barrier()
    times = []
    for _ in range(n):
        t0 = time.perf_counter()
        rc = call()
        times.append(time.perf_counter() - t0)
        assert rc == 0, pxq.last_error()
    dist.barrier()
    t = dist.max(statistics.mean(times))
    return {"value": round(ops / t / 1e12, 3), "unit": "TOPS", "h2d_bytes_per_step": int(x_host.nbytes),
            "d2h_bytes_per_step": int(M * rows * 4), "ms_per_step": round(t * 1e3, 3),
            "timing": "host wall clock around the synchronous C-ABI call (pinned host buffers)",
            "api": "pxq_quant_matmul (cpu_quant_matmul drop-in)"}


def cpu_library():
    from oracle.oracle import Oracle, Reference, oracle_available, reference_available

    if reference_available():
        return Reference(), "reference"
    if oracle_available():
        return Oracle(), "port"
    return None, None


def cpu_baseline(wbytes, wtype, x_host, rows, ops, target_s: float = 12.0, y_dev=None):
    """Reference CPU cpu_quant_matmul on the host cores, bounded sample: a set
    of weight rows spread over every output tile, against all activation
    rows.  With y_dev (the GPU's output of the timed steps) the reference's
    outputs for those rows are also the parity check: returns (baseline,
    parity) then."""
    lib, kind = cpu_library()
    if lib is None:
        none = {"value": None, "unit": "TOPS", "cores": 0, "kind": "unavailable", "sample": "no CPU library built"}
        return (none, None) if y_dev is not None else none
    cores = os.cpu_count() or 1
    if kind == "reference":
        lib.set_threads(cores)
    M, K = x_host.shape
    # calibrate on a slice of weight rows, then size the sample to ~target_s
    probe_rows = 64 if kind == "reference" else 16
    t0 = time.perf_counter()
    ok, _ = lib.quant_matmul(wbytes[:probe_rows], wtype, x_host, probe_rows)
    t_probe = time.perf_counter() - t0
    per_row = t_probe / probe_rows
    sample_rows = int(min(rows, max(16, target_s / 3 / max(per_row, 1e-9))))
    sample_rows -= sample_rows % 16 or 0
    sample_rows = max(16, sample_rows)
    # rows spread evenly over the whole weight, so every output tile is sampled
    idx = np.unique(np.linspace(0, rows - 1, sample_rows).round().astype(np.int64))
    wsample = np.ascontiguousarray(wbytes[idx])
    times, ref = [], None
    for _ in range(3):
        t0 = time.perf_counter()
        ok, ref = lib.quant_matmul(wsample, wtype, x_host, len(idx))
        times.append(time.perf_counter() - t0)
        assert ok
    t = statistics.median(times)
    sample_ops = ops * len(idx) / rows
    base = {"value": round(sample_ops / t / 1e12, 5), "unit": "TOPS", "cores": cores if kind == "reference" else 1,
            "kind": kind, "sample": f"{M}x{K} activations against {len(idx)} of {rows} weight rows spread over all output "
                                    f"tiles, incl. quantize; median of 3 ({t:.2f} s each)"}
    if y_dev is None:
        return base
    import torch

    got = y_dev[:, torch.from_numpy(idx).to(y_dev.device)].cpu().numpy().astype(np.float64)
    err = float(np.abs(got - ref).max()) / max(float(np.abs(ref).max()), 1e-30)
    parity = {"max_abs_rel": err, "tolerance": 1e-3, "ok": err <= 1e-3, "against": f"{kind} cpu_quant_matmul",
              "elements_checked": int(got.size), "of_elements": int(M * rows)}
    return base, parity


# -------------------------------------------------------- reference arm ---

def run_reference(args, dist: Dist):
    from pixelina_b200 import synth

    wl = GEMM_WORKLOADS.get(args.workload, GEMM_WORKLOADS["q8_0_large"])
    M, N, K, wtype = wl["M"], wl["N"], wl["K"], wl["wtype"]
    lib, kind = cpu_library()
    if lib is None:
        return {"impl": "reference", "unavailable": "the reference CPU library (oracle/_ref) was not built"}
    cores = os.cpu_count() or 1
    if kind == "reference":
        lib.set_threads(cores)
    wbytes = synth.weights_for(wtype, N, K, seed=1)
    x = synth.activations(M, K, seed=100)
    ops_full = 2.0 * M * N * K
    # size each step so that warmup + steps stay within ~3 minutes
    t0 = time.perf_counter()
    lib.quant_matmul(wbytes[:64], wtype, x, 64)
    per_row = (time.perf_counter() - t0) / 64
    budget = 90.0 / max(1, args.steps + args.warmup)
    rows = int(min(N, max(16, budget / max(per_row, 1e-9))))
    rows -= rows % 16
    rows = max(16, rows)
    for _ in range(args.warmup):
        lib.quant_matmul(wbytes[:rows], wtype, x, rows)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ok, _ = lib.quant_matmul(wbytes[:rows], wtype, x, rows)
        times.append(time.perf_counter() - t0)
        assert ok
    t = statistics.mean(times)
    ops = ops_full * rows / N
    value = ops / t / 1e12
    sample = f"{M}x{K} activations against {rows} of {N} weight rows per step (incl. quantize), {cores} threads"
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 5), "unit": "TOPS", "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "i8xi8->f32",
        "data": "synthetic (seeded N(0,1) activations; " + ("weights with uniformly random Q6_K fields)" if wtype == Q6_K
                                                            else "weights encoded from N(0,0.02))"),
        "config": {"workload": f"{args.workload}: {wl['name']}", "M": M, "N": N, "K": K,
                   "weight_type": TYPE_NAMES[wtype], "parallelism": "host threads"},
        "cpu_baseline": {"value": round(value, 5), "unit": "TOPS", "cores": cores if kind == "reference" else 1,
                         "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 5), "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------- other workloads ---

def run_decode(args, dist: Dist, gated: bool = False):
    """Q5_K decode, 28 layers, M in {1,4,8}; one step =
    one token through every layer's matvecs (QKV, out, gate, up, down).
    gated: gate and up as one pxq_matmul_gated call, silu(gate) * up included
    (the callers' tensor_silu + tensor_gate).  Metric: weight GB/s."""
    import torch

    from pixelina_b200 import pxq

    pxq.init(dist.local)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(7)
    H, F, L, QKV = DECODE["hidden"], DECODE["ffn"], DECODE["layers"], DECODE["qkv"]
    shapes = [("qkv", QKV, H), ("out", H, H), ("gate", F, H), ("up", F, H), ("down", H, F)]
    layers = []
    for _ in range(L):
        ws = {}
        for name, n, k in shapes:
            if gated and name == "up":
                continue
            if gated and name == "gate":
                ws["gate_up"] = pxq.GatedWeight(gpu_random_q5_K(n, k, gen), gpu_random_q5_K(n, k, gen), Q5_K, k, n)
                continue
            ws[name] = pxq.Weight(gpu_random_q5_K(n, k, gen), Q5_K, k, n)
        layers.append(ws)
    torch.cuda.synchronize()
    wbytes_total = sum(pxq.weight_bytes(k, n, Q5_K) for _, n, k in shapes) * L
    results = {}
    hbm, bf16, _, peak_src = measured_peaks()
    for M in (1, 4, 8):
        xs = {H: torch.randn((M, H), device="cuda", generator=gen), F: torch.randn((M, F), device="cuda", generator=gen)}
        ys = {n: torch.empty((M, n), device="cuda") for _, n, _ in shapes}

        def token():
            for ws in layers:
                for name, n, k in shapes:
                    if gated and name == "up":
                        continue
                    if gated and name == "gate":
                        pxq.matmul_gated(ws["gate_up"], xs[k], out=ys[n])
                        continue
                    pxq.matmul(ws[name], xs[k], out=ys[n], path="matvec")

        # one token = 140 matvecs (112 with gate/up as one call), each a matvec that
        # quantizes its activation itself or a quantize kernel + matvec; replay it as
        # a CUDA graph so that host launch overhead does not hide the device time
        n0 = pxq.kernel_launches()
        token()
        launches = pxq.kernel_launches() - n0  # this library's kernels in one token
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            token()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph):
            token()
        torch.cuda.synchronize()

        def step(ev):
            if ev is not None:
                ev["start"], ev["end"] = ev_pair()
                ev["start"].record()
            graph.replay()
            if ev is not None:
                ev["end"].record()

        flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
        step_ms, _, clocks = time_steps(step, args.steps, args.warmup, flush_buf.zero_, args.soak, ClockSampler(dist.local),
                                        dist)
        ms = dist.max(statistics.mean(step_ms))
        gbs = wbytes_total / (ms * 1e-3) / 1e9
        results[f"M={M}"] = {"ms_per_token": round(ms, 4), "weight_GBps": round(gbs, 1), "hbm_frac": round(gbs / hbm, 4),
                             "launches_per_token": int(launches), "clocks": clocks}
        del graph
    name = "decode_gated: Q5_K matvec, 28 layers, gate/up as one gated call" if gated else \
        "decode: Q5_K matvec, 28 layers (BASELINE configs[3])"
    return {"metric": METRIC, "workload": name, "unit": "GB/s",
            "weight_bytes_per_token": wbytes_total, "peak_hbm_gbs": hbm, "peak_source": peak_src,
            "results": results}


def run_decode_shapes(args, dist: Dist):
    """Per-shape view of BASELINE configs[3]: each decode matrix (QKV, out,
    gate/up, down) at M = 1 and 8, one call = activation quantize + matvec;
    also gate/up and down as Q6_K (GGUF mixes Q6_K tensors into Q5_K models)
    and QKV, gate/up and down as Q8_0 (Q8_0 models: the streamed Q8_0 matvec).
    Each shape cycles through enough distinct copies of its weight to exceed
    the 126 MB L2, replayed as a CUDA graph, so the rate is HBM, not L2."""
    import torch

    from pixelina_b200 import pxq

    pxq.init(dist.local)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(9)
    H, F, QKV = DECODE["hidden"], DECODE["ffn"], DECODE["qkv"]
    hbm, _, _, peak_src = measured_peaks()
    results = {}
    shapes = [("qkv", QKV, H, Q5_K), ("out", H, H, Q5_K), ("gate_up", F, H, Q5_K), ("down", H, F, Q5_K),
              ("gate_up q6_K", F, H, Q6_K), ("down q6_K", H, F, Q6_K),
              ("qkv q8_0", QKV, H, Q8_0), ("gate_up q8_0", F, H, Q8_0), ("down q8_0", H, F, Q8_0)]
    for name, n, k, wtype in shapes:
        wbytes = pxq.weight_bytes(k, n, wtype)
        copies = max(2, -(-(320 << 20) // wbytes))
        make = {Q5_K: gpu_random_q5_K, Q6_K: gpu_random_q6_K, Q8_0: gpu_random_q8_0}[wtype]
        ws = [pxq.Weight(make(n, k, gen), wtype, k, n) for _ in range(copies)]
        for M in (1, 8):
            x = torch.randn((M, k), device="cuda", generator=gen)
            y = torch.empty((M, n), device="cuda")

            def calls():
                for w in ws:
                    pxq.matmul(w, x, out=y, path="matvec")

            calls()
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                calls()
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            with torch.cuda.graph(graph):
                calls()
            for _ in range(max(3, args.warmup)):
                graph.replay()
            torch.cuda.synchronize()
            e0, e1 = ev_pair()
            e0.record()
            for _ in range(args.steps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (args.steps * copies)
            us = dist.max(us)
            gbs = wbytes / (us * 1e-6) / 1e9
            results[f"{name} M={M}"] = {"us_per_call": round(us, 2), "weight_GBps": round(gbs, 1),
                                        "hbm_frac": round(gbs / hbm, 4)}
            del graph
        for w in ws:
            w.release()
    return {"metric": METRIC, "workload": "decode_shapes: Q5_K quantize + matvec per decode matrix (BASELINE configs[3])",
            "unit": "GB/s", "peak_hbm_gbs": hbm, "peak_source": peak_src, "results": results}


def run_dit(args, dist: Dist):
    """60 DiT blocks of Q8_0 linears, M = 4352.  One step =
    the linear stack of one forward pass (activation quantize + GEMM each)."""
    import torch

    from pixelina_b200 import pxq

    pxq.init(dist.local)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(11)
    H, F, B, M, QKV = DIT["hidden"], DIT["ffn"], DIT["blocks"], DIT["M"], DIT["qkv"]
    shapes = [("qkv", QKV, H), ("out", H, H), ("up", F, H), ("down", H, F)]
    blocks = []
    for _ in range(B):
        blocks.append({name: pxq.Weight(gpu_random_q8_0(n, k, gen), Q8_0, k, n) for name, n, k in shapes})
    xs = {H: torch.randn((M, H), device="cuda", generator=gen), F: torch.randn((M, F), device="cuda", generator=gen)}
    ys = {n: torch.empty((M, n), device="cuda") for _, n, _ in shapes}
    # build every operand copy before timing
    for blk in blocks:
        for name, n, k in shapes:
            pxq.matmul(blk[name], xs[k], out=ys[n], path="gemm")
    torch.cuda.synchronize()
    ops = sum(2.0 * M * n * k for _, n, k in shapes) * B

    def step(ev):
        if ev is not None:
            ev["start"], ev["end"] = ev_pair()
            ev["start"].record()
        for blk in blocks:
            for name, n, k in shapes:
                pxq.matmul(blk[name], xs[k], out=ys[n], path="gemm")
        if ev is not None:
            ev["end"].record()

    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    step_ms, _, clocks = time_steps(step, args.steps, args.warmup, flush_buf.zero_, args.soak, ClockSampler(dist.local), dist)
    for blk in blocks:
        for w in blk.values():
            w.release()
    ms = dist.max(statistics.mean(step_ms))
    _, bf16, _, peak_src = measured_peaks()
    tops = dist.world * ops / (ms * 1e-3) / 1e12
    return {"metric": METRIC, "workload": "dit: 60 Q8_0 DiT blocks, M=4352 (BASELINE configs[2])", "unit": "TOPS",
            "value": round(tops, 2), "ms_per_step": round(ms, 3), "ops_per_step": ops, "n_gpus": dist.world,
            "int8_frac": round(tops / dist.world / (2 * bf16), 4), "bf16_frac": round(tops / dist.world / bf16, 4),
            "peak_source": peak_src, "clocks": clocks}


def run_dit_sharded(args, dist: Dist):
    """BASELINE configs[2] N-sharded over the ranks: every linear's weight rows
    split evenly (rank r holds rows [r*n/G, (r+1)*n/G) of each of the 240
    weights), each call the sharded GEMM whose epilogue stores the rank's
    columns into every rank's output over NVLink (pxq_sharded_matmul), so each
    linear's whole output is on every rank.  value = the whole stack's
    2*M*N*K over the max over ranks of the step time (strong scaling)."""
    import torch

    from pixelina_b200 import pxq, sharded

    pxq.init(dist.local)
    G, r = dist.world, dist.rank
    comm = sharded.Comm(G, r, timeout_ms=120000)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(11)  # the same weights on every rank
    H, F, B, M, QKV = DIT["hidden"], DIT["ffn"], DIT["blocks"], DIT["M"], DIT["qkv"]
    shapes = [("qkv", QKV, H), ("out", H, H), ("up", F, H), ("down", H, F)]
    blocks = []
    for _ in range(B):
        blk = {}
        for name, n, k in shapes:
            full = gpu_random_q8_0(n, k, gen)
            blk[name] = sharded.ShardedWeight(full, Q8_0, k, n, G, r)
            del full
        blocks.append(blk)
    xs = {H: torch.randn((M, H), device="cuda", generator=gen), F: torch.randn((M, F), device="cuda", generator=gen)}
    outs = {n: sharded.ShardedOutput(comm, M, n) for n in sorted({n for _, n, _ in shapes})}
    ops = sum(2.0 * M * n * k for _, n, k in shapes) * B

    def step(ev):
        if ev is not None:
            ev["start"], ev["end"] = ev_pair()
            ev["start"].record()
        for blk in blocks:
            for name, n, k in shapes:
                sharded.sharded_matmul(comm, blk[name], xs[k], out=outs[n])
        if ev is not None:
            ev["end"].record()

    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    step_ms, _, clocks = time_steps(step, args.steps, args.warmup, flush_buf.zero_, args.soak, ClockSampler(dist.local), dist)
    comm.synchronize()
    ms = dist.max(statistics.mean(step_ms))
    _, bf16, _, peak_src = measured_peaks()
    tops = ops / (ms * 1e-3) / 1e12
    for o in outs.values():
        o.close()
    for blk in blocks:
        for w in blk.values():
            w.release()
    comm.close()
    return {"metric": METRIC, "workload": f"dit: 60 Q8_0 DiT blocks, M=4352 (BASELINE configs[2]), N-sharded over {G} GPUs",
            "unit": "TOPS", "value": round(tops, 2), "ms_per_step": round(ms, 3), "ops_per_step": ops, "n_gpus": G,
            "scaling": "strong", "per_gpu_bf16_frac": round(tops / G / bf16, 4), "peak_source": peak_src, "clocks": clocks}


def run_attention(args, dist: Dist):
    """The callers' attention step (tensor_attention) at the BASELINE models'
    shapes: DiT prefill (configs[2]: 4352 tokens, 24 heads of 128, non-causal)
    and VL decode (configs[3]: 28 heads of 128 over 4 kv heads, 8 query rows
    against a 4096-token key cache, causal).  fp32 on the CUDA cores; the
    prefill roofline is the fp32 FMA rate, the decode one HBM (keys + values)."""
    import torch

    from pixelina_b200 import pxq

    pxq.init(dist.local)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(13)
    cases = {
        "dit_prefill": dict(rows=DIT["M"], keys=DIT["M"], heads=24, kvh=24, d=128, ranges=None, off=0, causal=False),
        "vl_decode_8": dict(rows=8, keys=4096, heads=28, kvh=4, d=128, ranges=[(0, 8, 4096, True)], off=4088, causal=True),
    }
    hbm, _, _, peak_src = measured_peaks()
    props = torch.cuda.get_device_properties(dist.local)
    fp32_peak = props.multi_processor_count * 128 * 2 * 1.965e9 / 1e12  # TFLOP/s at the max SM clock
    results = {}
    for name, c in cases.items():
        q = torch.randn((c["rows"], c["heads"] * c["d"]), device="cuda", generator=gen)
        k = torch.randn((c["keys"], c["kvh"] * c["d"]), device="cuda", generator=gen)
        v = torch.randn((c["keys"], c["kvh"] * c["d"]), device="cuda", generator=gen)
        out = torch.empty_like(q)

        def step(ev):
            if ev is not None:
                ev["start"], ev["end"] = ev_pair()
                ev["start"].record()
            pxq.attention(q, k, v, c["heads"], c["kvh"], ranges=c["ranges"], query_offset=c["off"], causal=c["causal"], out=out)
            if ev is not None:
                ev["end"].record()

        flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
        step_ms, _, clocks = time_steps(step, args.steps, args.warmup, flush_buf.zero_, args.soak, ClockSampler(dist.local), dist)
        ms = dist.max(statistics.mean(step_ms))
        flops = 4.0 * c["rows"] * c["keys"] * c["heads"] * c["d"]
        kv_bytes = 2.0 * c["keys"] * c["kvh"] * c["d"] * 4
        results[name] = {"ms": round(ms, 4), "TFLOPs": round(flops / (ms * 1e-3) / 1e12, 2),
                         "fp32_frac": round(flops / (ms * 1e-3) / 1e12 / fp32_peak, 4),
                         "kv_GBps": round(kv_bytes / (ms * 1e-3) / 1e9, 1), "hbm_frac": round(kv_bytes / (ms * 1e-3) / 1e9 / hbm, 4),
                         "clocks": clocks}
        if dist.rank == 0 and not args.no_cpu_baseline:
            results[name]["cpu_baseline"] = attention_cpu_baseline(c, q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy())
    return {"metric": METRIC, "workload": "attention: DiT prefill and VL decode shapes (tensor_attention, fp32)",
            "unit": "TFLOP/s", "value": results["dit_prefill"]["TFLOPs"], "results": results, "n_gpus": dist.world,
            "fp32_peak_tflops": round(fp32_peak, 1), "peak_hbm_gbs": hbm, "peak_source": peak_src}


def attention_cpu_baseline(c, q, k, v, target_s: float = 6.0):
    """The reference's tensor_attention (oracle/_ref, all host threads) on the
    first query rows of the same inputs, sized to about target_s per call."""
    lib, kind = cpu_library()
    if kind != "reference":
        return {"value": None, "unit": "TFLOP/s", "cores": 0, "kind": "unavailable", "sample": "oracle/_ref was not built"}
    cores = os.cpu_count() or 1
    lib.set_threads(cores)

    def call(r):
        ranges = c["ranges"] if r == c["rows"] and c["ranges"] else [(0, r, c["keys"], c["causal"])]
        off = c["off"] + (c["rows"] - r if c["causal"] else 0)
        t0 = time.perf_counter()
        out = lib.attention(q[:r], k, v, c["heads"], c["kvh"], ranges, off)
        assert out is not None
        return time.perf_counter() - t0

    probe = min(c["rows"], 8)
    per_row = call(probe) / probe
    rows = int(min(c["rows"], max(probe, target_s / 3 / max(per_row, 1e-9))))
    t = statistics.median([call(rows) for _ in range(3)])
    flops = 4.0 * rows * c["keys"] * c["heads"] * c["d"]
    return {"value": round(flops / t / 1e12, 5), "unit": "TFLOP/s", "cores": cores, "kind": kind,
            "sample": f"first {rows} of {c['rows']} query rows against all {c['keys']} keys; median of 3 ({t:.2f} s each)"}


def run_gemm_sharded(args, dist: Dist, wl: dict):
    """The whole GEMM problem N-sharded over the ranks through libpxq's
    communicator (pxq_comm / pxq_sharded_matmul): rank r holds weight rows
    [r*N/G, (r+1)*N/G); one step = activation quantize + the GEMM whose
    epilogue stores every rank's columns into every rank's Y over NVLink,
    between device barriers.  value = 2*M*N*K / max over ranks of the step
    time (strong scaling)."""
    import torch

    from pixelina_b200 import pxq, sharded, synth

    pxq.init(dist.local)
    M, N, K, wtype = wl["M"], wl["N"], wl["K"], wl["wtype"]
    G, r = dist.world, dist.rank
    comm = sharded.Comm(G, r, timeout_ms=120000)
    wbytes = synth.weights_for(wtype, N, K, seed=1)  # the same bytes on every rank
    sw = sharded.ShardedWeight(wbytes, wtype, K, N, G, r)
    x_host = synth.activations(M, K, seed=100)       # replicated activation
    x = torch.from_numpy(x_host).cuda()
    out = sharded.ShardedOutput(comm, M, N)
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    ops = 2.0 * M * N * K

    def step(ev):
        if ev is not None:
            ev["start"], ev["end"] = ev_pair()
            ev["start"].record()
        sharded.sharded_matmul(comm, sw, x, out=out)
        if ev is not None:
            ev["end"].record()

    launches0 = pxq.kernel_launches()
    step_ms, _, clocks = time_steps(step, args.steps, args.warmup, flush_buf.zero_, args.soak, ClockSampler(dist.local), dist)
    comm.synchronize()
    launches = pxq.kernel_launches() - launches0
    ms = dist.max(statistics.mean(step_ms))
    value = ops / (ms * 1e-3) / 1e12
    # this rank's GEMM kernel alone, for the roofline (no collective)
    a = pxq.Activation(wtype, x)
    ylocal = torch.empty((M, sw.count), device="cuda")
    pxq.matmul_quantized(sw.weight, a, out=ylocal)
    torch.cuda.synchronize()
    g0, g1 = ev_pair()
    g0.record()
    for _ in range(5):
        pxq.matmul_quantized(sw.weight, a, out=ylocal)
    g1.record()
    torch.cuda.synchronize()
    gemm_ms = dist.max(g0.elapsed_time(g1) / 5)
    a.release()
    del ylocal
    # the NCCL all-gather + re-layout variant
    y_ag = torch.empty((M, N), device="cuda")

    def step_ag(ev):
        if ev is not None:
            ev["start"], ev["end"] = ev_pair()
            ev["start"].record()
        sharded.sharded_matmul(comm, sw, x, out=y_ag)
        if ev is not None:
            ev["end"].record()

    ag_ms, _, ag_clocks = time_steps(step_ag, args.steps, args.warmup, flush_buf.zero_, 1.0, ClockSampler(dist.local), dist)
    comm.synchronize()
    ag = dist.max(statistics.mean(ag_ms))
    same = bool(torch.equal(y_ag.view(torch.int32), out.tensor.view(torch.int32)))
    del y_ag
    # end to end: host buffers in and out through pxq_sharded_matmul_host
    xin = torch.from_numpy(x_host).pin_memory()
    yout = torch.empty((M, N), dtype=torch.float32).pin_memory()
    call = lambda: sharded.sharded_matmul_host_ptr(comm, sw, xin.data_ptr(), M, K, yout.data_ptr())  # noqa: E731
    assert call() == 0, pxq.last_error()
    n = max(3, min(args.steps, 10))
    dist.barrier()
    times = []
    for _ in range(n):
        t0 = time.perf_counter()
        rc = call()
        times.append(time.perf_counter() - t0)
        assert rc == 0, pxq.last_error()
    dist.barrier()
    t = dist.max(statistics.mean(times))
    hbm, bf16, _, peak_src = measured_peaks()
    gemm_ops = 2.0 * M * sw.count * K
    achieved = gemm_ops / (gemm_ms * 1e-3) / 1e12
    result = {
        "metric": METRIC, "value": round(value, 3), "unit": "TOPS", "n_gpus": G, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "i8xi8->f32",
        "data": "synthetic (seeded N(0,1) activations; weights encoded from N(0,0.02))",
        "config": {"workload": f"{args.workload}: {wl['name']}, N-sharded over {G} GPUs", "M": M, "N": N, "K": K,
                   "weight_type": TYPE_NAMES[wtype], "activation_quant": "Q8_0" if wtype == Q8_0 else "Q8_K",
                   "parallelism": f"N-sharded x{G} (rows {sw.count} per rank), Y assembled on every rank by the GEMM's "
                                  "peer stores over NVLink",
                   "l2": "flushed between timed steps (256 MB write, outside the events)"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), **gemm_peak(wtype, bf16, peak_src),
                     "frac": round(achieved / gemm_peak(wtype, bf16, peak_src)["peak"], 4),
                     "int8_peak_equiv": 2 * bf16, "int8_frac": round(achieved / (2 * bf16), 4),
                     "bf16_frac": round(achieved / bf16, 4),
                     "kernel": "k_gemm_q8s (this rank's shard)" if wtype == Q8_0 else "k_gemm (this rank's shard)",
                     "kernel_ms": round(gemm_ms, 4),
                     "traffic": None},
        "exchange": {"bytes_per_rank": int((G - 1) * M * sw.count * 4), "link_GBps_per_rank":
                     round((G - 1) * M * sw.count * 4 / (ms * 1e-3) / 1e9, 1),
                     "gemm_only_TOPS_per_rank": round(achieved, 2)},
        "allgather": {"value": round(ops / (ag * 1e-3) / 1e12, 3), "ms_per_step": round(ag, 4), "clocks": ag_clocks,
                      "bit_identical_to_fused": same},
        "clocks": clocks,
        "gpu_launches": int(dist.sum(launches)),
        "e2e": {"value": round(ops / t / 1e12, 3), "unit": "TOPS", "h2d_bytes_per_step": int(x_host.nbytes),
                "d2h_bytes_per_step": int(M * N * 4), "ms_per_step": round(t * 1e3, 3),
                "timing": "host wall clock around the synchronous C-ABI call on every rank (pinned host buffers; every "
                          "rank uploads X and downloads the full Y), max over ranks",
                "api": "pxq_sharded_matmul_host"},
    }
    out.close()
    sw.release()
    comm.close()
    return result


def run_extras(args, dist: Dist) -> dict:
    """The other BASELINE figures at N=1, each timed with CUDA events on its
    own: the Q5_K GEMM and Q8_0 GEMM with their
    activation quantize, the activation quantize kernels (HBM-bound), the
    Q8_0 DiT linear stack and the Q5_K decode."""
    import torch

    from pixelina_b200 import pxq

    hbm, bf16, _, peak_src = measured_peaks()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(17)
    flush_buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    out = {"peak_source": peak_src}
    for key, name in (("q5k_gemm_configs1", "q5k_gemm"), ("q8_0_gemm_configs0", "q8_0_gemm")):
        wl = GEMM_WORKLOADS[name]
        M, N, K, wtype = wl["M"], wl["N"], wl["K"], wl["wtype"]
        make = gpu_random_q5_K if wtype == Q5_K else gpu_random_q8_0
        W = pxq.Weight(make(N, K, gen), wtype, K, N)
        x = torch.randn((M, K), device="cuda", generator=gen)
        y = torch.empty((M, N), device="cuda")

        def step(ev):
            if ev is not None:
                ev["start"], ev["end"] = ev_pair()
                g0, g1 = ev_pair()
                ev["kernels"] = {"gemm": (g0, g1)}
                ev["start"].record()
            a = pxq.Activation(wtype, x)
            if ev is not None:
                g0.record()
            pxq.matmul_quantized(W, a, out=y)
            if ev is not None:
                g1.record()
                ev["end"].record()
            a.release()

        step_ms, kernel_ms, clocks = time_steps(step, args.steps, args.warmup, flush_buf.zero_, 0.5, ClockSampler(dist.local), dist)
        ops = 2.0 * M * N * K
        ms, gms = statistics.mean(step_ms), statistics.mean(kernel_ms["gemm"])
        out[key] = {"M": M, "N": N, "K": K, "weights": TYPE_NAMES[wtype], "TOPS": round(ops / (ms * 1e-3) / 1e12, 2),
                    "ms_per_step": round(ms, 4), "gemm_ms": round(gms, 4),
                    "gemm_TFLOPs": round(ops / (gms * 1e-3) / 1e12, 2),
                    "bf16_frac": round(ops / (gms * 1e-3) / 1e12 / bf16, 4),
                    "int8_frac": round(ops / (gms * 1e-3) / 1e12 / (2 * bf16), 4), "sm_mhz": clocks["sm_mhz"],
                    "reasons": clocks["reasons"]}
        W.release()
        del x, y
    # activation quantize kernels, inputs larger than L2
    for key, wtype, M, K, layout in (("quantize_q8_0_blocks", Q8_0, 16384, 3072, "gguf"),
                                     ("quantize_q8_0_operand", Q8_0, 16384, 3072, "operand"),
                                     ("quantize_q8_K_blocks", Q5_K, 16384, 3840, "gguf")):
        x = torch.randn((M, K), device="cuda", generator=gen)
        if layout == "gguf":
            fn = (lambda: pxq.quantize_q8_0(x)) if wtype == Q8_0 else (lambda: pxq.quantize_q8_K(x))
            wbytes = M * K // 32 * 34 if wtype == Q8_0 else M * K // 256 * 292
        else:
            def fn():
                pxq.Activation(wtype, x).release()
            kind = os.environ.get("PXQ_Q8_0_MMA", "f16s")  # the library's default operand kind
            # quants (int8 for kinds "i8" and "i8s", else fp16) and block scales (fp16 for "f16s" and "i8s", else fp32)
            wbytes = M * K * (1 if kind in ("i8", "i8s") else 2) + M * K // 32 * (2 if kind in ("f16s", "i8s") else 4)
        # 10 calls captured in a CUDA graph (no host launch gaps), replayed
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph):
            for _ in range(10):
                fn()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = ev_pair()
        e0.record()
        for _ in range(5):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / 50
        del graph
        nbytes = M * K * 4 + wbytes
        out[key] = {"M": M, "K": K, "ms": round(ms, 4), "GBps": round(nbytes / (ms * 1e-3) / 1e9, 1),
                    "hbm_frac": round(nbytes / (ms * 1e-3) / 1e9 / hbm, 4), "bytes": int(nbytes),
                    "timing": "10 calls per CUDA graph, 5 replays (each call one quantize kernel; inputs and outputs "
                              "larger than L2)"}
        del x
    # the DiT linear stack: 240 quantize + GEMM calls per step
    dit_args = argparse.Namespace(**{**vars(args), "steps": 3, "warmup": 1, "soak": 0.0})
    dit = run_dit(dit_args, dist)
    out["dit_configs2"] = {k: dit[k] for k in ("value", "unit", "ms_per_step", "ops_per_step", "bf16_frac", "int8_frac")}
    out["dit_configs2"]["sm_mhz"] = dit["clocks"]["sm_mhz"]
    torch.cuda.empty_cache()
    # the decode matvec stack, gate/up as one gated call
    dec = run_decode(args, dist, gated=True)
    out["decode_configs3"] = {"weight_bytes_per_token": dec["weight_bytes_per_token"],
                              **{m: {"ms_per_token": v["ms_per_token"], "weight_GBps": v["weight_GBps"],
                                     "hbm_frac": v["hbm_frac"], "launches_per_token": v["launches_per_token"],
                                     "sm_mhz": v["clocks"]["sm_mhz"]}
                                 for m, v in dec["results"].items()}}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="q8_0_large",
                    choices=sorted(GEMM_WORKLOADS) + ["attention", "decode", "decode_gated", "decode_shapes", "dit"])
    ap.add_argument("--soak", type=float, default=1.5, help="seconds of untimed steps before timing (clock settling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="N=1: skip the other BASELINE figures")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    dist = Dist(args.gpus)
    if args.impl == "reference":
        if dist.rank != 0:
            return
        print(json.dumps(run_reference(args, dist)), flush=True)
        return
    dist.init()
    try:
        if args.workload in GEMM_WORKLOADS and dist.world > 1:
            out = run_gemm_sharded(args, dist, GEMM_WORKLOADS[args.workload])
        elif args.workload in GEMM_WORKLOADS:
            out = run_gemm_workload(args, dist, GEMM_WORKLOADS[args.workload])
        elif args.workload == "decode":
            out = run_decode(args, dist)
        elif args.workload == "decode_gated":
            out = run_decode(args, dist, gated=True)
        elif args.workload == "attention":
            out = run_attention(args, dist)
        elif args.workload == "decode_shapes":
            out = run_decode_shapes(args, dist)
        else:
            out = run_dit_sharded(args, dist) if dist.world > 1 else run_dit(args, dist)
        if dist.rank == 0:
            print(json.dumps(out), flush=True)
    finally:
        dist.close()


if __name__ == "__main__":
    main()
