"""Benchmark of the quantized decode-GEMV hot path on B200 (driver contract: one JSON line).

Workload (the reference's op-sweep config): y = x . W^T at M = 1 (one decode
token, bf16 activations) for every feasible (format, shape) of
  formats Q4_K, Q6_K, Q8_0 (GGUF blocks) and FP8 E4M3 (per-channel scale)
  shapes (N, K) = (4096, 4096), (14336, 4096), (4096, 14336), (151936, 896)
(Q4_K / Q6_K need K % 256 == 0, so their K = 896 points are infeasible).
A "step" is one pass over the 14 GEMVs; every step reads 0.74 GB of distinct
weights, well above the 126 MB L2, so each weight byte comes from HBM.

Metric: quant-GEMV HBM GB/s from algorithmic bytes (packed weights + x + y (+ FP8
channel scales)); dequantized weights never count.  value = device-timed
(weights and x resident in HBM, CUDA graph of the step, CUDA events); e2e = the
same through the C ABI, every step copying its 14 activation rows in from pinned
host memory and reading its 14 outputs back before the next step.

The line also carries the roofline of the longest GEMV (against the measured HBM
copy bandwidth), the CPU baseline (the restated reference path on the host cores),
the SM clocks sampled during the timed steps, and:
  m_sweep  the rest of the config-1 token counts (M = 4..2048) at 14336 x 4096,
           1 GPU only (M >= 4 runs the tensor-core GEMM);
  tp       N > 1: the fused row-parallel linear against GEMV + NCCL all-reduce.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    python bench.py --profile-one FMT:N:K[:M] | sweep   (ncu target, no JSON line)

N > 1 runs under torchrun, one rank per GPU, each rank its own copy of the sweep
(weak scaling: independent weight shards), max time over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (151936, 896)]
FORMATS = [("Q4_K", 12), ("Q6_K", 14), ("Q8_0", 8), ("FP8", 0)]
METRIC = "quant-GEMV HBM GB/s (decode M=1, config-1 sweep)"
UNIT = "GB/s"


def sweep():
    out = []
    for name, t in FORMATS:
        for (n, k) in SHAPES:
            if t in (12, 14) and k % 256:
                continue
            out.append((name, t, n, k))
    return out


def weight_bytes(t, n, k):
    if t == 0:
        return n * k + 4 * n
    elems, bb = {8: (32, 34), 12: (256, 144), 14: (256, 210)}[t]
    return n * (k // elems) * bb


def alg_bytes(t, n, k, m=1):
    return weight_bytes(t, n, k) + m * k * 2 + m * n * 2  # bf16 x in, bf16 y out


def read_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(kernel_tag: str):
    """dram bytes per launch recorded in profiles/<kernel_tag>.md (line 'dram_bytes_per_launch: N')."""
    p = os.path.join(ROOT, "profiles", kernel_tag + ".md")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


class Clocks:
    """nvidia-smi sampling during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = os.path.join("/tmp", f"rtd_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def wait_first_sample(self, timeout_s: float = 5.0) -> None:
        """Block until the sampler has written its first line (nvidia-smi start-up)."""
        t0 = time.perf_counter()
        while self.proc is not None and time.perf_counter() - t0 < timeout_s:
            self.f.flush()
            if os.path.exists(self.path) and os.path.getsize(self.path) > 0:
                return
            time.sleep(0.05)

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": reasons, "samples": len(rows)}


_CPU_ROWS = 1024  # rows of each sweep point's CPU sample
_CPU_SAMPLES = {}  # (type, K) -> the sample rows of one sweep point, generated once per process


def _cpu_sample(t, k):
    from runtimed_b200 import synth

    key = (t, k)
    if key not in _CPU_SAMPLES:
        x = synth.bf16_round(synth.activations(1, k, seed=0))
        if t == 0:
            _CPU_SAMPLES[key] = (x, synth.fp8_matrix(_CPU_ROWS, k, seed=0))
        else:
            _CPU_SAMPLES[key] = (x, synth.quant_matrix(t, _CPU_ROWS, k, seed=0))
    return _CPU_SAMPLES[key]


def cpu_baseline(budget_s: float = 20.0):
    """The restated reference CPU path (oracle/: bit-exact block decode + f32 dot,
    OpenMP over all host threads) on a bounded row sample of every sweep point.  Only
    the oracle calls are timed; the samples are generated once per process."""
    import oracle

    threads = os.cpu_count() or 1
    tot_bytes, tot_s = 0.0, 0.0
    per = budget_s / len(sweep())
    rows_used = {}
    for name, t, n, k in sweep():
        rows = 64
        x, sample = _cpu_sample(t, k)
        if t == 0:
            w, s = sample
        else:
            raw = sample
        spent, done_b = 0.0, 0.0
        while spent < per:  # row blocks double up to the whole sample, then repeat
            t0 = time.perf_counter()
            if t == 0:
                oracle.ref_cpu_fp8_linear(x, w[:rows], s[:rows], rows, k, threads=threads)
            else:
                row_b = weight_bytes(t, 1, k)
                oracle.ref_cpu_linear(t, raw[: rows * row_b], rows, k, x, threads=threads)
            dt = time.perf_counter() - t0
            spent += dt
            done_b += alg_bytes(t, rows, k)
            if dt < 0.25 and rows < _CPU_ROWS:
                rows *= 2
        tot_bytes += done_b
        tot_s += spent
        rows_used[f"{name}:{n}x{k}"] = rows
    return {"value": tot_bytes / tot_s / 1e9, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"row samples of every sweep point (~{budget_s:.0f} s of CPU work), oracle/rtd_oracle.c "
                      f"restating the reference block decoders + f32 dot, OpenMP {threads} threads"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    base = None
    for _ in range(max(args.warmup, 0)):
        cpu_baseline(budget_s=2.0)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        base = cpu_baseline(budget_s=max(5.0, 60.0 / max(args.steps, 1)))
        vals.append(base["value"])
    wall = time.perf_counter() - t0
    value = statistics.mean(vals)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall * 1e3 / max(args.steps, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": config_dict(),
            "cpu_baseline": dict(base, value=value),
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def launches_per_gemv(t: int, n: int, k: int) -> int:
    """Kernels one M=1 bf16 call launches (rtd_gemv.cu launch_qgemv): the GEMV alone when
    the launch runs in whole mode (at least two 16-row tiles per warp of two 8-warp CTAs
    on each of the 148 SMs) and every CTA can stage the activation row itself (K % 8 == 0,
    the staged row plus its column-sum table within 40 KB); otherwise a prep kernel too."""
    gk, sbe = {0: (128, 32), 8: (128, 32), 12: (256, 32), 14: (256, 16)}[t]
    kp = -(-k // gk) * gk
    tab = (kp // gk) * (gk // sbe + 4)
    whole = -(-n // 16) >= 2 * 148 * 2 * 8
    return 1 if (whole and k % 8 == 0 and kp * 2 + tab * 4 <= 40 * 1024) else 2


def config_dict():
    return {"workload": "config1 quantized-linear op sweep at decode M=1 (y = x.W^T), one step = 14 GEMVs",
            "formats": [f for f, _ in FORMATS], "shapes_nk": SHAPES, "m": 1, "activations": "bf16",
            "weights": "random-init GGUF blocks with the config-1 distributions (seed 0)",
            "l2": "inputs larger than L2: 0.74 GB of distinct weights per step vs 126 MB L2",
            "parallelism": "replicas: each rank streams its own weight copy"}


def _time_steps(graph, stream, dev, n: int) -> float:
    import torch

    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(n):
        graph.replay()
    b.record(stream)
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b) * 1e-3


def _tp_rowparallel(world, rank, dev, stream, reps: int = 20):
    """Row-parallel down_proj of the 70B-shaped config (Q6_K, N = 8192, K = 28672 split
    over the ranks): the reduction fused into the GEMV epilogue (peer stores over NVLink)
    against the same GEMV followed by an NCCL all-reduce.  Each path is captured in a
    CUDA graph of `reps` calls (the fused call keeps its epoch on the device, so replays
    are valid); device time per call, max over ranks; every rank issues the same calls
    and collectives in the same order."""
    import torch
    import torch.distributed as dist
    from runtimed_b200 import synth
    from runtimed_b200.tp import RowParallelLinear, TpComm
    from runtimed_b200.weights import Context

    t, n, k = 14, 8192, 28672
    raw = synth.quant_matrix(t, n, k, seed=7)
    comm = TpComm(Context.for_device(dev), rank, world, max_n=n)
    rpl = RowParallelLinear.from_full_weight(raw, t, n, k, None, rank, world, comm=comm, device=dev)
    del raw
    out = {"shape_nk": [n, k], "format": "Q6_K", "world": world, "k_shard": k // world,
           "timing": f"CUDA graph of {reps} calls per path, 5 replays, CUDA events, max over ranks"}
    for m in (1, 4):
        x = torch.from_numpy(synth.activations(m, k // world, seed=rank)).to(torch.bfloat16).to(dev)
        res = {}
        for name, fn in (("fused", rpl.forward), ("nccl", rpl.forward_nccl)):
            for _ in range(3):
                fn(x)
            torch.cuda.synchronize(dev)
            dist.barrier()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(reps):
                    fn(x)
            g.replay()
            torch.cuda.synchronize(dev)
            dist.barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(5):
                g.replay()
            b.record(stream)
            torch.cuda.synchronize(dev)
            del g  # graphs holding NCCL work go before the process group
            ms = torch.tensor([a.elapsed_time(b) / (5 * reps)], dtype=torch.float64, device=dev)
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
            res[name] = float(ms.item()) * 1e3
        shard_bytes = n * (k // world // 256) * 210
        out[f"m{m}"] = {"fused_us": res["fused"], "nccl_us": res["nccl"],
                        "fused_shard_gbs": shard_bytes / (res["fused"] * 1e-6) / 1e9}
    torch.cuda.synchronize(dev)
    dist.barrier()
    comm.close()
    return out


def _m_sweep(dev, rank: int):
    """The rest of the config-1 sweep's token counts at (N, K) = (14336, 4096) for every
    format (the four M = 1 shapes are the headline step): skinny M = 4, 16, 64 in GB/s of
    algorithmic bytes (HBM roofline) and prefill M = 512, 2048 in TFLOP/s (tensor
    roofline against the measured bf16 burst peak).  Each point is a CUDA graph of 10
    calls over 3 weight copies (L2 is not reused between calls), 5 replays, CUDA events."""
    import torch
    from runtimed_b200 import _lib, synth
    from runtimed_b200.weights import Fp8Weight, QMatMul

    L = _lib.lib()
    n, k = 14336, 4096
    tflops_peak = None
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            tflops_peak = json.load(f).get("bf16_tflops")
    out = {"shape_nk": [n, k], "timing": "CUDA graph of 10 calls over 3 weight copies, 5 replays, CUDA events",
           "tflops_peak": tflops_peak, "tflops_peak_source": "MEASURED_PEAKS.json bf16_tflops (measured)"}
    for name, t in FORMATS:
        objs = []
        for c in range(3):
            if t == 0:
                w, sc = synth.fp8_matrix(n, k, seed=rank + 20 + c, stream=k)
                objs.append(Fp8Weight(w, sc, k, n, device=dev))
            else:
                objs.append(QMatMul(t, synth.quant_matrix(t, n, k, seed=rank + 20 + c, stream=k), n, k, device=dev))
        row = {}
        for m in (4, 16, 64, 512, 2048):
            x = torch.randn(m, k, device=dev).to(torch.bfloat16)
            y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)

            def call(o, st):
                if t == 0:
                    rc = L.rtd_fp8_linear(o.ctx.handle, o.handle, x.data_ptr(), _lib.DT_BF16, k, m, y.data_ptr(),
                                          _lib.DT_BF16, n, _lib.FP8_W8A16, st)
                else:
                    rc = L.rtd_qlinear(o.ctx.handle, o.handle, x.data_ptr(), _lib.DT_BF16, k, m, None, y.data_ptr(),
                                       _lib.DT_BF16, n, st)
                if rc != 0:
                    raise RuntimeError(f"m-sweep {name} M={m}: status {rc}")

            for o in objs:
                call(o, torch.cuda.current_stream(dev).cuda_stream)
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for r in range(10):
                    call(objs[r % 3], torch.cuda.current_stream(dev).cuda_stream)
            for _ in range(2):
                g.replay()
            torch.cuda.synchronize(dev)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(5):
                g.replay()
            b.record()
            torch.cuda.synchronize(dev)
            del g
            us = a.elapsed_time(b) * 1e3 / 50
            if m <= 64:
                gbs = (weight_bytes(t, n, k) + m * k * 2 + m * n * 2) / (us * 1e-6) / 1e9
                row[f"m{m}"] = {"us": round(us, 2), "gbs": round(gbs, 1)}
            else:
                tf = 2.0 * m * n * k / (us * 1e-6) / 1e12
                row[f"m{m}"] = {"us": round(us, 2), "tflops": round(tf, 1),
                                "frac": round(tf / tflops_peak, 3) if tflops_peak else None}
        out[name] = row
        del objs
    return out


def _dominant_launch_ms(it, call, stream, dev, rank, reps: int = 24) -> float:
    import torch
    from runtimed_b200 import synth
    from runtimed_b200.weights import Fp8Weight, QMatMul

    t, n, k = it["t"], it["n"], it["k"]
    copies = [it]
    for c in range(2):
        if t == 0:
            w, s = synth.fp8_matrix(n, k, seed=rank + 10 + c, stream=k)
            obj = Fp8Weight(w, s, k, n, device=dev)
        else:
            obj = QMatMul(t, synth.quant_matrix(t, n, k, seed=rank + 10 + c, stream=k), n, k, device=dev)
        copies.append(dict(it, obj=obj))
    for cp in copies:
        call(cp)
    torch.cuda.synchronize(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for r in range(reps):
            call(copies[r % 3], st=torch.cuda.current_stream(dev))
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(5):
        g.replay()
    b.record(stream)
    torch.cuda.synchronize(dev)
    del g
    return a.elapsed_time(b) / (5 * reps)


def profile_one(spec: str, calls: int) -> int:
    """Run `calls` bf16 calls of one linear (FMT:N:K, or FMT:N:K:M for M tokens; M = 1 by
    default), or of every sweep GEMV in step order ("sweep"), eagerly, and exit: the
    target of the ncu captures summarised under profiles/ (the bench's own step is a
    CUDA graph, which ncu reports as one result)."""
    import torch
    from runtimed_b200 import _lib, synth
    from runtimed_b200.weights import Fp8Weight, QMatMul

    m = 1
    if spec == "sweep":
        todo = [(t, n, k) for _, t, n, k in sweep()]
    else:
        parts = spec.split(":")
        name, n, k = parts[:3]
        m = int(parts[3]) if len(parts) > 3 else 1
        todo = [(dict(FORMATS)[name], int(n), int(k))]
    dev = torch.device("cuda", 0)
    L = _lib.lib()
    st = torch.cuda.current_stream(dev).cuda_stream
    items = []
    for t, n, k in todo:
        x = torch.from_numpy(synth.bf16_round(synth.activations(m, k, seed=0))).to(torch.bfloat16).to(dev)
        y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        if t == 0:
            w, s = synth.fp8_matrix(n, k, seed=0, stream=k)
            o = Fp8Weight(w, s, k, n, device=dev)
        else:
            o = QMatMul(t, synth.quant_matrix(t, n, k, seed=0, stream=k), n, k, device=dev)
        items.append((t, n, k, o, x, y))
    for _ in range(calls):
        for t, n, k, o, x, y in items:
            if t == 0:
                rc = L.rtd_fp8_linear(o.ctx.handle, o.handle, x.data_ptr(), _lib.DT_BF16, k, m, y.data_ptr(),
                                      _lib.DT_BF16, n, _lib.FP8_W8A16, st)
            else:
                rc = L.rtd_qlinear(o.ctx.handle, o.handle, x.data_ptr(), _lib.DT_BF16, k, m, None, y.data_ptr(),
                                   _lib.DT_BF16, n, st)
            if rc != 0:
                raise RuntimeError(f"status {rc}")
    torch.cuda.synchronize(dev)
    print(f"profile-one {spec}: {calls} calls of {len(items)} GEMVs ok")
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--profile-one", default=None, metavar="FMT:N:K[:M]|sweep",
                    help="only run a few eager calls of one sweep GEMV or of the whole sweep (ncu target), "
                         "no JSON line")
    ap.add_argument("--calls", type=int, default=4)
    args = ap.parse_args()
    if args.profile_one:
        return profile_one(args.profile_one, args.calls)
    if args.impl == "reference":
        run_reference(args)
        return 0

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    from runtimed_b200 import _lib, synth
    from runtimed_b200.weights import Fp8Weight, QMatMul

    L = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    items = []
    for name, t, n, k in sweep():
        if t == 0:
            w, s = synth.fp8_matrix(n, k, seed=rank, stream=k)
            obj = Fp8Weight(w, s, k, n, device=dev)
        else:
            obj = QMatMul(t, synth.quant_matrix(t, n, k, seed=rank, stream=k), n, k, device=dev)
        x = synth.bf16_round(synth.activations(1, k, seed=rank, stream=n))
        xd = torch.from_numpy(x).to(torch.bfloat16).to(dev)
        yd = torch.empty((1, n), dtype=torch.bfloat16, device=dev)
        items.append(dict(name=name, t=t, n=n, k=k, obj=obj, x=xd, y=yd, bytes=alg_bytes(t, n, k)))
    step_bytes = sum(it["bytes"] for it in items)

    def call(it, x=None, y=None, st=None):
        x = it["x"] if x is None else x
        y = it["y"] if y is None else y
        s = (stream if st is None else st).cuda_stream
        o = it["obj"]
        if it["t"] == 0:
            rc = L.rtd_fp8_linear(o.ctx.handle, o.handle, x.data_ptr(), _lib.DT_BF16, it["k"], 1, y.data_ptr(),
                                  _lib.DT_BF16, it["n"], _lib.FP8_W8A16, s)
        else:
            rc = L.rtd_qlinear(o.ctx.handle, o.handle, x.data_ptr(), _lib.DT_BF16, it["k"], 1, None, y.data_ptr(),
                               _lib.DT_BF16, it["n"], s)
        if rc != 0:
            raise RuntimeError(f"{it['name']} {it['n']}x{it['k']}: status {rc}: {L.rtd_last_error(o.ctx.handle)}")

    for it in items:  # first calls configure kernel attributes outside capture
        call(it)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for it in items:
            call(it, st=torch.cuda.current_stream(dev))
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize(dev)

    # ---- timed region (device time, CUDA events, max over ranks)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # nvidia-smi samples every 200 ms: the timed K steps sit inside a window of the same
    # load (an untimed pre-roll of about a second and a short post-roll), so the clock
    # samples are taken while the GPU runs exactly this work.
    step_s = max(1e-5, _time_steps(graph, stream, dev, 5) / 5)
    roll = max(1, int(1.0 / step_s))
    with Clocks(local) as clk:
        clk.wait_first_sample()
        for _ in range(roll):
            graph.replay()
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        for _ in range(roll // 2):
            graph.replay()
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    t_max = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms_max = float(t_max.item())
    value = world * step_bytes * args.steps / (ms_max * 1e-3) / 1e9

    # ---- per-GEMV device time (each call preceded by a sleep so only GPU time is measured)
    reps = 5
    per = {i: [] for i in range(len(items))}
    for _ in range(reps):
        for i, it in enumerate(items):
            torch.cuda._sleep(200_000)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            call(it)
            b.record(stream)
            per[i].append((a, b))
    torch.cuda.synchronize(dev)
    per_ms = {i: statistics.mean(a.elapsed_time(b) for a, b in v) for i, v in per.items()}
    dom = max(per_ms, key=lambda i: per_ms[i])
    dit = items[dom]
    peak, peak_kind = read_peaks()
    # roofline kernel: its average launch duration back to back, as inside the step --
    # a graph of R launches rotating over 3 weight copies (no launch re-reads L2)
    launch_ms = _dominant_launch_ms(dit, call, stream, dev, rank)
    achieved = dit["bytes"] / (launch_ms * 1e-3) / 1e9
    tag = f"qgemv_{dit['name'].lower()}_{dit['n']}x{dit['k']}_m1"
    traffic = profile_traffic(tag)
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "traffic": traffic, "kernel": f"qgemv_kernel, {dit['name']} {dit['n']}x{dit['k']} M=1",
                "launch_us": launch_ms * 1e3,
                "duration_source": "CUDA events around a graph of 24 back-to-back launches over 3 weight copies",
                "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                "per_gemv_gbs": {f"{it['name']}:{it['n']}x{it['k']}": round(it["bytes"] / (per_ms[i] * 1e-3) / 1e9, 1)
                                 for i, it in enumerate(items)}}

    # ---- end to end through the C ABI: every step copies its 14 activation rows from
    # pinned host memory (one copy into one device buffer), runs the 14 calls on them,
    # and reads the 14 outputs back into pinned host memory (one copy), then waits for it
    xoff, yoff, xo, yo = [], [], 0, 0
    for it in items:
        xoff.append(xo)
        yoff.append(yo)
        xo += it["k"]
        yo += it["n"]
    hx = torch.empty(xo, dtype=torch.bfloat16).pin_memory()
    hy = torch.empty(yo, dtype=torch.bfloat16).pin_memory()
    dx = torch.empty(xo, dtype=torch.bfloat16, device=dev)
    dy = torch.empty(yo, dtype=torch.bfloat16, device=dev)
    for i, it in enumerate(items):
        hx[xoff[i]:xoff[i] + it["k"]].copy_(it["x"].reshape(-1).cpu())
    xs = [dx[xoff[i]:xoff[i] + it["k"]] for i, it in enumerate(items)]
    ys = [dy[yoff[i]:yoff[i] + it["n"]] for i, it in enumerate(items)]
    e2e_steps = max(3, args.steps // 2)
    h2d = xo * 2
    d2h = yo * 2

    def e2e_step():
        dx.copy_(hx, non_blocking=True)
        for i, it in enumerate(items):
            call(it, x=xs[i], y=ys[i])
        hy.copy_(dy, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()

    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    b.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_val = world * step_bytes * e2e_steps / (float(e2e_ms.item()) * 1e-3) / 1e9
    # the outputs read back are the step's results: check one against the device copy
    if not torch.equal(hy[:items[0]["n"]].to(dev), dy[:items[0]["n"]]):
        raise RuntimeError("e2e: host copy of the outputs differs from the device")

    tp = None
    if world > 1:
        # the TP comparison runs after the headline is measured; a failure there is
        # reported in its own object instead of losing the line (a rank that fails
        # alone leaves the others to the process group's 120 s timeout)
        try:
            tp = _tp_rowparallel(world, rank, dev, stream)
        except Exception as e:  # noqa: BLE001 - reported in the JSON line
            tp = {"error": f"{type(e).__name__}: {e}"}
            torch.cuda.synchronize(dev)
    msweep = _m_sweep(dev, rank) if world == 1 else None
    cpu = cpu_baseline() if (rank == 0 and world == 1) else None
    del graph
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 tensor-core products of exact weight codes, f32 accumulate",
            "data": "synthetic", "config": config_dict(), "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "path": "rtd_qlinear / rtd_fp8_linear per GEMV, eager; per step one pinned-host copy of the 14 "
                            "activation rows in and one of the 14 outputs out, then a host wait"},
            "gpu_launches": sum(launches_per_gemv(it["t"], it["n"], it["k"]) for it in items) * args.steps,
            "tp": tp,
            "m_sweep": msweep,
            "clocks": clk.summary()}
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
