"""Benchmark of the quantized forward-pass hot path on B200 (driver contract: one JSON line).

Headline: decode tokens/s of config 3, the 70B-shaped Qwen2 decoder (hidden 8192, FFN
28672, 64 query / 8 KV heads of 128, 80 layers, Q4_K_M-style: Q4_K q/k/o/gate/up, Q6_K
v/down, q/k/v bias), batch 64, tensor parallel over the N GPUs of the run:
  * a step is one decode token for each of the 64 sequences through the seven linears of
    all 80 layers -- 43.5 GB of packed weights at N = 1, 1/N of them on each rank;
  * column parallel (output rows split, no exchange): attn_q / attn_k / attn_v, ffn_gate,
    ffn_up; row parallel (input columns split, all-reduce of the outputs): attn_output and
    ffn_down, through rtd_tp_qlinear_row -- the exchange fused into the GEMV epilogue up to
    three tokens, the tensor-core GEMM plus the library's two-shot NVLink all-reduce from
    four on;
  * the step carries the layer's real data flow between linears (q's head shard feeds
    attn_output, ffn_gate's shard feeds ffn_down); attention, RMSNorm and SwiGLU are not
    part of this path.  Each layer reads its own device copy of the weights (80 distinct
    copies of one seeded random layer: the kernels' work and HBM traffic do not depend on
    the weight values), so every step streams all 80 layers from HBM.
value = B * steps / device time of the step's CUDA graph (max over ranks, strong
scaling: the same model and batch at every N).  e2e = the same through the public API
with the step's hidden states copied in from pinned host memory and its outputs read
back every step.  The line also carries the batch-1 step, the roofline of the step's
dominant kernel and of the whole step, the CPU baseline (the reference's CPU quantized
matmul restated -- 8-bit activation blocks, AVX2 integer dots -- on the host cores, scaled
to the step), the SM clocks of the timed window, and:
  tp          N > 1: the config-3 row-parallel linears (attn_output, ffn_down) fused vs the
              library's all-reduce vs NCCL, at M = 1 and 64, each checked against the
              unsharded single-GPU result (rel_l2);
  gemv_sweep  N = 1: the config-1 quantized-linear sweep at decode M = 1 (14 GEMVs, HBM
              GB/s of algorithmic bytes) with the roofline of its longest GEMV;
  m_sweep     N = 1: the config-1 token counts M = 4..2048 at (14336, 4096);
  model_decode  N = 1: config 0 end to end (GGUF load, 128-token prompt, greedy decode
              steps as a CUDA graph, the pick in the LM head's epilogue) in tokens/s,
              beside the restated reference forward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
    python bench.py --profile-one FMT:N:K[:M] | sweep | tpstep[:B] | greedy:FMT:N:K
                                                                     (ncu target, no JSON line)
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

Q8_0, Q4_K, Q6_K = 8, 12, 14
# config 3: the 70B-shaped decoder
HIDDEN, FFN, N_HEAD, N_KV, HEAD_DIM, N_LAYERS = 8192, 28672, 64, 8, 128, 80
BATCH = 64
# (name, ggml type, N out, K in, split, bias): the seven linears of one layer in call order
LAYER_LINEARS = [
    ("attn_q", Q4_K, N_HEAD * HEAD_DIM, HIDDEN, "col", True),
    ("attn_k", Q4_K, N_KV * HEAD_DIM, HIDDEN, "col", True),
    ("attn_v", Q6_K, N_KV * HEAD_DIM, HIDDEN, "col", True),
    ("attn_output", Q4_K, HIDDEN, N_HEAD * HEAD_DIM, "row", False),
    ("ffn_gate", Q4_K, FFN, HIDDEN, "col", False),
    ("ffn_up", Q4_K, FFN, HIDDEN, "col", False),
    ("ffn_down", Q6_K, HIDDEN, FFN, "row", False),
]
TYPE_NAMES = {Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}
METRIC = "decode tokens/s (config-3 70B-shaped Qwen2, linears of all 80 layers, batch 64, TP over N GPUs)"
UNIT = "tokens/s"

SHAPES = [(4096, 4096), (14336, 4096), (4096, 14336), (151936, 896)]
FORMATS = [("Q4_K", 12), ("Q6_K", 14), ("Q8_0", 8), ("FP8", 0)]


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


def shard_shape(n, k, split, world):
    return (n // world, k) if split == "col" else (n, k // world)


def step_weight_bytes(world: int) -> int:
    """Packed weight bytes one rank streams per step (all layers, its shards)."""
    return N_LAYERS * sum(weight_bytes(t, *shard_shape(n, k, sp, world)) for _, t, n, k, sp, _ in LAYER_LINEARS)


def read_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured", d.get("bf16_tflops")
    return 6650.0, "fallback", 1590.0


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


# ---------------------------------------------------------------- CPU baseline
_CPU_ROWS = 256      # rows of each linear's CPU sample (full K)
_CPU_SAMPLES = {}    # (type, n, k) -> (x, raw rows), generated once per process


def _cpu_sample(t, k, m):
    from runtimed_b200 import synth

    key = (t, k, m)
    if key not in _CPU_SAMPLES:
        x = synth.bf16_round(synth.activations(m, k, seed=0))
        if t == 0:
            _CPU_SAMPLES[key] = (x, synth.fp8_matrix(_CPU_ROWS, k, seed=0))
        else:
            _CPU_SAMPLES[key] = (x, synth.quant_matrix(t, _CPU_ROWS, k, seed=0))
    return _CPU_SAMPLES[key]


def cpu_baseline(budget_s: float = 20.0, batch: int = BATCH):
    """The reference's CPU quantized matmul restated (oracle/rtd_cpu_qmatmul.c: candle's
    QMatMul algorithm -- activations quantized to Q8_K / Q8_0 blocks, integer dots with
    AVX2, f32 accumulation; OpenMP over all host threads) on a row sample of each of the
    seven layer linears at full K and M = batch; the measured seconds per row, times the
    rows of all 80 layers, give the step's CPU time and tokens/s.  Only the oracle calls
    are timed."""
    import oracle

    threads = os.cpu_count() or 1
    per = budget_s / len(LAYER_LINEARS)
    step_s = 0.0
    rows_used = {}
    for name, t, n, k, _, _ in LAYER_LINEARS:
        x, raw = _cpu_sample(t, k, batch)
        row_b = weight_bytes(t, 1, k)
        rows, spent, done = 8, 0.0, 0
        while spent < per:
            t0 = time.perf_counter()
            if t in (oracle.Q4_K, oracle.Q6_K, oracle.Q8_0):
                oracle.cpu_qmatmul(t, raw[: rows * row_b], rows, k, x, threads=threads)
            else:
                oracle.ref_cpu_linear(t, raw[: rows * row_b], rows, k, x, threads=threads)
            dt = time.perf_counter() - t0
            spent += dt
            done += rows
            if dt < 0.25 and rows < _CPU_ROWS:
                rows *= 2
        step_s += N_LAYERS * n * spent / done
        rows_used[name] = done
    return {"value": batch / step_s, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"row samples of the 7 config-3 layer linears at full K and M={batch} "
                      f"(~{budget_s:.0f} s of CPU work), scaled to the 80-layer step; oracle/rtd_cpu_qmatmul.c "
                      f"restating candle-core 0.11 QMatMul's CPU algorithm (x -> Q8_K blocks, AVX2 integer "
                      f"dots, f32 accumulation), OpenMP {threads} threads"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    base = None
    for _ in range(max(args.warmup, 0)):
        cpu_baseline(budget_s=1.0)
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        base = cpu_baseline(budget_s=max(3.5, 60.0 / max(args.steps, 1)))
        vals.append(base["value"])
    wall = time.perf_counter() - t0
    value = statistics.mean(vals)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall * 1e3 / max(args.steps, 1),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": config_dict(args.gpus),
            "cpu_baseline": dict(base, value=value),
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def config_dict(world: int):
    return {"workload": "config-3 decode step: 70B-shaped Qwen2 linears of all 80 layers, batch 64 "
                        "(one token per sequence), tensor parallel over the run's GPUs",
            "model": "config3-qwen2-70b-shaped (random init, Q4_K_M-style)", "layers": N_LAYERS,
            "hidden": HIDDEN, "ffn": FFN, "heads": [N_HEAD, N_KV, HEAD_DIM], "global_batch": BATCH,
            "linears": [f"{n}:{TYPE_NAMES[t]}:{N}x{K}:{sp}" for n, t, N, K, sp, _ in LAYER_LINEARS],
            "parallelism": f"tp{world}: column-parallel q/k/v/gate/up, row-parallel o/down (fused NVLink exchange)",
            "fused_calls": "attn_q + attn_k and ffn_gate + ffn_up each run as one call on row-concatenated weights",
            "activations": "bf16", "weights": "80 device copies of one seeded random-init layer (config-3 "
                                                "block distributions)",
            "l2": f"inputs larger than L2: {step_weight_bytes(world) / 1e9:.1f} GB of weights per rank per step "
                  "vs 126 MB L2",
            "not_in_step": "attention over the KV cache, RMSNorm, RoPE, SwiGLU, embedding and LM head"}


# ---------------------------------------------------------------- the TP decode step
# Linears of one layer that read the same input and share a format run as ONE call on
# row-concatenated weights (GGUF rows are independent, so the concatenation only places
# byte ranges side by side): attn_q + attn_k and ffn_gate + ffn_up.
FUSED = [("attn_qk", ("attn_q", "attn_k")), ("attn_v", ("attn_v",)), ("attn_output", ("attn_output",)),
         ("ffn_gate_up", ("ffn_gate", "ffn_up")), ("ffn_down", ("ffn_down",))]


class TpStack:
    """The linears of every layer, sharded for this rank (same-format siblings fused), and
    the step's buffers."""

    def __init__(self, rank, world, dev, comm, batches):
        import torch
        from runtimed_b200 import _lib, synth
        from runtimed_b200.weights import QMatMul

        self.L = _lib.lib()
        self.rank, self.world, self.dev, self.comm = rank, world, dev, comm
        spec = {n: (i, t, nn, kk, sp, hb) for i, (n, t, nn, kk, sp, hb) in enumerate(LAYER_LINEARS)}
        first = {}
        self.widths = {}
        for fname, parts in FUSED:
            raws, biases, ns_tot, t0, ks0 = [], [], 0, None, None
            for name in parts:
                i, t, n, k, sp, has_b = spec[name]
                ns, ks = shard_shape(n, k, sp, world)
                raws.append(synth.quant_matrix(t, ns, ks, seed=1000 + rank, stream=i))
                if has_b:
                    b = np.random.default_rng(50 + i).normal(0, 0.02, n).astype(np.float32)
                    biases.append(b[rank * ns:(rank + 1) * ns])
                ns_tot += ns
                t0, ks0 = t, ks
            qm = QMatMul(t0, np.concatenate(raws), ns_tot, ks0, device=dev)
            bias = torch.from_numpy(np.concatenate(biases)).to(dev) if biases else None
            first[fname] = (qm, bias)
            self.widths[fname] = ns_tot
        self.layers = []
        for layer in range(N_LAYERS):
            self.layers.append({f: (q if layer == 0 else q.to_device(dev), b) for f, (q, b) in first.items()})
        torch.cuda.synchronize(dev)
        self.nq = N_HEAD * HEAD_DIM // world   # q's columns at the front of attn_qk's output
        self.nf = FFN // world                 # gate's columns at the front of ffn_gate_up's output
        self.bufs = {}
        for b in batches:
            bf = torch.bfloat16
            self.bufs[b] = dict(
                x=torch.from_numpy(synth.activations(b, HIDDEN, seed=rank, stream=3)).to(bf).to(dev),
                qk=torch.empty((b, self.widths["attn_qk"]), dtype=bf, device=dev),
                v=torch.empty((b, self.widths["attn_v"]), dtype=bf, device=dev),
                o=torch.empty((b, HIDDEN), dtype=bf, device=dev),
                gu=torch.empty((b, self.widths["ffn_gate_up"]), dtype=bf, device=dev),
                d=torch.empty((b, HIDDEN), dtype=bf, device=dev))

    def _lin(self, qm, bias, x, ldx, y, m, st):
        from runtimed_b200 import _lib

        rc = self.L.rtd_qlinear(qm.ctx.handle, qm.handle, x.data_ptr(), _lib.DT_BF16, ldx, m,
                                None if bias is None else bias.data_ptr(), y.data_ptr(), _lib.DT_BF16, qm.n, st)
        if rc != 0:
            raise RuntimeError(f"rtd_qlinear status {rc}: {self.L.rtd_last_error(qm.ctx.handle)}")

    def _row(self, qm, x, ldx, y, m, st):
        from runtimed_b200 import _lib

        if self.world == 1:
            return self._lin(qm, None, x, ldx, y, m, st)
        rc = self.L.rtd_tp_qlinear_row(self.comm.handle, qm.handle, x.data_ptr(), _lib.DT_BF16, ldx, m, None,
                                       y.data_ptr(), _lib.DT_BF16, qm.n, st)
        if rc != 0:
            raise RuntimeError(f"rtd_tp_qlinear_row status {rc}: {self.L.rtd_last_error(qm.ctx.handle)}")

    def one(self, name, layer, b, st):
        """One (fused) linear of one layer."""
        B = self.bufs[b]
        qm, bias = self.layers[layer][name]
        if name == "attn_qk":
            self._lin(qm, bias, B["x"], HIDDEN, B["qk"], b, st)
        elif name == "attn_v":
            self._lin(qm, bias, B["x"], HIDDEN, B["v"], b, st)
        elif name == "attn_output":  # reads q's head shard: the front of attn_qk's rows
            self._row(qm, B["qk"], self.widths["attn_qk"], B["o"], b, st)
        elif name == "ffn_gate_up":
            self._lin(qm, bias, B["o"], HIDDEN, B["gu"], b, st)
        else:  # ffn_down reads gate's shard: the front of ffn_gate_up's rows
            self._row(qm, B["gu"], self.widths["ffn_gate_up"], B["d"], b, st)

    def step(self, b, st, layers=None):
        """One decode token for b sequences through every layer's linears."""
        n = N_LAYERS if layers is None else layers
        for layer in range(n):
            for fname, _ in FUSED:
                self.one(fname, layer, b, st)


def _capture(fn, dev):
    import torch

    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn(torch.cuda.current_stream(dev).cuda_stream)
    return g


def _time_graph(g, stream, dev, n: int) -> float:
    """Seconds per replay of n back-to-back replays (CUDA events on the launching stream)."""
    import torch

    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(n):
        g.replay()
    b.record(stream)
    torch.cuda.synchronize(dev)
    return a.elapsed_time(b) * 1e-3 / n


def _max_over_ranks(v: float, dev, world: int) -> float:
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _per_linear(stack, b, stream, dev, world, reps: int = 24):
    """Device time of each (fused) linear call at batch b: a graph of `reps` calls rotating
    over three layers' weight copies (no call re-reads another's weights from L2)."""
    import torch
    import torch.distributed as dist

    spec = {n: (t, nn, kk, sp) for n, t, nn, kk, sp, _ in LAYER_LINEARS}
    out = {}
    for fname, parts in FUSED:
        if world > 1:
            dist.barrier()
        g = _capture(lambda st: [stack.one(fname, r % 3, b, st) for r in range(reps)], dev)
        g.replay()
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        s = _max_over_ranks(_time_graph(g, stream, dev, 5) / reps, dev, world)
        del g
        byts, nk = 0, None
        for name in parts:
            t, n, k, sp = spec[name]
            ns, ks = shard_shape(n, k, sp, world)
            byts += weight_bytes(t, ns, ks) + b * (n if sp == "row" else ns) * 2
            nk = ks
        byts += b * nk * 2
        qm = stack.layers[0][fname][0]
        out[fname] = {"us": s * 1e6, "shard_nk": [qm.n, qm.k], "format": TYPE_NAMES[qm.ggml_type], "bytes": byts,
                      "gbs": byts / s / 1e9}
    return out


def _tp_rowparallel(world, rank, dev, stream, reps: int = 20):
    """The config-3 row-parallel linears (attn_output Q4_K 8192 x 8192, ffn_down Q6_K
    8192 x 28672, K split over the ranks) at M = 1 and 64: the fused call, the unfused GEMV
    plus the library's all-reduce, and the GEMV plus an NCCL all-reduce.  Each path is a
    CUDA graph of `reps` calls (device time per call, max over ranks); each output is
    checked against the unsharded single-GPU linear of the same full weight (rel_l2)."""
    import torch
    import torch.distributed as dist
    from runtimed_b200 import synth
    from runtimed_b200.tp import RowParallelLinear, TpComm
    from runtimed_b200.weights import Context, QMatMul

    comm = TpComm(Context.for_device(dev), rank, world, max_n=HIDDEN)
    out = {"timing": f"CUDA graph of {reps} calls per path, 5 replays, CUDA events, max over ranks",
           "parity": "rel_l2 of each rank's output against the unsharded single-GPU rtd_qlinear (f32 out)"}
    for name, t, n, k in (("attn_output", Q4_K, HIDDEN, HIDDEN), ("ffn_down", Q6_K, HIDDEN, FFN)):
        raw = synth.quant_matrix(t, n, k, seed=77, stream=t)
        full = QMatMul(t, raw, n, k, device=dev)
        rpl = RowParallelLinear.from_full_weight(raw, t, n, k, None, rank, world, comm=comm, device=dev)
        del raw
        ks = k // world
        res = {"shape_nk": [n, k], "format": "Q4_K" if t == Q4_K else "Q6_K", "k_shard": ks}
        for m in (1, 64):
            xf = torch.from_numpy(synth.activations(m, k, seed=9)).to(torch.bfloat16).to(dev)
            xs = xf[:, rank * ks:(rank + 1) * ks].contiguous()
            want = full.forward(xf, out_dtype=torch.float32).double()
            row = {}
            for path, fn in (("fused", rpl.forward), ("ar", rpl.forward_ar), ("nccl", rpl.forward_nccl)):
                got = fn(xs.float()).double()
                torch.cuda.synchronize(dev)
                rel = float(torch.linalg.norm(got - want) / torch.linalg.norm(want))
                rel = _max_over_ranks(rel, dev, world)
                for _ in range(3):
                    fn(xs)
                torch.cuda.synchronize(dev)
                dist.barrier()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    for _ in range(reps):
                        fn(xs)
                g.replay()
                torch.cuda.synchronize(dev)
                dist.barrier()
                s = _max_over_ranks(_time_graph(g, stream, dev, 5) / reps, dev, world)
                del g  # graphs holding NCCL work go before the process group
                row[path] = {"us": round(s * 1e6, 2), "rel_l2": rel}
            row["shard_gbs_fused"] = round(weight_bytes(t, n, ks) / (row["fused"]["us"] * 1e-6) / 1e9, 1)
            res[f"m{m}"] = row
        out[name] = res
        del full, rpl
    torch.cuda.synchronize(dev)
    dist.barrier()
    comm.close()
    return out


# ---------------------------------------------------------------- config-1 sweeps (N = 1)
def _gemv_sweep(dev, stream, rank, peak):
    """The config-1 quantized-linear sweep at decode M = 1: 14 GEMVs (0.74 GB of distinct
    weights per pass), a CUDA graph of the pass, HBM GB/s of algorithmic bytes; the roofline
    of its longest GEMV (a graph of 24 launches over 3 weight copies)."""
    import torch
    from runtimed_b200 import _lib, synth
    from runtimed_b200.weights import Fp8Weight, QMatMul

    L = _lib.lib()
    items = []
    for name, t, n, k in sweep():
        if t == 0:
            w, s = synth.fp8_matrix(n, k, seed=rank, stream=k)
            objs = [Fp8Weight(w, s, k, n, device=dev)]
        else:
            objs = [QMatMul(t, synth.quant_matrix(t, n, k, seed=rank, stream=k), n, k, device=dev)]
            objs += [objs[0].to_device(dev) for _ in range(2)]
        x = torch.from_numpy(synth.bf16_round(synth.activations(1, k, seed=rank, stream=n))).to(torch.bfloat16).to(dev)
        y = torch.empty((1, n), dtype=torch.bfloat16, device=dev)
        items.append(dict(name=name, t=t, n=n, k=k, objs=objs, x=x, y=y, bytes=alg_bytes(t, n, k)))

    def call(it, st, c=0):
        o = it["objs"][c % len(it["objs"])]
        if it["t"] == 0:
            rc = L.rtd_fp8_linear(o.ctx.handle, o.handle, it["x"].data_ptr(), _lib.DT_BF16, it["k"], 1,
                                  it["y"].data_ptr(), _lib.DT_BF16, it["n"], _lib.FP8_W8A16, st)
        else:
            rc = L.rtd_qlinear(o.ctx.handle, o.handle, it["x"].data_ptr(), _lib.DT_BF16, it["k"], 1, None,
                               it["y"].data_ptr(), _lib.DT_BF16, it["n"], st)
        if rc != 0:
            raise RuntimeError(f"sweep {it['name']} {it['n']}x{it['k']}: status {rc}")

    for it in items:
        call(it, stream.cuda_stream)
    torch.cuda.synchronize(dev)
    g = _capture(lambda st: [call(it, st) for it in items], dev)
    for _ in range(3):
        g.replay()
    s = _time_graph(g, stream, dev, 20)
    del g
    step_bytes = sum(it["bytes"] for it in items)
    per = {}
    for it in items:
        if it["t"] == 0:
            continue  # FP8 holds one copy: its per-call figure would re-read L2
        gi = _capture(lambda st: [call(it, st, c) for c in range(24)], dev)
        gi.replay()
        per[f"{it['name']}:{it['n']}x{it['k']}"] = it["bytes"] / (_time_graph(gi, stream, dev, 5) / 24) / 1e9
        del gi
    key = {f"{it['name']}:{it['n']}x{it['k']}": it for it in items}
    dom = max(per, key=lambda kk: key[kk]["bytes"] / per[kk])  # the longest GEMV
    dit = key[dom]
    achieved = per[dom]
    return {"workload": "config-1 sweep at decode M=1: 14 GEMVs (Q4_K/Q6_K/Q8_0/FP8 x (4096,4096), (14336,4096), "
                        "(4096,14336), (151936,896); K=896 Q4_K/Q6_K infeasible), bf16 activations",
            "value_gbs": step_bytes / s / 1e9, "ms_per_pass": s * 1e3, "bytes_per_pass": step_bytes,
            "frac_of_peak": step_bytes / s / 1e9 / peak,
            "roofline": {"bound": "hbm", "kernel": f"qgemv_kernel, {dit['name']} {dit['n']}x{dit['k']} M=1",
                         "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": profile_traffic(f"qgemv_{dit['name'].lower()}_{dit['n']}x{dit['k']}_m1")},
            "per_gemv_gbs": {k2: round(v, 1) for k2, v in per.items()},
            # the layer-shaped GEMVs beside the LM head: the fractions a Q4_K_M decode lives on
            "layer_frac": {k2: round(per[k2] / peak, 3) for k2 in ("Q4_K:4096x4096", "Q4_K:14336x4096",
                                                                   "Q6_K:4096x14336") if k2 in per},
            "timing": "CUDA graph of the 14-GEMV pass (20 replays); per GEMV a graph of 24 launches over 3 "
                      "device copies, CUDA events"}


def _m_sweep(dev, rank, tflops_peak):
    """The rest of the config-1 token counts at (N, K) = (14336, 4096) for every format:
    skinny M = 4, 16, 64 in GB/s of algorithmic bytes (HBM roofline) and prefill M = 512,
    2048 in TFLOP/s (against the measured bf16 burst peak).  Each point is a CUDA graph of
    10 calls over 3 weight copies, 5 replays, CUDA events."""
    import torch
    from runtimed_b200 import _lib, synth
    from runtimed_b200.weights import Fp8Weight, QMatMul

    L = _lib.lib()
    n, k = 14336, 4096
    out = {"shape_nk": [n, k], "timing": "CUDA graph of 10 calls over 3 weight copies, 5 replays, CUDA events",
           "tflops_peak": tflops_peak, "tflops_peak_source": "MEASURED_PEAKS.json bf16_tflops (measured)"}
    stream = torch.cuda.current_stream(dev)
    for name, t in FORMATS:
        objs = []
        for c in range(3):
            if t == 0:
                w, sc = synth.fp8_matrix(n, k, seed=rank + 20 + c, stream=k)
                objs.append(Fp8Weight(w, sc, k, n, device=dev))
            elif c == 0:
                objs.append(QMatMul(t, synth.quant_matrix(t, n, k, seed=rank + 20, stream=k), n, k, device=dev))
            else:
                objs.append(objs[0].to_device(dev))
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
                call(o, stream.cuda_stream)
            torch.cuda.synchronize(dev)
            g = _capture(lambda st: [call(objs[r % 3], st) for r in range(10)], dev)
            for _ in range(2):
                g.replay()
            us = _time_graph(g, stream, dev, 5) * 1e6 / 10
            del g
            if m <= 64:
                gbs = (weight_bytes(t, n, k) + m * k * 2 + m * n * 2) / (us * 1e-6) / 1e9
                row[f"m{m}"] = {"us": round(us, 2), "gbs": round(gbs, 1)}
            else:
                tf = 2.0 * m * n * k / (us * 1e-6) / 1e12
                row[f"m{m}"] = {"us": round(us, 2), "tflops": round(tf, 1),
                                "frac": round(tf / tflops_peak, 3) if tflops_peak else None}
        out[name] = row
        del objs
    out["FP8_W8A8"] = _fp8_w8a8_vs_cublaslt(dev, n, k, tflops_peak)
    out["INT4_MARLIN"] = _marlin_points(dev, n, k)
    return out


def _marlin_points(dev, n, k):
    """INT4 Marlin weights (marlin_gemv.rs: 0.5 byte a weight + a f32 scale a row) at the same
    (N, K), M = 1 and 64, in GB/s of algorithmic bytes; CUDA graph of 10 calls over 3 copies."""
    import torch
    from runtimed_b200 import _lib
    from runtimed_b200.weights import MarlinWeight, repack_marlin_tiles

    L = _lib.lib()
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((n, k)).astype(np.float32) * np.float32(0.02))
    packed, s = repack_marlin_tiles(w, np.abs(w).max(axis=1) / np.float32(7.0))
    objs = [MarlinWeight(packed, s, k, n, device=dev)]
    objs += [objs[0].to_device(dev) for _ in range(2)]
    stream = torch.cuda.current_stream(dev)
    row = {"bytes_per_weight": 0.5}
    for m in (1, 64):
        x = torch.randn(m, k, device=dev).to(torch.bfloat16)
        y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)

        def call(o, st):
            rc = L.rtd_qlinear(o.ctx.handle, o.handle, x.data_ptr(), _lib.DT_BF16, k, m, None, y.data_ptr(),
                               _lib.DT_BF16, n, st)
            if rc != 0:
                raise RuntimeError(f"marlin M={m}: status {rc}")

        for o in objs:
            call(o, stream.cuda_stream)
        torch.cuda.synchronize(dev)
        g = _capture(lambda st: [call(objs[r % 3], st) for r in range(10)], dev)
        for _ in range(2):
            g.replay()
        us = _time_graph(g, stream, dev, 5) * 1e6 / 10
        del g
        gbs = (n * k // 2 + 4 * n + m * k * 2 + m * n * 2) / (us * 1e-6) / 1e9
        row[f"m{m}"] = {"us": round(us, 2), "gbs": round(gbs, 1)}
    del objs
    return row


def _fp8_w8a8_vs_cublaslt(dev, n, k, tflops_peak):
    """FP8 W8A8 (the reference's CUDA semantics: x encoded to E4M3, E4M3 x E4M3 with f32
    accumulation, per-channel scale after) through rtd_fp8_linear -- the kind::f8f6f4 GEMM
    from four tokens on -- beside cuBLASLt's FP8 GEMM (torch._scaled_mm, per-tensor scales)
    on the same shapes; each a CUDA graph of 10 calls over 3 weight copies, 5 replays."""
    import torch
    from runtimed_b200 import _lib, synth
    from runtimed_b200.weights import Fp8Weight

    L = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    objs, mats = [], []
    for c in range(3):
        w, sc = synth.fp8_matrix(n, k, seed=40 + c, stream=k)
        objs.append(Fp8Weight(w, sc, k, n, device=dev))
        mats.append(torch.from_numpy(w).view(torch.float8_e4m3fn).to(dev))
    one = torch.ones((), dtype=torch.float32, device=dev)
    row = {}
    for m in (64, 512, 2048):
        x = torch.randn(m, k, device=dev).to(torch.bfloat16)
        y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        x8 = x.to(torch.float8_e4m3fn)

        def ours(o, st):
            rc = L.rtd_fp8_linear(o.ctx.handle, o.handle, x.data_ptr(), _lib.DT_BF16, k, m, y.data_ptr(),
                                  _lib.DT_BF16, n, _lib.FP8_W8A8, st)
            if rc != 0:
                raise RuntimeError(f"fp8 w8a8 M={m}: status {rc}")

        def lt(wm):
            return torch._scaled_mm(x8, wm.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)

        res = {}
        for label, fn in (("ours", lambda r, st: ours(objs[r % 3], st)), ("cublaslt", lambda r, st: lt(mats[r % 3]))):
            try:
                for r in range(3):
                    fn(r, stream.cuda_stream)
                torch.cuda.synchronize(dev)
                g = _capture(lambda st: [fn(r, st) for r in range(10)], dev)
                g.replay()
                us = _time_graph(g, stream, dev, 5) * 1e6 / 10
                del g
                tf = 2.0 * m * n * k / (us * 1e-6) / 1e12
                res[label] = {"us": round(us, 2), "tflops": round(tf, 1),
                              "frac_bf16_peak": round(tf / tflops_peak, 3) if tflops_peak else None}
            except Exception as e:  # noqa: BLE001 - the comparison arm is reported, not required
                res[label] = {"error": f"{type(e).__name__}: {e}"}
        row[f"m{m}"] = res
    row["note"] = "ours: rtd_fp8_linear W8A8 (E4M3 activations by the reference encoder); cublaslt: " \
                  "torch._scaled_mm E4M3 x E4M3, per-tensor scales (timing comparison only)"
    return row


def _model_decode(dev, steps: int = 128, warm: int = 8):
    """Config 0 end to end (Qwen2-0.5B-shaped, written as a GGUF and
    loaded through the library): batch 1, 128 prompt ids, then `steps` greedy tokens
    with the decode step captured as one CUDA graph (token and position on the device,
    the argmax feeding the next replay), f16 paged KV cache.  Device time of the timed
    replays (CUDA events), after `warm` untimed ones; the restated reference forward
    (oracle/qwen2_ref.py, numpy f32 on the host cores) times a few decode steps beside it."""
    import tempfile

    import torch
    from runtimed_b200 import fixtures
    from runtimed_b200.qwen2 import Qwen2Model

    shape = fixtures.CONFIGS["config0"]
    with tempfile.TemporaryDirectory(prefix="rtd_bench_") as d:
        path = os.path.join(d, "config0.gguf")
        fixtures.write_qwen2_gguf(path, shape, seed=0)
        prompt = list(np.random.default_rng(0).integers(0, shape.vocab, 128))
        model = Qwen2Model(path, device=dev, max_ctx=len(prompt) + steps + warm + 16)
        out, g, replay = model.greedy_graph(prompt, steps + warm)
        for _ in range(warm):
            replay()
        torch.cuda.synchronize(dev)
        stream = torch.cuda.current_stream(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            replay()
        b.record(stream)
        torch.cuda.synchronize(dev)
        s = a.elapsed_time(b) * 1e-3 / steps
        ids = [int(v) for v in out[:8].cpu()]
        del g, model
        torch.cuda.empty_cache()
        # the restated reference forward on the host cores: a few decode steps
        from oracle.qwen2_ref import RefQwen2

        ref = RefQwen2(path)
        logits = ref.forward(prompt, 0)[-1]
        tok, pos, n_cpu = int(np.argmax(logits)), len(prompt), 4
        t0 = time.perf_counter()
        for _ in range(n_cpu):
            logits = ref.forward([tok], pos)[-1]
            tok, pos = int(np.argmax(logits)), pos + 1
        cpu_s = (time.perf_counter() - t0) / n_cpu
    weights = sum(weight_bytes(fixtures.tensor_format(shape, kind, k), n, k)
                  for kind, n, k in fixtures.layer_tensors(shape)) * shape.n_layer + weight_bytes(8, shape.vocab, shape.hidden)
    return {"workload": "config0: Qwen2-0.5B-shaped GGUF (Q8_0 / Q6_K), batch 1, 128-token prompt, greedy decode, "
                        "f16 paged KV cache, decode step captured as a CUDA graph",
            "tokens_per_s": 1.0 / s, "ms_per_token": s * 1e3, "timed_steps": steps, "warm_steps": warm,
            "weight_bytes_per_token": weights, "gbs": weights / s / 1e9, "first_ids": ids,
            "cpu_reference_tokens_per_s": 1.0 / cpu_s, "cpu_reference": f"oracle/qwen2_ref.py (numpy f32, "
                                                                         f"{os.cpu_count()} host threads), {n_cpu} steps"}


def profile_tpstep(b: int, calls: int, layers: int = 4) -> int:
    """`calls` eager config-3 decode steps of `layers` layers at batch b on one GPU (the
    launch-list target: every kernel of a step in order)."""
    import torch

    global N_LAYERS
    N_LAYERS = layers  # the profile covers a few layers; every layer runs the same calls
    dev = torch.device("cuda", 0)
    stack = TpStack(0, 1, dev, None, batches=(b,))
    st = torch.cuda.current_stream(dev).cuda_stream
    for _ in range(calls):
        stack.step(b, st)
    torch.cuda.synchronize(dev)
    print(f"profile-one tpstep:{b}: {calls} steps of {layers} layers ok")
    return 0


def profile_greedy(spec: str, calls: int) -> int:
    """`calls` pairs of one-token LM-head calls (FMT:N:K, bf16 x): the plain GEMV writing the
    logits, then the same GEMV with the greedy pick in its epilogue and no logits."""
    import torch
    from runtimed_b200 import synth
    from runtimed_b200.weights import QMatMul

    name, n, k = spec.split(":")
    t, n, k = dict(FORMATS)[name], int(n), int(k)
    dev = torch.device("cuda", 0)
    qm = QMatMul(t, synth.quant_matrix(t, n, k, seed=0, stream=k), n, k, device=dev)
    x = torch.from_numpy(synth.bf16_round(synth.activations(1, k, seed=0))).to(torch.bfloat16).to(dev)
    for _ in range(calls):
        y = qm.forward(x, out_dtype=torch.float32)
        ids = qm.greedy(x)
    torch.cuda.synchronize(dev)
    assert int(ids[0]) == int(torch.argmax(y[0]))
    print(f"profile-one greedy:{spec}: {calls} pairs ok")
    return 0


def profile_one(spec: str, calls: int) -> int:
    """Run `calls` bf16 calls of one linear (FMT:N:K, or FMT:N:K:M for M tokens; M = 1 by
    default), or of every config-1 sweep GEMV in order ("sweep"), eagerly, and exit: the
    target of the ncu captures summarised under profiles/."""
    import torch
    from runtimed_b200 import _lib, synth
    from runtimed_b200.weights import Fp8Weight, QMatMul

    m = 1
    if spec.startswith("tpstep"):
        return profile_tpstep(int(spec.split(":")[1]) if ":" in spec else BATCH, calls)
    if spec.startswith("greedy:"):
        return profile_greedy(spec[len("greedy:"):], calls)
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
    print(f"profile-one {spec}: {calls} calls of {len(items)} linears ok")
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--profile-one", default=None, metavar="FMT:N:K[:M]|sweep|tpstep[:B]|greedy:FMT:N:K",
                    help="only run a few eager calls of one linear or of the config-1 sweep (ncu target), "
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

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180), device_id=dev)

    from runtimed_b200 import _lib
    from runtimed_b200.tp import TpComm
    from runtimed_b200.weights import Context

    L = _lib.lib()
    stream = torch.cuda.current_stream(dev)
    peak, peak_kind, tflops_peak = read_peaks()
    comm = TpComm(Context.for_device(dev), rank, world, max_n=HIDDEN) if world > 1 else None
    stack = TpStack(rank, world, dev, comm, batches=(BATCH, 1))
    w_bytes = step_weight_bytes(world)

    for b in (BATCH, 1):  # first calls configure kernel attributes outside capture
        stack.step(b, stream.cuda_stream, layers=1)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    n0 = L.rtd_kernel_launches()
    g64 = _capture(lambda st: stack.step(BATCH, st), dev)
    launches_per_step = L.rtd_kernel_launches() - n0
    g1 = _capture(lambda st: stack.step(1, st), dev)
    for _ in range(max(args.warmup, 3)):
        g64.replay()
        g1.replay()
    torch.cuda.synchronize(dev)

    # ---- timed region (device time, CUDA events, max over ranks).  nvidia-smi samples
    # every 200 ms: the timed steps sit inside a window of the same load (an untimed
    # pre-roll of about a second and a short post-roll).
    if world > 1:
        dist.barrier()
    step_s = max(1e-5, _time_graph(g64, stream, dev, 2))
    roll = max(1, int(1.0 / step_s))
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        clk.wait_first_sample()
        for _ in range(roll):
            g64.replay()
        e0.record(stream)
        for _ in range(args.steps):
            g64.replay()
        e1.record(stream)
        for _ in range(max(1, roll // 2)):
            g64.replay()
        torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms_max = _max_over_ranks(e0.elapsed_time(e1), dev, world)
    value = BATCH * args.steps / (ms_max * 1e-3)
    if world > 1:
        dist.barrier()
    s1 = _max_over_ranks(_time_graph(g1, stream, dev, max(5, args.steps // 2)), dev, world)

    # ---- roofline: the step's dominant kernel and the whole step
    per64 = _per_linear(stack, BATCH, stream, dev, world)
    per1 = _per_linear(stack, 1, stream, dev, world)
    dom = max(per64, key=lambda n: per64[n]["us"])
    d = per64[dom]
    fmt = d["format"].lower().replace("_", "")
    step_gbs = w_bytes / (ms_max * 1e-3 / args.steps) / 1e9
    roofline = {"bound": "hbm", "achieved": d["gbs"], "peak": peak, "unit": "GB/s", "frac": d["gbs"] / peak,
                # up to 64 tokens run the skinny GEMM (decoded weights in tensor memory)
                "traffic": profile_traffic(f"qgemm_ts_{fmt}_{d['shard_nk'][0]}x{d['shard_nk'][1]}_m{BATCH}"),
                "kernel": f"{dom} ({d['format']}, rank shard {d['shard_nk'][0]}x{d['shard_nk'][1]}, M={BATCH}): "
                          f"skinny tensor-core GEMM (qgemm_ts_kernel) with its prep and fixup",
                "launch_us": d["us"], "duration_source": "CUDA events around a graph of 24 back-to-back calls over "
                                                         "3 layers' weight copies",
                "peak_source": f"MEASURED_PEAKS.json hbm_gbs ({peak_kind})",
                "step": {"weight_bytes_per_rank": w_bytes, "gbs": step_gbs, "frac": step_gbs / peak},
                "per_linear_b64": {n: {"us": round(v["us"], 2), "gbs": round(v["gbs"], 1)} for n, v in per64.items()},
                "per_linear_b1": {n: {"us": round(v["us"], 2), "gbs": round(v["gbs"], 1)} for n, v in per1.items()}}

    # ---- end to end through the public API: every step copies the 64 hidden states in
    # from pinned host memory, replays the step, and reads the last layer's outputs back
    B = stack.bufs[BATCH]
    hx = torch.empty(B["x"].shape, dtype=torch.bfloat16).pin_memory()
    hx.copy_(B["x"].cpu())
    hy = torch.empty(B["d"].shape, dtype=torch.bfloat16).pin_memory()
    e2e_steps = max(3, args.steps // 2)

    def e2e_step():
        B["x"].copy_(hx, non_blocking=True)
        g64.replay()
        hy.copy_(B["d"], non_blocking=True)
        stream.synchronize()

    for _ in range(2):
        e2e_step()
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    b.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = _max_over_ranks(a.elapsed_time(b), dev, world)
    e2e_val = BATCH * e2e_steps / (e2e_ms * 1e-3)
    if not torch.equal(hy.to(dev), B["d"]):
        raise RuntimeError("e2e: host copy of the outputs differs from the device")
    del g64, g1

    tp = None
    if world > 1:
        # measured after the headline; a failure is reported in its own object (every
        # rank runs the same steps, so a failure is seen by all of them)
        try:
            tp = _tp_rowparallel(world, rank, dev, stream)
        except Exception as e:  # noqa: BLE001 - reported in the JSON line
            tp = {"error": f"{type(e).__name__}: {e}"}
            torch.cuda.synchronize(dev)
    del stack
    gemv = _gemv_sweep(dev, stream, rank, peak) if world == 1 else None
    try:
        model = _model_decode(dev) if world == 1 else None
    except Exception as e:  # noqa: BLE001 - reported in the JSON line
        model = {"error": f"{type(e).__name__}: {e}"}
    msweep = _m_sweep(dev, rank, tflops_peak) if world == 1 else None
    cpu = cpu_baseline() if (rank == 0 and world == 1) else None
    if comm is not None:
        torch.cuda.synchronize(dev)
        dist.barrier()
        comm.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16 activations; f16 tensor-core products of the decoded weights, f32 accumulate",
            "data": "synthetic (seeded random-init weights and hidden states)", "config": config_dict(world),
            "decode_b1": {"tokens_per_s": 1.0 / s1, "ms_per_step": s1 * 1e3,
                          "gbs": w_bytes / s1 / 1e9, "frac": w_bytes / s1 / 1e9 / peak},
            "roofline": roofline, "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": int(hx.numel() * 2),
                    "d2h_bytes_per_step": int(hy.numel() * 2),
                    "path": "per step: pinned-host copy of the 64 hidden states in, replay of the step's CUDA graph "
                            "of C-ABI calls, pinned-host copy of the last layer's outputs out, host wait"},
            "gpu_launches": int(launches_per_step) * args.steps,
            "launches_per_step": int(launches_per_step),
            "tp": tp, "gemv_sweep": gemv, "m_sweep": msweep, "model_decode": model, "clocks": clk.summary()}
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
