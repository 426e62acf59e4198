"""Tensor-core (tcgen05) GEMM path: calls with four or more tokens.

Weights are decoded in shared memory to f16 (the reference dequantisation formulas
in f32, rounded once) and multiplied on the 5th-generation tensor cores with f32
accumulation in tensor memory, so outputs are gated at the north-star relative L2
of 1e-3 against the f64 oracle.
"""
import numpy as np
import pytest

import oracle
from runtimed_b200 import synth

pytestmark = pytest.mark.gpu

RTOL = 1e-3
FORMATS = [("Q4_K", 12), ("Q6_K", 14), ("Q8_0", 8)]


def rel_l2(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))


@pytest.mark.parametrize("name,t", FORMATS)
@pytest.mark.parametrize("M", [5, 16, 64, 200, 512])
def test_gemm_parity(name, t, M):
    import torch
    from runtimed_b200.weights import QMatMul

    N, K = 200, 2048  # N: one full and one partial 128-row CTA tile
    raw = synth.quant_matrix(t, N, K, seed=M, stream=t)
    qm = QMatMul(t, raw, N, K)
    x = synth.bf16_round(synth.activations(M, K, seed=M, stream=3))
    y = qm.forward(torch.from_numpy(x).to(torch.bfloat16).cuda(), out_dtype=torch.float32).cpu().numpy()
    assert rel_l2(y, oracle.qgemv_f64(t, raw, N, K, x)) <= RTOL


@pytest.mark.parametrize("M", [7, 130])
def test_gemm_fp8_parity(M):
    import torch
    from runtimed_b200.weights import Fp8Weight

    N, K = 136, 1000  # ragged K: a zero-padded trailing group
    w, s = synth.fp8_matrix(N, K, seed=M)
    fw = Fp8Weight(w, s, K, N)
    x = synth.activations(M, K, seed=M)
    for mode, ref in (("w8a16", oracle.fp8_gemm_cpu_f64), ("w8a8", oracle.fp8_gemm_w8a8_f64)):
        y = fw.forward(torch.from_numpy(x).cuda(), mode=mode).cpu().numpy()
        assert rel_l2(y, ref(x, w, s, N, K)) <= RTOL, mode


def test_gemm_bias_strides_dtypes_and_determinism():
    import torch
    from runtimed_b200 import _lib
    from runtimed_b200.weights import QMatMul

    N, K, M = 300, 1024, 40
    raw = synth.quant_matrix(12, N, K, seed=2)
    qm = QMatMul(12, raw, N, K)
    x = synth.activations(M, K, seed=2)
    bias = (synth.rng(2, 5).standard_normal(N) * 0.02).astype(np.float32)
    want = oracle.qgemv_f64(12, raw, N, K, x, bias)
    xs = torch.zeros((M, K + 32), dtype=torch.float32, device="cuda")
    xs[:, :K] = torch.from_numpy(x).cuda()
    ys = torch.full((M, N + 8), 7.0, dtype=torch.float32, device="cuda")
    bt = torch.from_numpy(bias).cuda()
    L = _lib.lib()
    outs = []
    for _ in range(2):
        st = L.rtd_qlinear(qm.ctx.handle, qm.handle, xs.data_ptr(), _lib.DT_F32, K + 32, M, bt.data_ptr(),
                           ys.data_ptr(), _lib.DT_F32, N + 8, torch.cuda.current_stream().cuda_stream)
        assert st == 0
        outs.append(ys.cpu().numpy().copy())
    assert np.array_equal(outs[0], outs[1])
    assert rel_l2(outs[0][:, :N], want) <= RTOL
    assert np.all(outs[0][:, N:] == 7.0)
    for odt, tol in ((torch.float16, RTOL), (torch.bfloat16, 8e-3)):
        y = qm.forward(torch.from_numpy(x).cuda(), bias=bt, out_dtype=odt).float().cpu().numpy()
        assert rel_l2(y, want) <= tol


def test_gemm_prefill_shape():
    """Config-1-sized prefill chunk: M = 512 tokens, K = 4096."""
    import torch
    from runtimed_b200.weights import QMatMul

    N, K, M = 1024, 4096, 512
    raw = synth.quant_matrix(12, N, K, seed=9)
    qm = QMatMul(12, raw, N, K)
    x = synth.bf16_round(synth.activations(M, K, seed=9))
    y = qm.forward(torch.from_numpy(x).to(torch.bfloat16).cuda(), out_dtype=torch.float32).cpu().numpy()
    assert rel_l2(y, oracle.qgemv_f64(12, raw, N, K, x)) <= RTOL


def test_gemm_staging_paths():
    """Activation staging: rows whose stride is not a multiple of 16 bytes (element
    loads), f16 input, and K past what a staging thread holds in registers (the row
    is read a second time)."""
    import torch
    from runtimed_b200 import _lib
    from runtimed_b200.weights import QMatMul

    N, K, M = 64, 33024, 6
    raw = synth.quant_matrix(12, N, K, seed=5)
    qm = QMatMul(12, raw, N, K)
    x16 = synth.activations(M, K, seed=5).astype(np.float16)
    want = oracle.qgemv_f64(12, raw, N, K, x16.astype(np.float32))
    ld = K + 3
    xs = torch.zeros((M, ld), dtype=torch.float16, device="cuda")
    xs[:, :K] = torch.from_numpy(x16).cuda()
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    L = _lib.lib()
    st = L.rtd_qlinear(qm.ctx.handle, qm.handle, xs.data_ptr(), _lib.DT_F16, ld, M, None, y.data_ptr(),
                       _lib.DT_F32, N, torch.cuda.current_stream().cuda_stream)
    assert st == 0
    assert rel_l2(y.cpu().numpy(), want) <= RTOL
    xa = torch.from_numpy(x16).cuda()  # aligned rows: 16-byte loads, same result bits
    ya = qm.forward(xa, out_dtype=torch.float32)
    assert torch.equal(ya, y)


@pytest.mark.parametrize("M", [9, 300])
def test_gemm_fp8_ragged_k(M):
    import torch
    from runtimed_b200.weights import Fp8Weight

    N, K = 72, 1003  # K % 8 != 0: the row tail is staged element by element
    w, s = synth.fp8_matrix(N, K, seed=M + 1)
    fw = Fp8Weight(w, s, K, N)
    x = synth.bf16_round(synth.activations(M, K, seed=M + 1))
    xt = torch.from_numpy(x).to(torch.bfloat16).cuda()
    for mode, ref in (("w8a16", oracle.fp8_gemm_cpu_f64), ("w8a8", oracle.fp8_gemm_w8a8_f64)):
        y = fw.forward(xt, mode=mode).float().cpu().numpy()
        assert rel_l2(y, ref(x, w, s, N, K)) <= RTOL, mode


_SWEEP_CACHE = {}


def _sweep_weight(t, N, K):
    """One device weight per (format, shape), shared by the sweep tests below."""
    key = (t, N, K)
    if key not in _SWEEP_CACHE:
        from runtimed_b200.weights import Fp8Weight, QMatMul

        _SWEEP_CACHE.clear()  # one shape resident at a time
        if t == 0:
            w, s = synth.fp8_matrix(N, K, seed=31, stream=K)
            _SWEEP_CACHE[key] = (Fp8Weight(w, s, K, N), (w, s))
        else:
            raw = synth.quant_matrix(t, N, K, seed=31, stream=K)
            _SWEEP_CACHE[key] = (QMatMul(t, raw, N, K), raw)
    return _SWEEP_CACHE[key]


def _sampled_rows(N, n=96):
    rows = np.unique(np.linspace(0, N - 1, n).astype(np.int64))
    return np.concatenate([rows, [N - 1]]) if rows[-1] != N - 1 else rows


@pytest.mark.parametrize("name,t", FORMATS + [("FP8", 0)])
@pytest.mark.parametrize("N,K", [(14336, 4096), (4096, 14336)])
@pytest.mark.parametrize("M", [16, 64, 512, 2048])
def test_gemm_parity_config1_sweep_points(name, t, N, K, M):
    # the bench's m_sweep points at full size: the whole [M, N] output is computed on the
    # GPU and a spread of 96 rows (first and last included) is checked against the oracle
    import torch

    obj, host = _sweep_weight(t, N, K)
    x = synth.bf16_round(synth.activations(M, K, seed=M, stream=K))
    xt = torch.from_numpy(x).to(torch.bfloat16).cuda()
    rows = _sampled_rows(N)
    if t == 0:
        y = obj.forward(xt.float())
        w, s = host
        want = oracle.fp8_gemm_cpu_f64(x, np.ascontiguousarray(w[rows]), np.ascontiguousarray(s[rows]),
                                       len(rows), K)
    else:
        y = obj.forward(xt, out_dtype=torch.float32)
        elems, bb = synth.BLOCK[t]
        row_bytes = (K // elems) * bb
        sub = np.ascontiguousarray(host.reshape(N, row_bytes)[rows]).reshape(-1)
        want = oracle.qgemv_f64(t, sub, len(rows), K, x)
    got = y[:, torch.from_numpy(rows).cuda()].cpu().numpy()
    assert np.isfinite(y.cpu().numpy()).all()
    assert rel_l2(got, want) <= RTOL


@pytest.mark.parametrize("name,t", [("Q6_K", 14), ("Q8_0", 8)])
def test_lm_head_vocab_152064(name, t):
    # the 152064-row LM head of the 7B- and 70B-shaped configs (K = 3584), sampled rows,
    # at decode (GEMV, M = 1) and speculative-verify (GEMM, M = 5) token counts
    import torch
    from runtimed_b200.weights import QMatMul

    N, K = 152064, 3584
    raw = synth.quant_matrix(t, N, K, seed=11, stream=t)
    qm = QMatMul(t, raw, N, K)
    rows = _sampled_rows(N, 128)
    elems, bb = synth.BLOCK[t]
    sub = np.ascontiguousarray(raw.reshape(N, (K // elems) * bb)[rows]).reshape(-1)
    del raw
    for M in (1, 5):
        x = synth.bf16_round(synth.activations(M, K, seed=12))
        y = qm.forward(torch.from_numpy(x).to(torch.bfloat16).cuda(), out_dtype=torch.float32)
        want = oracle.qgemv_f64(t, sub, len(rows), K, x)
        got = y[:, torch.from_numpy(rows).cuda()].cpu().numpy()
        assert rel_l2(got, want) <= (RTOL if M >= 4 else 2e-5), M


_TWO_CTA_CHILD = r'''
import json, sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
import oracle
from runtimed_b200 import synth
from runtimed_b200.weights import Fp8Weight, QMatMul
out = {}
for t in (12, 14, 8, 0):
    N, K = 1000, 2048
    for M in (5, 17, 40, 64):
        x = synth.bf16_round(synth.activations(M, K, seed=M, stream=t))
        if t == 0:
            w, s = synth.fp8_matrix(N, K, seed=M)
            y = Fp8Weight(w, s, K, N).forward(torch.from_numpy(x).cuda()).cpu().numpy()
            want = oracle.fp8_gemm_cpu_f64(x, w, s, N, K)
        else:
            raw = synth.quant_matrix(t, N, K, seed=M, stream=t)
            y = QMatMul(t, raw, N, K).forward(torch.from_numpy(x).to(torch.bfloat16).cuda(),
                                             out_dtype=torch.float32).cpu().numpy()
            want = oracle.qgemv_f64(t, raw, N, K, x)
        out[f"{t}:{M}"] = float(np.linalg.norm(y - want) / np.linalg.norm(want))
print(json.dumps(out))
'''


@pytest.mark.parametrize("dw", ["8", "16"])
def test_gemm_both_cta_configurations(dw):
    # the GEMM's two shapes of CTA -- sixteen decode warps alone on an SM, or eight with a
    # second CTA beside it -- forced in a child process (RTD_GEMM_DW is read once), every
    # format at skinny token counts against the oracle
    import json
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, RTD_GEMM_DW=dw)
    r = subprocess.run([sys.executable, "-c", _TWO_CTA_CHILD, root], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    errs = json.loads(r.stdout.strip().splitlines()[-1])
    assert max(errs.values()) <= RTOL, errs


@pytest.mark.parametrize("M", [4, 40, 512])
def test_fp8_w8a8_tensor_core_path(M):
    # W8A8 from four tokens on runs tcgen05.mma.kind::f8f6f4 on the E4M3 codes themselves
    # (no decode); E4M3 x E4M3 products are exact in f32, so the result sits at f32
    # accumulation error from the restated reference semantics
    import torch
    from runtimed_b200.weights import Fp8Weight

    N, K = 300, 1000 + 24  # ragged K: a zero-padded trailing group
    w, s = synth.fp8_matrix(N, K, seed=M)
    x = synth.activations(M, K, seed=M + 1)
    fw = Fp8Weight(w, s, K, N)
    for dt in (torch.float32, torch.bfloat16):
        xt = torch.from_numpy(x).to(dt)
        y = fw.forward(xt.cuda(), mode="w8a8").float().cpu().numpy()
        want = oracle.fp8_gemm_w8a8_f64(xt.float().numpy(), w, s, N, K)
        assert rel_l2(y, want) <= 2e-6, dt


# The rank shards of the config-3 (70B-shaped) decoder's linears at 2, 4 and 8 GPUs:
# column-parallel attn_q+k / attn_v / ffn_gate+up split N, row-parallel attn_output /
# ffn_down split K.  The 8-GPU shards are the smallest shapes the tensor-parallel step runs
# (a 128-row attn_v shard is one row tile shared by eight CTAs of the skinny GEMM).
_TP_SHARDS = sorted({
    (name, t, n, k)
    for w in (2, 4, 8)
    for name, t, n, k in [("attn_qk", 12, (8192 + 1024) // w, 8192), ("attn_v", 14, 1024 // w, 8192),
                          ("ffn_gate_up", 12, 2 * 28672 // w, 8192), ("attn_output", 12, 8192, 8192 // w),
                          ("ffn_down", 14, 8192, 28672 // w)]
})


@pytest.mark.parametrize("M", [1, 64])
@pytest.mark.parametrize("name,t,N,K", _TP_SHARDS)
def test_config3_tp_shard_shapes(name, t, N, K, M):
    import torch
    from runtimed_b200.weights import QMatMul

    key = ("tp", t, N, K)
    if key not in _SWEEP_CACHE:
        _SWEEP_CACHE.clear()  # one shard resident at a time
        raw = synth.quant_matrix(t, N, K, seed=N + K, stream=t)
        _SWEEP_CACHE[key] = (QMatMul(t, raw, N, K), raw)
    qm, raw = _SWEEP_CACHE[key]
    x = synth.bf16_round(synth.activations(M, K, seed=M, stream=K))
    y = qm.forward(torch.from_numpy(x).to(torch.bfloat16).cuda(), out_dtype=torch.float32)
    rows = _sampled_rows(N, 64)
    elems, bb = synth.BLOCK[t]
    sub = np.ascontiguousarray(raw.reshape(N, (K // elems) * bb)[rows]).reshape(-1)
    want = oracle.qgemv_f64(t, sub, len(rows), K, x)
    got = y[:, torch.from_numpy(rows).cuda()].cpu().numpy()
    assert np.isfinite(y.cpu().numpy()).all()
    assert rel_l2(got, want) <= (2e-5 if M == 1 else RTOL)
