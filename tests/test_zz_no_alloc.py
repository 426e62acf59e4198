"""The allocation-free linear, rtd_qlinear_noalloc, against rtd_qlinear.

Both run the same kernels. The allocation-free entry takes its scratch from a fixed
array inside the library instead of a context workspace. Two calls in a row, with
different activations, must each match the context-based entry point on the same
input. A call whose staging would not fit the fixed scratch is refused before any
launch. This file is collected last, and it must also pass alone in a fresh process
(the first call on a device sets the scratch up).
"""
import ctypes

import numpy as np
import pytest

from runtimed_b200 import _lib, synth

pytestmark = pytest.mark.gpu

RTOL_EXACT = 2e-5  # the GEMV tests' bound for exact-product kernels (f32 rounding only)
DT = {"f32": _lib.DT_F32, "f16": _lib.DT_F16, "bf16": _lib.DT_BF16}


def rel_l2(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))


def _torch_dtype(torch, name):
    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[name]


def _call(L, fn, qm, x, y, xdt, bias=None):
    torch = pytest.importorskip("torch")
    stream = torch.cuda.current_stream().cuda_stream
    M, K = x.shape
    N = y.shape[1]
    bp = None if bias is None else bias.data_ptr()
    if fn == "ctx":
        return L.rtd_qlinear(qm.ctx.handle, qm.handle, x.data_ptr(), DT[xdt], K, M, bp, y.data_ptr(),
                             _lib.DT_F32, N, stream)
    return L.rtd_qlinear_noalloc(qm.handle, x.data_ptr(), DT[xdt], K, M, bp, y.data_ptr(), _lib.DT_F32, N, stream)


@pytest.mark.parametrize("t", [12, 14, 8])
@pytest.mark.parametrize("xdt,M", [("bf16", 1), ("f16", 3), ("f32", 2)])
def test_noalloc_matches_qlinear_twice(t, xdt, M):
    torch = pytest.importorskip("torch")
    from runtimed_b200.weights import QMatMul

    N, K = 200, 2048
    qm = QMatMul(t, synth.quant_matrix(t, N, K, seed=7, stream=t), N, K)
    bias = torch.from_numpy(np.random.default_rng(3).normal(0, 0.02, N).astype(np.float32)).cuda()
    L = _lib.lib()
    for call in range(2):  # two calls in a row share the one scratch array
        x = torch.from_numpy(synth.activations(M, K, seed=100 + call, stream=t)).to(_torch_dtype(torch, xdt)).cuda()
        want = torch.empty((M, N), dtype=torch.float32, device="cuda")
        got = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        assert _call(L, "ctx", qm, x, want, xdt, bias) == 0
        rc = _call(L, "noalloc", qm, x, got, xdt, bias)
        assert rc == 0, L.rtd_last_error(None)
        torch.cuda.synchronize()
        assert rel_l2(got.cpu().numpy(), want.cpu().numpy()) <= RTOL_EXACT


def test_noalloc_rejects_oversized_staging():
    torch = pytest.importorskip("torch")
    from runtimed_b200.weights import QMatMul

    # f32 rows this long are staged through the scratch (hi and lo f16 halves per
    # token): 4 columns of 262400 halves exceed the fixed 1 MiB
    N, K, M = 16, 262400, 2
    qm = QMatMul(12, synth.quant_matrix(12, N, K, seed=1), N, K)
    L = _lib.lib()
    x = torch.zeros((M, K), dtype=torch.float32, device="cuda")
    y = torch.full((M, N), 7.0, dtype=torch.float32, device="cuda")
    rc = _call(L, "noalloc", qm, x, y, "f32")
    assert rc == _lib.RTD_ERR_WORKSPACE
    msg = L.rtd_last_error(None)
    msg = msg.decode() if isinstance(msg, bytes) else str(msg)
    assert "static scratch" in msg
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())  # nothing was launched
