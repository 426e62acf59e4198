"""The allocation-free linear, rtd_qlinear_noalloc, against the CPU oracle and rtd_qlinear.

Some callers cannot allocate device memory while they run: code that works inside
another allocator's fixed device-memory budget, where an extra cudaMalloc can fail or
stall every stream on the device.  rtd_qlinear_noalloc serves them: it dispatches like
rtd_qlinear but takes its scratch from a fixed array inside the library instead of a
context workspace.  Two calls in a row, with different activations, must each match
the oracle within the path's bar and match rtd_qlinear on the same input.  The cases
cover one-launch GEMV calls, a multi-pass GEMV call (f32 rows at M = 3 run as 2 + 1
tokens, both passes on the one scratch array) and the tensor-core GEMM (M = 5).  A call
whose staging would not fit is refused before any launch, and the status word of the
scratch is read through rtd_noalloc_check_status.  This file is collected last, and it
must also pass alone in a fresh process (the first call on a device sets the scratch up).
"""
import numpy as np
import pytest

import oracle
from runtimed_b200 import _lib, synth

pytestmark = pytest.mark.gpu

RTOL_EXACT = 2e-5  # exact-product GEMV passes (f32 rounding only)
RTOL_GEMM = 1e-3   # the tensor-core GEMM rounds decoded weights once to f16
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
@pytest.mark.parametrize("xdt,M", [("bf16", 1), ("f16", 3), ("f32", 2), ("f32", 3), ("bf16", 5)])
def test_noalloc_matches_oracle_and_qlinear_twice(t, xdt, M):
    torch = pytest.importorskip("torch")
    from runtimed_b200.weights import QMatMul

    N, K = 200, 2048
    raw = synth.quant_matrix(t, N, K, seed=7, stream=t)
    qm = QMatMul(t, raw, N, K)
    bias_np = np.random.default_rng(3).normal(0, 0.02, N).astype(np.float32)
    bias = torch.from_numpy(bias_np).cuda()
    tol = RTOL_GEMM if M >= 4 else RTOL_EXACT
    L = _lib.lib()
    for call in range(2):  # two calls in a row share the one scratch array
        xt = torch.from_numpy(synth.activations(M, K, seed=100 + call, stream=t)).to(_torch_dtype(torch, xdt))
        want = oracle.qgemv_f64(t, raw, N, K, xt.float().numpy()) + bias_np[None, :]
        x = xt.cuda()
        ref = torch.empty((M, N), dtype=torch.float32, device="cuda")
        got = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        assert _call(L, "ctx", qm, x, ref, xdt, bias) == 0
        rc = _call(L, "noalloc", qm, x, got, xdt, bias)
        assert rc == 0, L.rtd_last_error(None)
        assert L.rtd_noalloc_check_status(0, torch.cuda.current_stream().cuda_stream) == 0
        assert rel_l2(got.cpu().numpy(), want) <= tol
        assert rel_l2(got.cpu().numpy(), ref.cpu().numpy()) <= tol


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
    assert L.rtd_noalloc_check_status(0, None) == 0
