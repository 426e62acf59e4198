"""GPU parity of the quantized linear path against the CPU oracle.

Dequantization is compared bit for bit (memcmp of the f32 words); GEMV/GEMM
outputs are gated at relative L2 <= 1e-3 (the tolerance the reference's own
north-star check states), and the measured error is asserted far tighter where
the kernels are exact in their products (RTOL_EXACT).
"""
import os

import numpy as np
import pytest

import oracle
from runtimed_b200 import synth

pytestmark = pytest.mark.gpu

RTOL = 1e-3          # relative L2 gate on GEMV / GEMM outputs
RTOL_EXACT = 2e-5    # what exact-product kernels actually reach (f32 rounding only)
GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))
FORMATS = [("Q4_K", 12), ("Q6_K", 14), ("Q8_0", 8)]


def _torch():
    import torch

    return torch


def rel_l2(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))


def make_qm(t, N, K, seed=0, stream=0):
    from runtimed_b200.weights import QMatMul

    raw = synth.quant_matrix(t, N, K, seed=seed, stream=stream)
    return QMatMul(t, raw, N, K), raw


@pytest.mark.parametrize("name,t", FORMATS)
@pytest.mark.parametrize("N,K", [(1, 256), (16, 512), (37, 768), (130, 2048)])
def test_dequant_bit_exact(name, t, N, K):
    qm, raw = make_qm(t, N, K, seed=N + K, stream=t)
    got = qm.dequantize().cpu().numpy()
    rc, want = oracle.dequant_tensor(t, raw, N * K)
    assert rc == oracle.OK
    assert np.array_equal(got.reshape(-1).view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("name,t", FORMATS)
def test_dequant_golden_blocks(name, t):
    blocks = GOLDEN[f"{name}_blocks"]
    elems, _ = synth.BLOCK[t]
    from runtimed_b200.weights import QMatMul

    qm = QMatMul(t, blocks.reshape(-1), blocks.shape[0], elems)
    got = qm.dequantize().cpu().numpy().reshape(-1)
    assert np.array_equal(got.view(np.uint32), GOLDEN[f"{name}_dequant"].view(np.uint32))


@pytest.mark.parametrize("name,t", FORMATS)
def test_gemv_golden(name, t):
    torch = _torch()
    from runtimed_b200.weights import QMatMul

    N, K, M = (int(v) for v in GOLDEN[f"{name}_gemv_shape"])
    qm = QMatMul(t, GOLDEN[f"{name}_gemv_raw"], N, K)
    x = torch.from_numpy(GOLDEN[f"{name}_gemv_x"]).to(torch.bfloat16).cuda()
    b = torch.from_numpy(GOLDEN[f"{name}_gemv_bias"]).cuda()
    y = qm.forward(x, bias=b, out_dtype=torch.float32).cpu().numpy()
    assert rel_l2(y, GOLDEN[f"{name}_gemv_y"]) <= RTOL_EXACT


@pytest.mark.parametrize("name,t", FORMATS)
@pytest.mark.parametrize("M", [1, 2, 3, 4, 5, 8, 9, 16, 17, 33])
@pytest.mark.parametrize("xdt", ["bf16", "f16", "f32"])
def test_gemv_parity_small(name, t, M, xdt):
    torch = _torch()
    N, K = 72, 1024
    qm, raw = make_qm(t, N, K, seed=M, stream=t)
    x32 = synth.activations(M, K, seed=M, stream=50 + t)
    dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[xdt]
    xt = torch.from_numpy(x32).to(dt)
    want = oracle.qgemv_f64(t, raw, N, K, xt.float().numpy())
    y = qm.forward(xt.cuda(), out_dtype=torch.float32).cpu().numpy()
    err = rel_l2(y, want)
    # M >= 4 runs the tensor-core GEMM, whose weights are rounded once to f16
    assert err <= (RTOL_EXACT if M <= 3 else RTOL), err


@pytest.mark.parametrize("name,t", FORMATS)
@pytest.mark.parametrize("N,K", [(4096, 4096), (14336, 4096), (4096, 14336)])
def test_gemv_parity_config1_shapes(name, t, N, K):
    torch = _torch()
    qm, raw = make_qm(t, N, K, seed=1, stream=t)
    for M in (1, 3, 4):
        x = synth.bf16_round(synth.activations(M, K, seed=2, stream=M))
        want = oracle.qgemv_f64(t, raw, N, K, x)
        y = qm.forward(torch.from_numpy(x).to(torch.bfloat16).cuda(), out_dtype=torch.float32).cpu().numpy()
        # M >= 4 runs the tensor-core GEMM (weights rounded once to f16)
        assert rel_l2(y, want) <= (RTOL_EXACT if M <= 3 else RTOL)


def test_gemv_parity_vocab_q8_0():
    torch = _torch()
    N, K = 151936, 896
    qm, raw = make_qm(8, N, K, seed=3)
    x = synth.bf16_round(synth.activations(1, K, seed=3))
    want = oracle.qgemv_f64(8, raw, N, K, x)
    y = qm.forward(torch.from_numpy(x).to(torch.bfloat16).cuda(), out_dtype=torch.float32).cpu().numpy()
    assert rel_l2(y, want) <= RTOL_EXACT


@pytest.mark.parametrize("name,t", FORMATS)
def test_bias_strides_and_output_dtypes(name, t):
    torch = _torch()
    import ctypes
    from runtimed_b200 import _lib

    N, K, M = 48, 512, 3
    qm, raw = make_qm(t, N, K, seed=7, stream=t)
    x = synth.activations(M, K, seed=7)
    bias = (synth.rng(7, 9).standard_normal(N) * 0.02).astype(np.float32)
    want = oracle.qgemv_f64(t, raw, N, K, x, bias)
    # strided x and y through the raw C ABI
    xs = torch.zeros((M, K + 64), dtype=torch.float32, device="cuda")
    xs[:, :K] = torch.from_numpy(x).cuda()
    ys = torch.full((M, N + 16), 7.0, dtype=torch.float32, device="cuda")
    bt = torch.from_numpy(bias).cuda()
    st = _lib.lib().rtd_qlinear(qm.ctx.handle, qm.handle, xs.data_ptr(), _lib.DT_F32, K + 64, M, bt.data_ptr(),
                                ys.data_ptr(), _lib.DT_F32, N + 16, torch.cuda.current_stream().cuda_stream)
    assert st == 0
    ys = ys.cpu().numpy()
    assert rel_l2(ys[:, :N], want) <= RTOL_EXACT
    assert np.all(ys[:, N:] == 7.0)
    for odt in (torch.float16, torch.bfloat16):
        y = qm.forward(torch.from_numpy(x).cuda(), bias=bt, out_dtype=odt).float().cpu().numpy()
        tol = 1e-3 if odt == torch.float16 else 8e-3
        assert rel_l2(y, want) <= tol


def test_split_k_many_calls_stay_consistent():
    """Long rows use split-K with self-re-arming counters: repeated calls must agree."""
    torch = _torch()
    N, K = 256, 14336
    qm, raw = make_qm(12, N, K, seed=5)
    x = torch.from_numpy(synth.activations(2, K, seed=5)).cuda()
    first = qm.forward(x).cpu().numpy()
    for _ in range(5):
        assert np.array_equal(qm.forward(x).cpu().numpy(), first)
    want = oracle.qgemv_f64(12, raw, N, K, x.cpu().numpy())
    assert rel_l2(first, want) <= RTOL_EXACT


def test_edge_cases_empty_and_zero_k():
    torch = _torch()
    from runtimed_b200.weights import QMatMul

    qm, _ = make_qm(12, 32, 256)
    y = qm.forward(torch.zeros((0, 256), device="cuda"))
    assert tuple(y.shape) == (0, 32)
    q0 = QMatMul(12, b"", 5, 0)
    b = torch.arange(5, dtype=torch.float32, device="cuda")
    y0 = q0.forward(torch.zeros((2, 0), device="cuda"), bias=b)
    assert y0.cpu().tolist() == [[0, 1, 2, 3, 4]] * 2


def test_errors_mirror_reference():
    torch = _torch()
    from runtimed_b200 import GgufError, ShapeError
    from runtimed_b200.weights import QMatMul

    with pytest.raises(GgufError):
        QMatMul(12, b"\x00" * 144, 1, 255)  # not a multiple of 256 (dequant.rs:87-91)
    with pytest.raises(GgufError):
        QMatMul(12, b"\x00" * 100, 1, 256)  # truncated (dequant.rs:92-95)
    with pytest.raises(GgufError):
        QMatMul(2, b"\x00" * 18, 1, 32)     # Q4_0 is off this path
    qm, _ = make_qm(12, 16, 256)
    with pytest.raises(ShapeError):
        qm.forward(torch.zeros((1, 512), device="cuda"))


@pytest.mark.parametrize("name,t", FORMATS)
def test_embed_rows_bit_exact(name, t):
    torch = _torch()
    from runtimed_b200.weights import Weights

    N, K = 300, 512
    qm, raw = make_qm(t, N, K, seed=11, stream=t)
    w = Weights(q_map={"token_embd.weight": qm})
    ids = [5, 0, 299, 17, 5]
    y = w.embed("token_embd.weight", ids)
    assert tuple(y.shape) == (1, len(ids), K)
    rc, full = oracle.dequant_tensor(t, raw, N * K)
    want = full.reshape(N, K)[ids]
    assert np.array_equal(y[0].cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert tuple(w.embed("token_embd.weight", []).shape) == (1, 0, K)
    # Weights::candidate_weights (embed_layer.rs:59-82): the same rows, [n, K]
    cw = w.candidate_weights("token_embd.weight", ids)
    assert tuple(cw.shape) == (len(ids), K)
    assert np.array_equal(cw.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert tuple(w.candidate_weights("token_embd.weight", []).shape) == (0, K)


def test_embed_out_of_range_raises_status():
    torch = _torch()
    from runtimed_b200 import ConfigError

    qm, _ = make_qm(14, 10, 256)
    y = qm.embedding(torch.tensor([1, 10], dtype=torch.int32))
    with pytest.raises(ConfigError):
        qm.ctx.check_device_status()
    assert np.all(y[1].cpu().numpy() == 0)
    qm.ctx.check_device_status()  # the status word was cleared


@pytest.mark.parametrize("name,t", FORMATS)
def test_to_device_copy_is_identical(name, t):
    # rtd_qweight_to_device: a second device copy that dequantizes and multiplies to the
    # same bits as the original, and stays valid after the original is freed
    torch = _torch()
    qm, raw = make_qm(t, 100, 512, seed=3, stream=t)
    cp = qm.to_device("cuda:0")
    x = torch.from_numpy(synth.activations(2, 512, seed=4)).cuda()
    y0 = qm.forward(x)
    d0 = qm.dequantize()
    qm.free()
    y1 = cp.forward(x)
    assert torch.equal(y0, y1)
    assert torch.equal(d0, cp.dequantize())
    assert cp.storage_size_in_bytes() == len(raw)


def test_row_views_of_a_fused_upload():
    # rtd_qweight_rows: q | k | v uploaded as one matrix, each addressed by its rows, give
    # the same bits as separate uploads; the view shares the parent's memory
    torch = _torch()
    from runtimed_b200.weights import QMatMul

    K = 512
    parts = [synth.quant_matrix(8, n, K, seed=n, stream=8) for n in (96, 32, 48)]
    fused = QMatMul(8, np.concatenate(parts), 176, K)
    x = torch.from_numpy(synth.activations(2, K, seed=5)).cuda()
    row = 0
    yf = fused.forward(x)
    for raw, n in zip(parts, (96, 32, 48)):
        view = fused.rows(row, n)
        alone = QMatMul(8, raw, n, K)
        assert torch.equal(view.forward(x), alone.forward(x))
        assert torch.equal(yf[:, row:row + n], alone.forward(x))
        assert view.device_bytes() == 0 and view.storage_size_in_bytes() == len(raw)
        row += n
    with pytest.raises(Exception):
        fused.rows(8, 16)  # a view must start on a 16-row tile
