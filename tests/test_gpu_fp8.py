"""GPU parity of the FP8 E4M3 path and of the Weights operator mirror.

- The device encoder must equal the reference encoder bit for bit
  (crates/runtimed-model/src/weights/load_safetensors.rs:53-69).
- W8A16 follows the CPU semantics x . (LUT(W) * s)^T
  (crates/runtimed-model/src/ops/fp8_gemm.rs:55-74).
- W8A8 follows the reference's CUDA semantics: x encoded to E4M3 unscaled, then
  the channel scale (fp8_gemm.rs:96-101,180-186).
- Outputs are gated at relative L2 <= 1e-3, and asserted at the exact-product bound
  where products are exact (E4M3 -> f16 is exact).
"""
import numpy as np
import pytest

import oracle
from runtimed_b200 import _lib, synth

pytestmark = pytest.mark.gpu

RTOL = 1e-3
RTOL_EXACT = 2e-5


def rel_l2(got, want):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))


def _encode_inputs():
    lut = oracle.fp8_lut()
    fin = np.sort(np.unique(lut[np.isfinite(lut)]))
    mids = (fin[:-1] + fin[1:]) / 2  # exact ties between neighbouring codes
    g = np.random.Generator(np.random.PCG64(17))
    parts = [fin, mids, np.nextafter(mids, np.inf), np.nextafter(mids, -np.inf)]
    parts += [g.standard_normal(4096) * s for s in (1e-3, 0.05, 1.0, 30.0, 600.0)]
    parts.append(np.array([0.0, -0.0, 448.0, 449.0, 464.0, 1e6, -1e6, np.inf, -np.inf, np.nan, 2.0 ** -9,
                           2.0 ** -10, 3 * 2.0 ** -11, 1e-30, -1e-30]))
    x = np.concatenate([np.asarray(p, dtype=np.float64) for p in parts]).astype(np.float32)
    return np.concatenate([x, -x])


def test_fp8_encode_bit_exact():
    torch = pytest.importorskip("torch")
    from runtimed_b200.weights import fp8_encode

    x = _encode_inputs()
    got = fp8_encode(torch.from_numpy(x).cuda()).cpu().numpy()
    want = oracle.f32_to_fp8(x)
    assert np.array_equal(got, want)


def _fp8(N, K, seed, per_tensor=False):
    w, s = synth.fp8_matrix(N, K, seed=seed)
    if per_tensor:
        s = np.array([float(np.max(s))], np.float32)
    return w, s


@pytest.mark.parametrize("M", [1, 2, 5, 17, 33])
@pytest.mark.parametrize("xdt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("per_tensor", [False, True])
def test_fp8_linear_w8a16_parity(M, xdt, per_tensor):
    torch = pytest.importorskip("torch")
    from runtimed_b200.weights import Fp8Weight

    N, K = 72, 1024
    w, s = _fp8(N, K, seed=M, per_tensor=per_tensor)
    fw = Fp8Weight(w, s, K, N)
    dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[xdt]
    xt = torch.from_numpy(synth.activations(M, K, seed=M, stream=9)).to(dt)
    want = oracle.fp8_gemm_cpu_f64(xt.float().numpy(), w, s, N, K)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    x = xt.cuda()
    L = _lib.lib()
    st = L.rtd_fp8_linear(fw.ctx.handle, fw.handle, x.data_ptr(), {"bf16": 2, "f16": 1, "f32": 0}[xdt], K, M,
                          y.data_ptr(), _lib.DT_F32, N, _lib.FP8_W8A16, torch.cuda.current_stream().cuda_stream)
    assert st == 0
    # M >= 4 runs the tensor-core GEMM: E4M3 weights stay exact, f32 activations round to f16
    assert rel_l2(y.cpu().numpy(), want) <= (RTOL_EXACT if M <= 3 else RTOL)


@pytest.mark.parametrize("M", [1, 3, 16])
@pytest.mark.parametrize("K", [1024, 1000])
def test_fp8_linear_w8a8_parity(M, K):
    torch = pytest.importorskip("torch")
    from runtimed_b200.weights import Fp8Weight

    N = 96
    w, s = _fp8(N, K, seed=K + M)
    fw = Fp8Weight(w, s, K, N)
    x = synth.activations(M, K, seed=M, stream=11) * 4.0
    want = oracle.fp8_gemm_w8a8_f64(x, w, s, N, K)
    got = fw.forward(torch.from_numpy(x).cuda(), mode="w8a8").cpu().numpy()
    assert got.dtype == np.float32  # f32 in -> f32 out (fp8_gemm.rs:106)
    assert rel_l2(got, want) <= (RTOL_EXACT if M <= 3 else RTOL)


def test_fp8_ragged_k_and_vocab_shape():
    torch = pytest.importorskip("torch")
    from runtimed_b200.weights import Fp8Weight

    for (N, K) in [(37, 1000), (151936, 896)]:
        w, s = _fp8(N, K, seed=3)
        fw = Fp8Weight(w, s, K, N)
        x = synth.bf16_round(synth.activations(1, K, seed=2))
        want = oracle.fp8_gemm_cpu_f64(x, w, s, N, K)
        got = fw.forward(torch.from_numpy(x).to(torch.bfloat16).cuda()).float().cpu().numpy()
        assert rel_l2(got, want) <= RTOL_EXACT


def test_fp8_reference_known_answers():
    """fp8_gemm.rs:197-207 and fp8_weight.rs:117-133 through the device path."""
    torch = pytest.importorskip("torch")
    from runtimed_b200.weights import Fp8Weight

    fw = Fp8Weight(np.array([[0x38, 0x00], [0x00, 0x40]], np.uint8), np.array([2.0, 0.5], np.float32), 2, 2)
    y = fw.forward(torch.tensor([[1.0, 2.0], [3.0, 4.0]], device="cuda")).cpu().numpy()
    assert y.tolist() == [[2.0, 2.0], [6.0, 4.0]]
    fw = Fp8Weight(np.array([[0x38, 0x40], [0x30, 0x44]], np.uint8), np.array([2.0, 0.5], np.float32), 2, 2)
    y = fw.forward(torch.tensor([[1.5, -2.0]], device="cuda")).cpu().numpy()
    deq = np.array([[1.0, 2.0], [0.5, 3.0]]) * np.array([2.0, 0.5])[:, None]
    assert np.allclose(y, np.array([[1.5, -2.0]]) @ deq.T, rtol=0, atol=0)


def test_fp8_output_dtype_and_shape_errors():
    torch = pytest.importorskip("torch")
    from runtimed_b200.errors import ShapeError
    from runtimed_b200.weights import Fp8Weight

    w, s = _fp8(16, 64, seed=1)
    fw = Fp8Weight(w, s, 64, 16)
    x16 = torch.randn(2, 3, 64, device="cuda").half()
    y = fw.forward(x16)
    assert y.dtype == torch.float16 and tuple(y.shape) == (2, 3, 16)
    want = oracle.fp8_gemm_cpu_f64(x16.float().cpu().numpy().reshape(6, 64), w, s, 16, 64)
    assert rel_l2(y.float().cpu().numpy().reshape(6, 16), want) <= RTOL
    with pytest.raises(ShapeError):
        fw.forward(torch.randn(1, 63, device="cuda"))
    with pytest.raises(ShapeError):
        Fp8Weight(w[:, :32], s, 64, 16)
    with pytest.raises(ShapeError):
        Fp8Weight(w, s[:8], 64, 16)


def test_weights_mirror_routes_and_errors():
    """Weights::linear / linear_bias / embed / get / resident_bytes
    (crates/runtimed-model/src/weights/{linear_layer,embed_layer,store}.rs)."""
    torch = pytest.importorskip("torch")
    from runtimed_b200.errors import MissingWeight, ModelError
    from runtimed_b200.weights import Fp8Weight, QMatMul, Weights

    N, K = 48, 512
    raw = synth.quant_matrix(12, N, K, seed=4)
    qm = QMatMul(12, raw, N, K)
    w, s = _fp8(N, K, seed=4)
    fw = Fp8Weight(w, s, K, N)
    bias = torch.from_numpy(np.random.default_rng(1).normal(0, 0.02, N).astype(np.float32)).cuda()
    ws = Weights(map={"b": bias}, q_map={"q": qm, "q_alias": qm}, fp8_map={"f": fw})
    x = torch.from_numpy(synth.activations(1, K, seed=4)).cuda()

    yq = ws.linear(x, "q").cpu().numpy()
    assert rel_l2(yq, oracle.qgemv_f64(12, raw, N, K, x.cpu().numpy())) <= RTOL_EXACT
    yb = ws.linear_bias(x, "q", "b").cpu().numpy()
    assert rel_l2(yb, yq + bias.cpu().numpy()[None, :]) <= RTOL_EXACT
    yf = ws.linear(x, "f").cpu().numpy()
    assert rel_l2(yf, oracle.fp8_gemm_cpu_f64(x.cpu().numpy(), w, s, N, K)) <= RTOL_EXACT

    e = ws.embed("q", [3, 0, 47]).cpu().numpy()
    deq = ws.get("q").cpu().numpy()
    assert e.shape == (1, 3, K)
    assert np.array_equal(e[0], deq[[3, 0, 47]])
    # q_map entries sharing one QMatMul count once; fp8 bytes = codes + scales
    assert ws.resident_bytes() == N * 4 + raw.size + w.size + 4 * s.size
    for bad in (lambda: ws.linear(x, "nope"), lambda: ws.get("nope"), lambda: ws.embed("nope", [0])):
        with pytest.raises(MissingWeight):
            bad()
    with pytest.raises(ModelError):
        ws.embed("q", [N])


def test_weights_linear_dense_scale_key_lookup():
    # Weights::linear_dense on an E4M3 map entry: the scale comes from the first of
    # "{name}.scale", "{name}_scale", "{name}.weight_scale_inv", else ones
    # (crates/runtimed-model/src/weights/linear_layer.rs:78-86); the GEMM runs the
    # reference CUDA semantics (W8A8)
    import torch
    from runtimed_b200.weights import Weights

    N, K, M = 48, 256, 3
    w, s = synth.fp8_matrix(N, K, seed=8)
    x = synth.bf16_round(synth.activations(M, K, seed=9))
    wt = torch.from_numpy(w).view(torch.float8_e4m3fn)
    for key in (".scale", "_scale", ".weight_scale_inv", None):
        m = {"blk.w": wt}
        if key is not None:
            m["blk.w" + key] = torch.from_numpy(s)
        W = Weights(device="cuda:0", map=m)
        y = W.linear(torch.from_numpy(x).cuda(), "blk.w").cpu().numpy()
        sc = s if key is not None else np.ones(N, np.float32)
        want = oracle.fp8_gemm_w8a8_f64(x, w, sc, N, K)
        assert rel_l2(y, want) <= 1e-3, key
