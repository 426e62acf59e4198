"""The timed CPU baseline: candle-core 0.11's QMatMul CPU algorithm restated in
oracle/rtd_cpu_qmatmul.c (behind Weights::linear, crates/runtimed-model/src/weights/
linear_layer.rs:45-52).  CPU only.

  * its activation quantizers follow the published Q8_K / Q8_0 rules (checked against a
    numpy statement of them, zero blocks included);
  * its integer arithmetic is exact: the result equals the float64 product of the
    dequantized weights with the DEQUANTIZED 8-bit activations to f32 rounding, and the
    AVX2 and plain-C forms agree bit for bit;
  * against the exact product with the original activations it is off by the 8-bit
    activation rounding only (below 2e-2 relative on Gaussian activations).
"""
import numpy as np
import pytest

import oracle
from runtimed_b200 import synth


def rel_l2(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))


def _q8k_numpy(x):
    x = np.asarray(x, np.float32)
    i = int(np.argmax(np.abs(x)))  # the first value of largest magnitude
    if x[i] == 0:
        return np.zeros(256, np.int8), np.float32(0)
    iscale = np.float32(-128.0) / x[i]
    q = np.rint((iscale * x).astype(np.float32))
    return np.minimum(q, 127).astype(np.int8), np.float32(1.0) / iscale


def _q8_0_numpy(x):
    x = np.asarray(x, np.float32)
    amax = np.float32(np.abs(x).max())
    d = amax / np.float32(127.0)
    idv = np.float32(1.0) / d if d != 0 else np.float32(0.0)
    v = (x * idv).astype(np.float32)
    q = np.sign(v) * np.floor(np.abs(v) + np.float32(0.5))  # half away from zero
    return q.astype(np.int8), np.float32(np.float16(d))


def test_activation_quantizers_follow_the_published_rules():
    rng = np.random.default_rng(5)
    x = rng.normal(0, 1, 1024).astype(np.float32)
    x[300] = -7.5  # block 1's value of largest magnitude, negative: code -128, d > 0
    x[512:768] = 0.0  # a zero block
    codes, scales, bsums = oracle.cpu_quantize_x(oracle.Q4_K, x)
    for b in range(4):
        q, d = _q8k_numpy(x[256 * b:256 * (b + 1)])
        assert np.array_equal(codes[256 * b:256 * (b + 1)], q), b
        assert scales[b] == d, b
    assert np.array_equal(bsums, codes.reshape(-1, 16).astype(np.int32).sum(1))
    assert codes[300] == -128 and scales[1] > 0  # d = max / -128, of the opposite sign to max
    codes, scales, _ = oracle.cpu_quantize_x(oracle.Q8_0, x)
    for b in range(32):
        q, d = _q8_0_numpy(x[32 * b:32 * (b + 1)])
        assert np.array_equal(codes[32 * b:32 * (b + 1)], q), b
        assert scales[b] == d, b


@pytest.mark.parametrize("t,N,K", [(oracle.Q4_K, 131, 1024), (oracle.Q6_K, 130, 2048), (oracle.Q8_0, 129, 896)])
@pytest.mark.parametrize("M", [1, 5])
def test_integer_arithmetic_is_exact(t, N, K, M):
    raw = synth.quant_matrix(t, N, K, seed=7, stream=t)
    x = synth.bf16_round(synth.activations(M, K, seed=8))
    qk = 32 if t == oracle.Q8_0 else 256
    xd = []
    for r in x:
        c, s, _ = oracle.cpu_quantize_x(t, r)
        xd.append(c.astype(np.float64) * np.repeat(s.astype(np.float64), qk))
    want_q = oracle.qgemv_f64(t, raw, N, K, np.array(xd))  # f64 dot of the dequantized codes
    got = oracle.cpu_qmatmul(t, raw, N, K, x, threads=2)
    plain = oracle.cpu_qmatmul(t, raw, N, K, x, threads=3, simd=False)
    assert np.array_equal(got.view(np.uint32), plain.view(np.uint32))
    assert rel_l2(got, want_q) <= 1e-6
    assert rel_l2(got, oracle.qgemv_f64(t, raw, N, K, x)) <= 2e-2


def test_rejects_other_types_and_ragged_k():
    x = np.zeros((1, 100), np.float32)
    with pytest.raises(ValueError):
        oracle.cpu_qmatmul(oracle.Q4_K, np.zeros(144, np.uint8), 1, 100, x)
    with pytest.raises(ValueError):
        oracle.cpu_qmatmul(30, np.zeros(200, np.uint8), 1, 100, x)
