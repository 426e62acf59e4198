"""Pins the CPU oracle before anything is checked against it.

Known-answer tests restated from the reference's own unit tests (values copied
as data, file:line cited), plus the committed golden fixtures made by
tests/golden/make_golden.py from independent decoders (gguf-py, torch).
"""
import math
import os

import numpy as np
import pytest

import oracle
from runtimed_b200 import synth

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "golden.npz"))


# ---- crates/runtimed-gguf/src/quant/dequant.rs:152-159 (f16_corners)
def test_f16_corners():
    assert oracle.f16_to_f32(0x3C00) == 1.0
    assert oracle.f16_to_f32(0xBC00) == -1.0
    assert oracle.f16_to_f32(0x0000) == 0.0
    assert math.isinf(oracle.f16_to_f32(0x7C00))
    assert abs(oracle.f16_to_f32(0x0001) - 2.0 ** -24) < 1e-30


def test_f16_all_bit_patterns_match_numpy():
    bits = np.arange(65536, dtype=np.uint32)
    ours = np.array([oracle.f16_to_f32(int(b)) for b in bits[::7]], dtype=np.float32)
    ref = bits[::7].astype(np.uint16).view(np.float16).astype(np.float32)
    finite = np.isfinite(ref)
    assert np.array_equal(ours[finite].view(np.uint32), ref[finite].view(np.uint32))
    assert np.array_equal(np.isnan(ours), np.isnan(ref))


# ---- crates/runtimed-gguf/src/quant/dequant.rs:161-169 (q8_0_scales_ints)
def test_q8_0_kat():
    block = bytes([0x00, 0x3C]) + bytes(range(32))
    out = oracle.dequant_block(oracle.Q8_0, block)
    assert list(out) == [float(i) for i in range(32)]


# ---- crates/runtimed-gguf/src/quant/dequant_k.rs:117-129 (q4_k_nibbles_and_high_bits)
def test_q4_k_kat():
    block = bytes([0x00, 0x3C, 0x00, 0x00]) + bytes([65] + [1] * 11) + bytes([0x11] * 128)
    out = oracle.dequant_block(oracle.Q4_K, block)
    assert out.size == 256
    assert np.all(out[0:32] == 1.0)
    assert np.all(out[32:64] == 1.0)
    assert np.all(out[128:160] == 17.0)


# ---- crates/runtimed-gguf/src/quant/dequant_k.rs:154-178 (q6_k_signed_values_and_scales)
def test_q6_k_kat():
    block = bytearray(208) + bytearray([0x00, 0x3C])
    block[192:208] = bytes([1] * 16)
    out = oracle.dequant_block(oracle.Q6_K, bytes(block))
    assert np.all(out == -32.0)
    bq = bytearray(block)
    bq[0] = 0x11
    bq[128] = 0xFF
    bq[192:200] = bytes([1, 2, 3, 4, 5, 6, 7, 8])
    oq = oracle.dequant_block(oracle.Q6_K, bytes(bq))
    assert oq[0] == 17.0 and oq[32] == 48.0 and oq[64] == 85.0 and oq[96] == 112.0
    bl = bytearray(block)
    bl[192:200] = bytes([1, 2, 3, 4, 5, 6, 7, 8])
    bl[16] = 0x11
    ol = oracle.dequant_block(oracle.Q6_K, bytes(bl))
    assert ol[16] == -62.0


# ---- crates/runtimed-gguf/src/quant/dtype.rs:75-94 (block_geometry)
def test_block_geometry():
    assert oracle.block_geometry(8) == (32, 34)
    assert oracle.block_geometry(10) == (256, 84)
    assert oracle.block_geometry(11) == (256, 110)
    assert oracle.block_geometry(12) == (256, 144)
    assert oracle.block_geometry(13) == (256, 176)
    assert oracle.block_geometry(14) == (256, 210)
    assert oracle.block_geometry(0) == (1, 4)
    assert oracle.block_geometry(99) is None


# ---- crates/runtimed-gguf/src/quant/dequant.rs:83-95 (dispatcher errors)
def test_dequant_tensor_errors():
    raw = synth.quant_matrix(oracle.Q4_K, 1, 256)
    assert oracle.dequant_tensor(oracle.Q4_K, raw, 255)[0] == oracle.NOT_MULTIPLE
    assert oracle.dequant_tensor(oracle.Q4_K, raw[:100], 256)[0] == oracle.TRUNCATED
    assert oracle.dequant_tensor(99, raw, 256)[0] == oracle.UNSUPPORTED
    assert oracle.dequant_tensor(oracle.Q4_K, raw, 0)[0] == oracle.OK


@pytest.mark.parametrize("name,t", [("Q4_K", 12), ("Q6_K", 14), ("Q8_0", 8)])
def test_dequant_matches_gguf_py_golden(name, t):
    blocks = GOLDEN[f"{name}_blocks"]
    want = GOLDEN[f"{name}_dequant"]
    elems, _ = synth.BLOCK[t]
    rc, got = oracle.dequant_tensor(t, blocks.reshape(-1), blocks.shape[0] * elems)
    assert rc == oracle.OK
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("name,t", [("Q4_K", 12), ("Q6_K", 14), ("Q8_0", 8)])
def test_gemv_matches_golden(name, t):
    N, K, M = GOLDEN[f"{name}_gemv_shape"]
    y = oracle.qgemv_f64(t, GOLDEN[f"{name}_gemv_raw"], int(N), int(K), GOLDEN[f"{name}_gemv_x"],
                         GOLDEN[f"{name}_gemv_bias"])
    want = GOLDEN[f"{name}_gemv_y"]
    assert y.shape == (M, N)
    assert np.linalg.norm(y - want) <= 1e-12 * np.linalg.norm(want)


# ---- crates/runtimed-model/src/weights/load_safetensors.rs:14-29 vs torch float8_e4m3fn
def test_e4m3_lut_matches_torch():
    lut = oracle.fp8_lut()
    ref = GOLDEN["e4m3_lut_torch"]
    nan = (np.arange(256) & 0x7F) == 0x7F
    assert np.all(np.isnan(lut[nan]))
    assert np.array_equal(lut[~nan].view(np.uint32), ref[~nan].view(np.uint32))


# ---- crates/runtimed-model/src/weights/fp8_weight.rs:117-133 (byte values)
def test_e4m3_byte_kat():
    assert oracle.fp8_to_f32(0x38) == 1.0
    assert oracle.fp8_to_f32(0x40) == 2.0
    assert oracle.fp8_to_f32(0x30) == 0.5
    assert oracle.fp8_to_f32(0x44) == 3.0


# ---- load_safetensors.rs:53-69: the encoder
def test_e4m3_encoder_non_ties_match_torch():
    got = oracle.f32_to_fp8(GOLDEN["e4m3_enc_x"])
    assert np.array_equal(got, GOLDEN["e4m3_enc_code"])


def test_e4m3_encoder_ties_go_to_lower_magnitude_and_saturate():
    lut = oracle.fp8_lut()
    pos = lut[:127]
    mids = ((pos[1:126].astype(np.float64) + pos[2:127]) / 2).astype(np.float32)
    codes = oracle.f32_to_fp8(mids)
    assert np.array_equal(codes, np.arange(1, 126, dtype=np.uint8))
    codes_neg = oracle.f32_to_fp8(-mids)
    assert np.array_equal(codes_neg, np.arange(1, 126, dtype=np.uint8) | 0x80)
    assert list(oracle.f32_to_fp8([448.0, 1e9, -1e9, float("nan"), -0.0, 0.0])) == [0x7E, 0x7E, 0xFE, 0x7F, 0x80, 0x00]
    # the smallest subnormal is 2^-9; half of it is a tie with zero -> zero
    assert list(oracle.f32_to_fp8([2.0 ** -10, 2.0 ** -10 * 1.01])) == [0x00, 0x01]


# ---- crates/runtimed-model/src/ops/fp8_gemm.rs:197-207 (cpu_fp8_gemm_matches_reference)
def test_fp8_gemm_cpu_kat():
    x = np.array([[1.0, 2.0], [3.0, 4.0]], np.float32)
    w = np.array([[0x38, 0x00], [0x00, 0x40]], np.uint8)  # [[1, 0], [0, 2]]
    s = np.array([2.0, 0.5], np.float32)
    y = oracle.fp8_gemm_cpu_f64(x, w, s, 2, 2)
    assert list(y.ravel()) == [2.0, 2.0, 6.0, 4.0]


# ---- crates/runtimed-model/src/weights/fp8_weight.rs:117-133 (forward == x . dequant^T)
def test_fp8_weight_forward_kat():
    w = np.array([0x38, 0x40, 0x30, 0x44], np.uint8).reshape(2, 2)
    s = np.array([2.0, 0.5], np.float32)
    x = np.array([[1.5, -2.0]], np.float32)
    y = oracle.fp8_gemm_cpu_f64(x, w, s, 2, 2)
    deq = np.array([[1.0, 2.0], [0.5, 3.0]]) * s[:, None]
    assert np.allclose(y, x @ deq.T, atol=1e-3)


def test_w8a8_semantics_match_explicit_formula():
    g = np.random.Generator(np.random.PCG64(5))
    N, K, M = 8, 64, 3
    w, s = synth.fp8_matrix(N, K, seed=5)
    x = g.standard_normal((M, K)).astype(np.float32) * 3
    lut = oracle.fp8_lut().astype(np.float64)
    xq = lut[oracle.f32_to_fp8(x)].reshape(M, K)
    want = (xq @ lut[w].T) * s[None, :]
    got = oracle.fp8_gemm_w8a8_f64(x, w, s, N, K)
    assert np.allclose(got, want, rtol=1e-12, atol=1e-12)


def test_ref_cpu_linear_close_to_f64_oracle():
    N, K, M = 40, 512, 2
    for t in (12, 14, 8):
        raw = synth.quant_matrix(t, N, K, seed=11, stream=t)
        x = synth.activations(M, K, seed=11)
        y32 = oracle.ref_cpu_linear(t, raw, N, K, x, threads=2)
        y64 = oracle.qgemv_f64(t, raw, N, K, x)
        assert np.linalg.norm(y32 - y64) <= 1e-5 * np.linalg.norm(y64)
