"""CPU oracle for the quantized-linear hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import this package.  The product
(``runtimed_b200`` and ``libruntimed_b200.so``) never imports, links or calls it.

It wraps ``oracle/liboracle.so``, a C restatement of the reference's own CPU
arithmetic (every function in ``rtd_oracle.c`` cites the reference file:line it
follows), and ``rtd_cpu_qmatmul.c``, the reference's CPU quantized matmul (candle's
8-bit activation blocks and integer dots) restated as the timed CPU baseline.  The
library is built by ``make -C oracle`` (``__graft_entry__.build()`` runs that).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

Q8_0, Q4_K, Q6_K = 8, 12, 14
F32, F16, BF16 = 0, 1, 30
OK, UNSUPPORTED, NOT_MULTIPLE, TRUNCATED = 0, 1, 2, 3


def build() -> str:
    """Compile liboracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or any(
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, src))
            for src in ("rtd_oracle.c", "rtd_cpu_qmatmul.c")
        ):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        c_u8p = ctypes.POINTER(ctypes.c_uint8)
        c_fp = ctypes.POINTER(ctypes.c_float)
        c_dp = ctypes.POINTER(ctypes.c_double)
        L.rtdo_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.rtdo_f16_to_f32.restype = ctypes.c_float
        L.rtdo_block_geometry.argtypes = [ctypes.c_uint32, ctypes.POINTER(ctypes.c_uint64),
                                          ctypes.POINTER(ctypes.c_uint64)]
        L.rtdo_block_geometry.restype = ctypes.c_int
        for name in ("rtdo_dequant_q8_0_block", "rtdo_dequant_q4_k_block", "rtdo_dequant_q6_k_block"):
            getattr(L, name).argtypes = [c_u8p, c_fp]
            getattr(L, name).restype = None
        L.rtdo_dequant_tensor.argtypes = [ctypes.c_uint32, c_u8p, ctypes.c_uint64, ctypes.c_uint64, c_fp]
        L.rtdo_dequant_tensor.restype = ctypes.c_int
        L.rtdo_qgemv_f64.argtypes = [ctypes.c_uint32, c_u8p, ctypes.c_uint64, ctypes.c_int64,
                                     ctypes.c_int64, c_fp, ctypes.c_int64, c_fp, c_dp]
        L.rtdo_qgemv_f64.restype = ctypes.c_int
        L.rtdo_ref_cpu_linear.argtypes = [ctypes.c_uint32, c_u8p, ctypes.c_int64, ctypes.c_int64,
                                          c_fp, ctypes.c_int64, c_fp, ctypes.c_int]
        L.rtdo_ref_cpu_linear.restype = ctypes.c_int
        L.rtdo_fp8_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        L.rtdo_fp8_e4m3_to_f32.restype = ctypes.c_float
        L.rtdo_f32_to_fp8_e4m3.argtypes = [ctypes.c_float]
        L.rtdo_f32_to_fp8_e4m3.restype = ctypes.c_uint8
        L.rtdo_f32_to_fp8_e4m3_array.argtypes = [c_fp, ctypes.c_int64, c_u8p]
        L.rtdo_f32_to_fp8_e4m3_array.restype = None
        for name in ("rtdo_fp8_gemm_cpu_f64", "rtdo_fp8_gemm_w8a8_f64"):
            getattr(L, name).argtypes = [c_fp, c_u8p, c_fp, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_int64, c_dp]
            getattr(L, name).restype = None
        L.rtdo_ref_cpu_fp8_linear.argtypes = [c_fp, c_u8p, c_fp, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int64, ctypes.c_int64, c_fp, ctypes.c_int]
        L.rtdo_ref_cpu_fp8_linear.restype = None
        L.rtdo_max_threads.argtypes = []
        L.rtdo_max_threads.restype = ctypes.c_int
        L.rtdo_cpu_qmatmul.argtypes = [ctypes.c_uint32, c_u8p, ctypes.c_int64, ctypes.c_int64, c_fp,
                                       ctypes.c_int64, c_fp, ctypes.c_int, ctypes.c_int]
        L.rtdo_cpu_qmatmul.restype = ctypes.c_int
        L.rtdo_cpu_quantize_x.argtypes = [ctypes.c_uint32, c_fp, ctypes.c_int64, ctypes.POINTER(ctypes.c_int8),
                                          c_fp, ctypes.POINTER(ctypes.c_int16)]
        L.rtdo_cpu_quantize_x.restype = ctypes.c_int
        _lib = L
    return _lib


def _u8(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))


def _f32(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def _f64(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def f16_to_f32(bits: int) -> float:
    return lib().rtdo_f16_to_f32(bits)


def block_geometry(ggml_type: int):
    e, b = ctypes.c_uint64(), ctypes.c_uint64()
    if lib().rtdo_block_geometry(ggml_type, ctypes.byref(e), ctypes.byref(b)) != 0:
        return None
    return int(e.value), int(b.value)


def dequant_block(ggml_type: int, block: bytes) -> np.ndarray:
    buf = np.frombuffer(bytes(block), dtype=np.uint8).copy()
    n = 32 if ggml_type == Q8_0 else 256
    out = np.zeros(n, dtype=np.float32)
    fn = {Q8_0: "rtdo_dequant_q8_0_block", Q4_K: "rtdo_dequant_q4_k_block",
          Q6_K: "rtdo_dequant_q6_k_block"}[ggml_type]
    getattr(lib(), fn)(_u8(buf), _f32(out))
    return out


def dequant_tensor(ggml_type: int, raw: np.ndarray, n_elements: int):
    """Returns (status, f32 array).  status follows dequant.rs:83-146."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.zeros(max(n_elements, 1), dtype=np.float32)
    rc = lib().rtdo_dequant_tensor(ggml_type, _u8(raw), raw.size, n_elements, _f32(out))
    return rc, out[:n_elements]


def qgemv_f64(ggml_type: int, raw: np.ndarray, N: int, K: int, x: np.ndarray, bias=None) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    M = x.shape[0]
    y = np.zeros((M, N), dtype=np.float64)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    rc = lib().rtdo_qgemv_f64(ggml_type, _u8(raw), raw.size, N, K, _f32(x), M,
                              None if b is None else _f32(b), _f64(y))
    if rc != OK:
        raise ValueError(f"oracle qgemv failed with status {rc}")
    return y


def ref_cpu_linear(ggml_type: int, raw: np.ndarray, N: int, K: int, x: np.ndarray, threads: int = 0):
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    y = np.zeros((x.shape[0], N), dtype=np.float32)
    lib().rtdo_ref_cpu_linear(ggml_type, _u8(raw), N, K, _f32(x), x.shape[0], _f32(y), threads)
    return y


def cpu_qmatmul(ggml_type: int, raw: np.ndarray, N: int, K: int, x: np.ndarray, threads: int = 0,
                simd: bool = True) -> np.ndarray:
    """The reference's CPU quantized matmul (candle-core 0.11 QMatMul::forward behind
    linear_layer.rs:45-52): x quantized to Q8_K blocks (Q8_0 for Q8_0 weights), integer
    dots per block, f32 accumulation.  The timed CPU baseline of the bench."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    y = np.zeros((x.shape[0], N), dtype=np.float32)
    rc = lib().rtdo_cpu_qmatmul(ggml_type, _u8(raw), N, K, _f32(x), x.shape[0], _f32(y), threads, int(simd))
    if rc != 0:
        raise ValueError(f"rtdo_cpu_qmatmul: status {rc} (type {ggml_type}, K {K})")
    return y


def cpu_quantize_x(ggml_type: int, x: np.ndarray):
    """(codes int8 [K], scales f32 [K / QK], bsums int16 [K / 16] or None) of the
    activation blocks rtdo_cpu_qmatmul builds for x[K]."""
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    qk = 32 if ggml_type == Q8_0 else 256
    codes = np.zeros(x.size, dtype=np.int8)
    scales = np.zeros(x.size // qk, dtype=np.float32)
    bsums = None if ggml_type == Q8_0 else np.zeros(x.size // 16, dtype=np.int16)
    rc = lib().rtdo_cpu_quantize_x(ggml_type, _f32(x), x.size, codes.ctypes.data_as(ctypes.POINTER(ctypes.c_int8)),
                                   _f32(scales),
                                   None if bsums is None else bsums.ctypes.data_as(ctypes.POINTER(ctypes.c_int16)))
    if rc != 0:
        raise ValueError(f"rtdo_cpu_quantize_x: status {rc}")
    return codes, scales, bsums


def fp8_to_f32(b: int) -> float:
    return lib().rtdo_fp8_e4m3_to_f32(b)


def f32_to_fp8(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    out = np.zeros(x.size, dtype=np.uint8)
    lib().rtdo_f32_to_fp8_e4m3_array(_f32(x), x.size, _u8(out))
    return out


def fp8_lut() -> np.ndarray:
    return np.array([fp8_to_f32(b) for b in range(256)], dtype=np.float32)


def fp8_gemm_cpu_f64(x, w, scale, N, K) -> np.ndarray:
    """fp8_gemm.rs:55-74 CPU fallback semantics (x . (LUT(w) * s)^T)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(N, K)
    s = None if scale is None else np.ascontiguousarray(scale, dtype=np.float32).ravel()
    y = np.zeros((x.shape[0], N), dtype=np.float64)
    lib().rtdo_fp8_gemm_cpu_f64(_f32(x), _u8(w), None if s is None else _f32(s),
                                1 if s is None else s.size, x.shape[0], N, K, _f64(y))
    return y


def fp8_gemm_w8a8_f64(x, w, scale, N, K) -> np.ndarray:
    """fp8_gemm.rs:96-101,180-186 CUDA semantics (x -> E4M3 unscaled, then scale)."""
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(N, K)
    s = None if scale is None else np.ascontiguousarray(scale, dtype=np.float32).ravel()
    y = np.zeros((x.shape[0], N), dtype=np.float64)
    lib().rtdo_fp8_gemm_w8a8_f64(_f32(x), _u8(w), None if s is None else _f32(s),
                                 1 if s is None else s.size, x.shape[0], N, K, _f64(y))
    return y


def ref_cpu_fp8_linear(x, w, scale, N, K, threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, K)
    w = np.ascontiguousarray(w, dtype=np.uint8).reshape(N, K)
    s = np.ascontiguousarray(scale, dtype=np.float32).ravel()
    y = np.zeros((x.shape[0], N), dtype=np.float32)
    lib().rtdo_ref_cpu_fp8_linear(_f32(x), _u8(w), _f32(s), s.size, x.shape[0], N, K, _f32(y), threads)
    return y


def max_threads() -> int:
    return int(lib().rtdo_max_threads())


# ---------------------------------------------------------------- INT4 Marlin
# crates/runtimed-model/src/ops/marlin_gemv.rs: the packed layout [ceil(K/32)][N][4] u32,
# nibble `nib` of word `w` of chunk `c` is k = 32c + 8w + nib (:47-59, :76-94).

def marlin_repack(weight, scales):
    """repack_marlin_tiles (marlin_gemv.rs:64-97): q = clamp(round(w * inv_s) + 8, 0, 15)
    with f32 arithmetic, round half away from zero, inv_s = 1 / s unless |s| <= 1e-12."""
    w = np.asarray(weight, dtype=np.float32)
    n, k = w.shape
    s = np.asarray(scales, dtype=np.float32).reshape(-1)
    kc = (k + 31) // 32
    packed = np.zeros((kc, n, 4), dtype=np.uint32)
    for c in range(kc):
        for r in range(n):
            inv = np.float32(1.0) / s[r] if abs(float(s[r])) > 1e-12 else np.float32(1.0)
            for wi in range(4):
                word = 0
                for nib in range(8):
                    kk = c * 32 + wi * 8 + nib
                    if kk < k:
                        v = np.float32(w[r, kk] * inv)
                        rv = np.floor(abs(float(v)) + 0.5) * (1.0 if v >= 0 else -1.0)
                        q = int(min(max(rv + 8.0, 0.0), 15.0))
                    else:
                        q = 8
                    word |= (q & 0xF) << (4 * nib)
                packed[c, r, wi] = word
    return packed


def marlin_dequant(packed, scales, n: int, k: int) -> np.ndarray:
    """MarlinWeight::dequantize (marlin_gemv.rs:42-60): ((q as i32 - 8) as f32) * s[n] in f32."""
    p = np.asarray(packed, dtype=np.uint32).reshape(-1)
    s = np.asarray(scales, dtype=np.float32).reshape(-1)
    kc = (k + 31) // 32
    out = np.zeros((n, k), dtype=np.float32)
    for c in range(kc):
        base = (c * n + np.arange(n)) * 4
        for wi in range(4):
            words = p[base + wi]
            for nib in range(8):
                kk = c * 32 + wi * 8 + nib
                if kk < k:
                    q = ((words >> np.uint32(4 * nib)) & np.uint32(0xF)).astype(np.int32) - 8
                    out[:, kk] = q.astype(np.float32) * s
    return out


def marlin_gemv_f64(x, packed, scales, n: int, k: int) -> np.ndarray:
    """cpu_marlin_gemv_fallback (marlin_gemv.rs:99-110) accumulated in f64."""
    w = marlin_dequant(packed, scales, n, k).astype(np.float64)
    return np.asarray(x, dtype=np.float64).reshape(-1, k) @ w.T
