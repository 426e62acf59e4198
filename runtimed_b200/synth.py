"""Seeded random-init GGUF blocks with the value distributions of the benchmark configs.

The reference's benchmark configs use random-init weights written as GGUF, so
these generators produce raw superblock bytes exactly as a GGUF file stores them
(little-endian, the block layouts of crates/runtimed-gguf/src/quant/dequant.rs
and dequant_k.rs):

  Q4_K  [d f16][dmin f16][scales 12][qs 128]   d, dmin = f16(|N(0,1)| * 2e-3); other bytes uniform
  Q6_K  [ql 128][qh 64][scales i8 16][d f16]   d = f16(|N(0,1)| * 1e-3); scales uniform [-32, 31]
  Q8_0  [d f16][qs i8 32]                      d = f16(|N(0,1)| * 4e-3); codes uniform [-127, 127]
  FP8   E4M3 bytes, per-row scale s = amax/448, W ~ N(0, 0.02), byte = E4M3(W / s)

Every stream is a numpy PCG64 generator seeded from (seed, tensor index).
"""
from __future__ import annotations

import numpy as np

Q8_0, Q4_K, Q6_K = 8, 12, 14
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}
NAMES = {Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}


def rng(seed: int, stream: int = 0) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64([seed, stream]))


def _f16_bits(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint16)


def q4_k_blocks(n_blocks: int, g: np.random.Generator) -> np.ndarray:
    out = g.integers(0, 256, size=(n_blocks, 144), dtype=np.uint8)
    d = _f16_bits(np.abs(g.standard_normal(n_blocks)) * 2e-3)
    dmin = _f16_bits(np.abs(g.standard_normal(n_blocks)) * 2e-3)
    out[:, 0:2] = d.view(np.uint8).reshape(n_blocks, 2)
    out[:, 2:4] = dmin.view(np.uint8).reshape(n_blocks, 2)
    return out


def q6_k_blocks(n_blocks: int, g: np.random.Generator) -> np.ndarray:
    out = g.integers(0, 256, size=(n_blocks, 210), dtype=np.uint8)
    out[:, 192:208] = g.integers(-32, 32, size=(n_blocks, 16), dtype=np.int8).view(np.uint8)
    d = _f16_bits(np.abs(g.standard_normal(n_blocks)) * 1e-3)
    out[:, 208:210] = d.view(np.uint8).reshape(n_blocks, 2)
    return out


def q8_0_blocks(n_blocks: int, g: np.random.Generator) -> np.ndarray:
    out = np.empty((n_blocks, 34), dtype=np.uint8)
    d = _f16_bits(np.abs(g.standard_normal(n_blocks)) * 4e-3)
    out[:, 0:2] = d.view(np.uint8).reshape(n_blocks, 2)
    out[:, 2:34] = g.integers(-127, 128, size=(n_blocks, 32), dtype=np.int8).view(np.uint8)
    return out


def quant_matrix(ggml_type: int, N: int, K: int, seed: int = 0, stream: int = 0) -> np.ndarray:
    """Raw GGUF bytes of an [N, K] matrix: N rows of K/elems blocks, flattened."""
    elems, _ = BLOCK[ggml_type]
    if K % elems:
        raise ValueError(f"K={K} is not a multiple of the {NAMES[ggml_type]} block ({elems})")
    nb = N * (K // elems)
    g = rng(seed, stream)
    fn = {Q8_0: q8_0_blocks, Q4_K: q4_k_blocks, Q6_K: q6_k_blocks}[ggml_type]
    return fn(nb, g).reshape(-1)


def e4m3_table() -> np.ndarray:
    """E4M3 decode table (sign, 4-bit exponent bias 7, 3-bit mantissa, 0x7f/0xff NaN)."""
    b = np.arange(256)
    sign = np.where(b & 0x80, -1.0, 1.0)
    exp = (b >> 3) & 0xF
    mant = (b & 7).astype(np.float64)
    v = np.where(exp == 0, sign * 2.0 ** -6 * (mant / 8.0), sign * 2.0 ** (exp - 7) * (1.0 + mant / 8.0))
    v[(exp == 15) & ((b & 7) == 7)] = np.nan
    return v.astype(np.float32)


def encode_e4m3(x: np.ndarray) -> np.ndarray:
    """Vectorised E4M3 encoder with ties to the lower magnitude and saturation at 448."""
    lut = e4m3_table()[:127].astype(np.float64)
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64)
    idx = np.searchsorted(lut, a, side="left")
    idx = np.clip(idx, 1, 126)
    lo, hi = lut[idx - 1], lut[idx]
    exact = lut[np.clip(np.searchsorted(lut, a, side="left"), 0, 126)] == a
    pick = np.where(a - lo <= hi - a, idx - 1, idx)
    code = np.where(exact, np.clip(np.searchsorted(lut, a, side="left"), 0, 126), pick)
    code = np.where(a >= 448.0, 0x7E, code)
    code = np.where(a <= 0.0, 0, code)
    sign = np.signbit(x).astype(np.uint8) << 7
    out = (code.astype(np.uint8) | sign).astype(np.uint8)
    out = np.where(np.isnan(x), np.uint8(0x7F), out)
    return out.astype(np.uint8)


def fp8_matrix(N: int, K: int, seed: int = 0, stream: int = 0):
    """(E4M3 bytes [N, K], per-row f32 scale [N]) with W ~ N(0, 0.02), s = amax/448."""
    g = rng(seed, stream)
    w = (g.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    s = (np.abs(w).max(axis=1) / np.float32(448.0)).astype(np.float32)
    s[s == 0] = 1.0
    q = encode_e4m3(w / s[:, None])
    return q, s


def activations(M: int, K: int, seed: int = 0, stream: int = 1) -> np.ndarray:
    """f32 activations ~ N(0, 1) (callers round to bf16 where the config says bf16)."""
    return rng(seed, stream).standard_normal((M, K), dtype=np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round f32 to the nearest bf16 (ties to even) and return it as f32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)
