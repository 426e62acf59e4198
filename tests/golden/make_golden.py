"""Generate the committed golden fixtures under tests/golden/.

Independent implementations only -- nothing here calls the oracle:
  * dequantized blocks come from gguf-py ``gguf.quants.dequantize`` (the GGML
    project's own Python decoder, version recorded in the fixture);
  * GEMV goldens are ``x . dequant(W)^T`` in float64 numpy over the gguf-py
    dequantization;
  * E4M3 decode values come from torch's ``float8_e4m3fn`` (exact for every
    non-NaN code) and encoder goldens for non-tie inputs from torch's
    round-to-nearest cast (ties are pinned separately in the tests, because the
    reference rounds ties toward the lower magnitude).

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

from runtimed_b200 import synth  # noqa: E402


def main() -> None:
    import gguf
    from gguf import quants
    from gguf import GGMLQuantizationType as T
    import torch

    gt = {synth.Q4_K: T.Q4_K, synth.Q6_K: T.Q6_K, synth.Q8_0: T.Q8_0}
    out = {"gguf_py_version": np.array(getattr(gguf, "__version__", "unknown"))}
    # Dequant goldens: 24 random blocks per format with the benchmark distributions,
    # plus a block with f16 subnormal / negative-zero scales to cover the f16 corners.
    for t, name in synth.NAMES.items():
        elems, bb = synth.BLOCK[t]
        raw = synth.quant_matrix(t, 3, elems * 8, seed=1234, stream=t).reshape(-1, bb)
        special = raw[0].copy()
        # d = 0x0001 (smallest subnormal); for Q4_K dmin = 0x8000 (-0.0)
        if t == synth.Q6_K:
            special[208:210] = [0x01, 0x00]
        else:
            special[0:2] = [0x01, 0x00]
            if t == synth.Q4_K:
                special[2:4] = [0x00, 0x80]
        raw = np.concatenate([raw, special[None, :]], axis=0)
        deq = quants.dequantize(raw, gt[t]).astype(np.float32).reshape(-1)
        out[f"{name}_blocks"] = raw
        out[f"{name}_dequant"] = deq
    # GEMV goldens on a small matrix per format (N=24 rows, K=512, M=3).
    for t, name in synth.NAMES.items():
        N, K, M = 24, 512, 3
        raw = synth.quant_matrix(t, N, K, seed=99, stream=t)
        w = quants.dequantize(raw.reshape(N, -1), gt[t]).astype(np.float32).reshape(N, K)
        x = synth.bf16_round(synth.activations(M, K, seed=99, stream=100 + t))
        bias = (synth.rng(99, 200 + t).standard_normal(N) * 0.02).astype(np.float32)
        y = x.astype(np.float64) @ w.astype(np.float64).T + bias.astype(np.float64)
        out[f"{name}_gemv_raw"] = raw
        out[f"{name}_gemv_x"] = x
        out[f"{name}_gemv_bias"] = bias
        out[f"{name}_gemv_y"] = y
        out[f"{name}_gemv_shape"] = np.array([N, K, M])
    # E4M3 decode table from torch, NaN codes excluded.
    codes = torch.arange(256, dtype=torch.uint8)
    lut = codes.view(torch.float8_e4m3fn).to(torch.float32).numpy()
    out["e4m3_lut_torch"] = lut
    # Encoder goldens at non-tie inputs (torch casts with round-to-nearest-even;
    # saturate first because torch maps overflow to NaN).
    g = np.random.Generator(np.random.PCG64(7))
    xs = np.concatenate([
        g.standard_normal(4000).astype(np.float32) * np.float32(40.0),
        g.standard_normal(2000).astype(np.float32) * np.float32(0.01),
        np.array([0.0, -0.0, 1.0, 2.0, 0.5, 3.0, 447.0, -447.99, 2.0 ** -9, -(2.0 ** -9)], np.float32),
    ])
    pos = np.sort(lut[:127].astype(np.float64))
    a = np.abs(xs.astype(np.float64))
    idx = np.clip(np.searchsorted(pos, a), 1, 126)
    is_tie = np.isclose(a - pos[idx - 1], pos[idx] - a, rtol=0, atol=0)
    xs = xs[(~is_tie) & (a < 448.0)]
    enc = torch.from_numpy(xs).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    out["e4m3_enc_x"] = xs
    out["e4m3_enc_code"] = enc
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
