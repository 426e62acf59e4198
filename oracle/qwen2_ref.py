"""CPU restatement of the reference Qwen2 forward (test infrastructure, never the product).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs use this module: it is the
end-to-end checker of the GPU forward (runtimed_b200.qwen2).  It reads the GGUF with
gguf-py's own reader (independent of the product's parser), decodes every quantized
tensor with the restated reference dequantizers (oracle/rtd_oracle.c, bit-exact with
crates/runtimed-gguf/src/quant/dequant*.rs) and runs the layer math of
crates/runtimed-model/src/arch/qwen2.rs in float32 numpy, one step at a time:

  layer (qwen2.rs:68-127):  n = rmsnorm(h, attn_norm); q, k, v = linear_bias(n)
                            q, k = rope(q), rope(k); append k, v to the cache
                            o = attention(q, K, V, causal mask, 1/sqrt(head_dim))
                            h += linear(o, attn_output); n = rmsnorm(h, ffn_norm)
                            h += linear(silu(linear(n, gate)) * linear(n, up), down)
  forward (qwen2.rs:217-229): h = embed(ids); layers; rmsnorm(output_norm); linear(output)
  rmsnorm    ops/norm.rs:7-11        x / sqrt(mean(x^2) + eps) * w
  rope       ops/rope.rs:24-60       NeoX halves, inv = theta^(-2i/rot_dim) in f32
  attention  ops/attention.rs:107-128  GQA head h reads kv head h // (n_head / n_kv),
                                       softmax(q k^T * scale + mask) v, mask :38-58
  silu       ops/activation.rs:6-10  x * 1 / (exp(-x) + 1)

The KV cache keeps float32 values (the reference's CPU cache); the GPU keeps f16, so the
two agree to the logits tolerance the configs state (1e-2 relative), not bit for bit.
"""
from __future__ import annotations

import numpy as np

from . import dequant_tensor

F32 = np.float32


def _rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    m2 = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    denom = np.sqrt(m2 + F32(eps))
    return (x / denom) * w


def _rope(x: np.ndarray, positions: np.ndarray, theta: float, rot_dim: int) -> np.ndarray:
    """x [heads, t, d] (rope.rs:24-60, factors None)."""
    half = rot_dim // 2
    i = np.arange(half, dtype=F32)
    inv = np.power(F32(theta), (F32(-2.0) * i) / F32(rot_dim)).astype(F32)
    ang = positions.astype(F32)[:, None] * inv[None, :]
    cos, sin = np.cos(ang).astype(F32), np.sin(ang).astype(F32)
    x1, x2 = x[..., :half], x[..., half:rot_dim]
    o1 = x1 * cos - x2 * sin
    o2 = x2 * cos + x1 * sin
    return np.concatenate([o1, o2, x[..., rot_dim:]], axis=-1).astype(F32)


def _silu(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):  # exp(-x) overflows to inf for x < -88: silu -> -0, as in f32
        return x * (F32(1.0) / (np.exp(-x) + F32(1.0)))


class RefQwen2:
    """The restated forward over one GGUF file; ``forward(ids, q0)`` -> logits [t, vocab]."""

    def __init__(self, path: str, kv_f16: bool = False):
        """kv_f16 rounds the cached keys and values to f16, as the GPU's cache stores them
        (a diagnostic knob: the reference's CPU cache is f32)."""
        import gguf

        self.kv_f16 = kv_f16

        r = gguf.GGUFReader(path)
        meta = {f.name: f for f in r.fields.values()}

        def scalar(key):
            f = meta[key]
            return f.parts[f.data[0]][0].item()

        self.n_layer = int(scalar("qwen2.block_count"))
        self.hidden = int(scalar("qwen2.embedding_length"))
        self.n_head = int(scalar("qwen2.attention.head_count"))
        self.n_kv = int(scalar("qwen2.attention.head_count_kv"))
        self.eps = float(np.float32(scalar("qwen2.attention.layer_norm_rms_epsilon")))
        self.theta = float(np.float32(scalar("qwen2.rope.freq_base")))
        self.head_dim = self.hidden // self.n_head
        self.w = {}
        for t in r.tensors:
            dims = [int(d) for d in t.shape]  # GGUF order, fastest first
            n_el = int(np.prod(dims))
            raw = np.ascontiguousarray(np.asarray(t.data).reshape(-1).view(np.uint8))
            if int(t.tensor_type) == 0:
                v = raw.view(F32).copy()
            else:
                rc, v = dequant_tensor(int(t.tensor_type), raw, n_el)
                if rc != 0:
                    raise ValueError(f"{t.name}: dequant status {rc}")
            self.w[t.name] = v.reshape(dims[::-1]) if len(dims) == 2 else v
        self.vocab = self.w["token_embd.weight"].shape[0]
        self.reset()

    def reset(self) -> None:
        self.k_cache = [np.zeros((self.n_kv, 0, self.head_dim), F32) for _ in range(self.n_layer)]
        self.v_cache = [np.zeros((self.n_kv, 0, self.head_dim), F32) for _ in range(self.n_layer)]

    def truncate(self, length: int) -> None:
        self.k_cache = [k[:, :length] for k in self.k_cache]
        self.v_cache = [v[:, :length] for v in self.v_cache]

    def _lin(self, x, name, bias=None):
        y = x @ self.w[name].T
        if bias is not None:
            y = y + self.w[bias]
        return y.astype(F32)

    def _layer(self, i: int, h: np.ndarray, q0: int) -> np.ndarray:
        p = f"blk.{i}"
        t = h.shape[0]
        hd, G = self.head_dim, self.n_head // self.n_kv
        n = _rmsnorm(h, self.w[f"{p}.attn_norm.weight"], self.eps)
        q = self._lin(n, f"{p}.attn_q.weight", f"{p}.attn_q.bias").reshape(t, self.n_head, hd).transpose(1, 0, 2)
        k = self._lin(n, f"{p}.attn_k.weight", f"{p}.attn_k.bias").reshape(t, self.n_kv, hd).transpose(1, 0, 2)
        v = self._lin(n, f"{p}.attn_v.weight", f"{p}.attn_v.bias").reshape(t, self.n_kv, hd).transpose(1, 0, 2)
        pos = np.arange(q0, q0 + t)
        q = _rope(q, pos, self.theta, hd)
        k = _rope(k, pos, self.theta, hd)
        if self.kv_f16:
            k, v = k.astype(np.float16).astype(F32), v.astype(np.float16).astype(F32)
        self.k_cache[i] = np.concatenate([self.k_cache[i], k], axis=1)
        self.v_cache[i] = np.concatenate([self.v_cache[i], v], axis=1)
        K = np.repeat(self.k_cache[i], G, axis=0)  # head h -> kv head h // G
        V = np.repeat(self.v_cache[i], G, axis=0)
        total = K.shape[1]
        scores = (q @ K.transpose(0, 2, 1)) * F32(1.0 / np.sqrt(np.float32(hd)))
        if t > 1:
            qi = np.arange(t)[:, None] + q0
            kj = np.arange(total)[None, :]
            scores = np.where(kj <= qi, scores, -np.inf).astype(F32)
        e = np.exp(scores - scores.max(axis=-1, keepdims=True))
        probs = (e / e.sum(axis=-1, keepdims=True)).astype(F32)
        o = (probs @ V).transpose(1, 0, 2).reshape(t, self.n_head * hd)
        h = h + self._lin(o, f"{p}.attn_output.weight")
        n = _rmsnorm(h, self.w[f"{p}.ffn_norm.weight"], self.eps)
        g = self._lin(n, f"{p}.ffn_gate.weight")
        u = self._lin(n, f"{p}.ffn_up.weight")
        return (h + self._lin(_silu(g) * u, f"{p}.ffn_down.weight")).astype(F32)

    def forward(self, ids, q0: int, trace=None) -> np.ndarray:
        """Logits [t, vocab] of ids at positions q0 .. q0 + t - 1 (qwen2.rs:217-229);
        `trace` (a list) receives the residual stream after every layer."""
        h = self.w["token_embd.weight"][np.asarray(ids, dtype=np.int64)].astype(F32)
        for i in range(self.n_layer):
            h = self._layer(i, h, q0)
            if trace is not None:
                trace.append(h.copy())
        h = _rmsnorm(h, self.w["output_norm.weight"], self.eps)
        return self._lin(h, "output.weight")

    def greedy(self, prompt, steps: int):
        """Prefill the prompt, then `steps` greedy tokens; returns (ids, logits per step)."""
        self.reset()
        logits = self.forward(prompt, 0)[-1]
        out, per = [], [logits]
        pos = len(prompt)
        for _ in range(steps):
            nxt = int(np.argmax(logits))
            out.append(nxt)
            logits = self.forward([nxt], pos)[-1]
            per.append(logits)
            pos += 1
        return out, per
