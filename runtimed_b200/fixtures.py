"""Seeded random-init Qwen2 decoders written as GGUF files the reference loads.

The benchmark configs describe random-init Qwen2-architecture models "written as a GGUF
file the reference loads".  ``write_qwen2_gguf`` writes one with gguf-py's GGUFWriter
(GGUF v3, alignment 32), with the metadata ``parse_gguf_config`` reads
(crates/runtimed-model/src/config/parse_gguf.rs:52-90: ``qwen2.block_count``,
``embedding_length``, ``attention.head_count(_kv)``,
``attention.layer_norm_rms_epsilon``, ``rope.freq_base``, ``feed_forward_length``), the
q/k/v biases and an explicit ``output.weight`` (a copy of ``token_embd.weight`` for
tied embeddings: the reference refuses a Qwen2 file without one, parse_gguf.rs:220-222).

Formats are Q4_K_M-style: Q4_K for attn_q / attn_k / attn_output / ffn_gate / ffn_up,
Q6_K for attn_v / ffn_down / token_embd.  K-quant superblocks run along K in 256s, so
a tensor whose K is not a multiple of 256 (hidden 896 in config 0) falls back to Q8_0;
``formats`` can override any of them (config 4's target model is all Q8_0).  Block
fields follow the configs' distributions (runtimed_b200.synth); biases N(0, 0.02),
norm weights 1.0.  Every tensor draws from its own seeded stream.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, Optional

import numpy as np

from . import synth

F32 = 0


@dataclass
class Qwen2Shape:
    hidden: int
    n_layer: int
    n_head: int
    n_kv: int
    ffn: int
    vocab: int
    eps: float = 1e-6
    rope_theta: float = 1e6
    tied: bool = True
    context: int = 32768
    formats: Dict[str, int] = field(default_factory=dict)

    @property
    def head_dim(self) -> int:
        return self.hidden // self.n_head


CONFIGS = {
    # Qwen2-0.5B-shaped
    "config0": Qwen2Shape(hidden=896, n_layer=24, n_head=14, n_kv=2, ffn=4864, vocab=151936),
    # Qwen2-7B-shaped
    "config2": Qwen2Shape(hidden=3584, n_layer=28, n_head=28, n_kv=4, ffn=18944, vocab=152064, tied=False),
}

DEFAULT_FORMATS = {"attn_q": synth.Q4_K, "attn_k": synth.Q4_K, "attn_v": synth.Q6_K, "attn_output": synth.Q4_K,
                   "ffn_gate": synth.Q4_K, "ffn_up": synth.Q4_K, "ffn_down": synth.Q6_K, "token_embd": synth.Q6_K,
                   "output": synth.Q6_K}


def tensor_format(shape: Qwen2Shape, kind: str, k: int) -> int:
    t = shape.formats.get(kind, DEFAULT_FORMATS[kind])
    if t in (synth.Q4_K, synth.Q6_K) and k % 256:
        return synth.Q8_0  # K-quant superblocks need K % 256 == 0
    return t


def layer_tensors(shape: Qwen2Shape):
    """(kind, N, K) of one layer's quantized linears, in call order."""
    h, hd = shape.hidden, shape.head_dim
    return [("attn_q", shape.n_head * hd, h), ("attn_k", shape.n_kv * hd, h), ("attn_v", shape.n_kv * hd, h),
            ("attn_output", h, shape.n_head * hd), ("ffn_gate", shape.ffn, h), ("ffn_up", shape.ffn, h),
            ("ffn_down", h, shape.ffn)]


def write_qwen2_gguf(path: str, shape: Qwen2Shape, seed: int = 0) -> Dict[str, int]:
    """Write the model to `path`; returns {tensor name: ggml type} of the quantized tensors."""
    import gguf

    w = gguf.GGUFWriter(path, "qwen2")
    w.add_block_count(shape.n_layer)
    w.add_context_length(shape.context)
    w.add_embedding_length(shape.hidden)
    w.add_feed_forward_length(shape.ffn)
    w.add_head_count(shape.n_head)
    w.add_head_count_kv(shape.n_kv)
    w.add_layer_norm_rms_eps(shape.eps)
    w.add_rope_freq_base(shape.rope_theta)
    stream = [0]
    types: Dict[str, int] = {}

    def quant(name: str, kind: str, n: int, k: int) -> np.ndarray:
        t = tensor_format(shape, kind, k)
        stream[0] += 1
        raw = synth.quant_matrix(t, n, k, seed=seed, stream=stream[0])
        elems, bb = synth.BLOCK[t]
        w.add_tensor(name, raw.reshape(n, (k // elems) * bb), raw_dtype=gguf.GGMLQuantizationType(t))
        types[name] = t
        return raw

    def dense(name: str, v: np.ndarray) -> None:
        w.add_tensor(name, np.ascontiguousarray(v, dtype=np.float32))

    emb = quant("token_embd.weight", "token_embd", shape.vocab, shape.hidden)
    for i in range(shape.n_layer):
        p = f"blk.{i}"
        dense(f"{p}.attn_norm.weight", np.ones(shape.hidden, np.float32))
        for kind, n, k in layer_tensors(shape):
            quant(f"{p}.{kind}.weight", kind, n, k)
            if kind in ("attn_q", "attn_k", "attn_v"):
                stream[0] += 1
                b = synth.rng(seed, stream[0]).normal(0.0, 0.02, n).astype(np.float32)
                dense(f"{p}.{kind}.bias", b)
        dense(f"{p}.ffn_norm.weight", np.ones(shape.hidden, np.float32))
    dense("output_norm.weight", np.ones(shape.hidden, np.float32))
    if shape.tied:
        t = types["token_embd.weight"]
        elems, bb = synth.BLOCK[t]
        w.add_tensor("output.weight", emb.reshape(shape.vocab, (shape.hidden // elems) * bb),
                     raw_dtype=gguf.GGMLQuantizationType(t))
        types["output.weight"] = t
    else:
        quant("output.weight", "output", shape.vocab, shape.hidden)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return types


def small_shape(n_layer: int = 2, vocab: int = 1000, formats: Optional[Dict[str, int]] = None) -> Qwen2Shape:
    """A few-layer Qwen2 with config 0's head layout (for quick tests)."""
    return Qwen2Shape(hidden=256, n_layer=n_layer, n_head=4, n_kv=2, ffn=512, vocab=vocab, formats=dict(formats or {}))
