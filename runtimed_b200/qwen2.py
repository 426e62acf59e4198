"""Qwen2 decoder on the device: the caller of the quantized-linear path.

Mirrors crates/runtimed-model/src/arch/qwen2.rs (``layer`` :68-127, ``forward`` :217-229)
with the model's arithmetic in libruntimed_b200.so: ``rtd_qembed`` for the embedding,
``rtd_qlinear`` for every linear (bias fused), and the decoder-layer operations
``rtd_rmsnorm`` (residual add fused), ``rtd_rope_kv_append``, ``rtd_attention_paged``,
``rtd_silu_mul`` and ``rtd_argmax``.  The residual stream and every linear's input and
output are f32, as in the reference's CPU path; the KV cache is f16 and PAGED
(``PagedKvCache``: 16-token blocks from one pool, a block table per sequence,
crates/runtimed-model/src/cache/paged/table.rs:57-145), which the reference leaves
unwired for Qwen2 (its forward is batch-1 over a contiguous cache).  Every token of a
call carries its own (sequence, position), so ``forward`` serves a prefill chunk of one
sequence, ``decode_batch`` one token of many sequences, and a speculative verify of
k + 1 positions followed by ``PagedKvCache.truncate`` (the rollback of rejected
positions, crates/runtimed-model/src/decode/speculate.rs:31-199).

With a communicator (one process per GPU) the decoder runs tensor parallel over N ranks,
the reference's dual-GPU blocks (crates/runtimed-model/src/tp/dual_gpu.rs:52-186,
arch/qwen2.rs:142-197) generalised: every rank holds its query / kv heads and FFN rows of
the column-parallel linears and the matching input columns of attn_output and ffn_down,
whose outputs are summed over the ranks inside rtd_tp_qlinear_row; the embedding, norms
and LM head are replicated, so every rank carries the same residual stream bit for bit
and takes the same greedy token.

The configuration comes from the GGUF metadata as ``parse_gguf_config`` reads it
(crates/runtimed-model/src/config/parse_gguf.rs:52-90 for arch "qwen2": head_dim =
hidden / n_head, rope over the whole head, q/k/v bias when ``blk.0.attn_q.bias``
exists; a file without ``output.weight`` is refused).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from . import _lib
from .errors import ConfigError, MissingWeight
from .gguf import GgufFile
from .weights import Context, QMatMul, Weights, _raise, _stream_ptr

KV_BLOCK = 16


@dataclass
class Qwen2Config:
    n_layer: int
    hidden: int
    n_head: int
    n_kv: int
    head_dim: int
    ffn: int
    vocab: int
    eps: float
    rope_theta: float
    has_qkv_bias: bool

    @classmethod
    def from_gguf(cls, f: GgufFile) -> "Qwen2Config":
        arch = f.meta_str("general.architecture")
        if arch != "qwen2":
            raise ConfigError(f"unsupported architecture {arch!r} (this decoder is qwen2)")

        def u32(key):
            v = f.metadata.get(key)
            if not isinstance(v, int) or isinstance(v, bool):
                raise ConfigError(f"{key} missing, got {v!r}")
            return int(v)

        def f32(key):
            v = f.metadata.get(key)
            if not isinstance(v, float):
                raise ConfigError(f"{key} missing, got {v!r}")
            return float(np.float32(v))

        emb = f.tensor("token_embd.weight")
        if emb is None:
            raise MissingWeight("token_embd.weight")
        if f.tensor("output.weight") is None:
            raise ConfigError("qwen2 without output.weight: refusing to guess")
        hidden, n_head = u32("qwen2.embedding_length"), u32("qwen2.attention.head_count")
        return cls(n_layer=u32("qwen2.block_count"), hidden=hidden, n_head=n_head,
                   n_kv=u32("qwen2.attention.head_count_kv"), head_dim=hidden // n_head,
                   ffn=u32("qwen2.feed_forward_length"), vocab=int(emb.dims[1]),
                   eps=f32("qwen2.attention.layer_norm_rms_epsilon"), rope_theta=f32("qwen2.rope.freq_base"),
                   has_qkv_bias=f.tensor("blk.0.attn_q.bias") is not None)


class PagedKvCache:
    """f16 K / V of every layer in 16-token blocks from one pool, with a block table per
    sequence.  Block ids come from a free list; ``reserve`` grows a sequence to a length,
    ``truncate`` shrinks it (blocks past the new length return to the pool), ``release``
    frees it."""

    def __init__(self, cfg: Qwen2Config, num_blocks: int, max_seqs: int, max_ctx: int, device,
                 dtype: torch.dtype = torch.float16):
        if dtype not in (torch.float16, torch.float32):
            raise ConfigError(f"KV cache dtype {dtype} (f16 or f32)")
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        self.abi_dtype = _lib.DT_F16 if dtype == torch.float16 else _lib.DT_F32
        self.num_blocks, self.max_seqs = int(num_blocks), int(max_seqs)
        self.max_blocks = -(-int(max_ctx) // KV_BLOCK)
        shape = (self.num_blocks, cfg.n_kv, KV_BLOCK, cfg.head_dim)
        self.k = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in range(cfg.n_layer)]
        self.v = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in range(cfg.n_layer)]
        self.table = torch.zeros((self.max_seqs, self.max_blocks), dtype=torch.int32, device=self.device)
        self._host_table = np.zeros((self.max_seqs, self.max_blocks), dtype=np.int32)
        self._free: List[int] = list(range(self.num_blocks - 1, -1, -1))
        self._blocks: Dict[int, List[int]] = {}
        self.lengths: Dict[int, int] = {}
        self._dirty = False

    def reserve(self, seq: int, length: int) -> None:
        if not 0 <= seq < self.max_seqs:
            raise ConfigError(f"sequence {seq} outside 0..{self.max_seqs - 1}")
        need = -(-int(length) // KV_BLOCK)
        if need > self.max_blocks:
            raise ConfigError(f"sequence {seq}: {length} tokens exceed the cache's {self.max_blocks * KV_BLOCK}")
        blocks = self._blocks.setdefault(seq, [])
        while len(blocks) < need:
            if not self._free:
                raise ConfigError("KV cache out of blocks")
            b = self._free.pop()
            self._host_table[seq, len(blocks)] = b
            blocks.append(b)
            self._dirty = True
        self.lengths[seq] = max(self.lengths.get(seq, 0), int(length))

    def truncate(self, seq: int, length: int) -> None:
        """Keep the first `length` positions (speculative rollback, Cache::truncate)."""
        blocks = self._blocks.get(seq, [])
        keep = -(-int(length) // KV_BLOCK)
        while len(blocks) > keep:
            self._free.append(blocks.pop())
        self.lengths[seq] = min(self.lengths.get(seq, 0), int(length))

    def release(self, seq: int) -> None:
        self.truncate(seq, 0)
        self._blocks.pop(seq, None)
        self.lengths.pop(seq, None)

    def sync_table(self) -> None:
        if self._dirty:
            self.table.copy_(torch.from_numpy(self._host_table))
            self._dirty = False


class Qwen2Model:
    """Weights on one device and the forward over a paged KV cache.

    ``kv_dtype`` is the cache precision (f16 by default, as the configs run; f32 is the
    reference CPU cache's precision).  ``exact_linears`` runs every linear through the
    decode GEMV in passes of at most three tokens, whose products are exact (f32 rounding
    only), instead of the tensor-core GEMM, whose f16-rounded weights cost about 3e-4
    relative per linear; the parity checks use it to separate the layer math from the
    GEMM's rounding, which peaked attention over a long prompt amplifies."""

    def __init__(self, path_or_file, device="cuda:0", max_seqs: int = 1, max_ctx: int = 4096,
                 kv_blocks: Optional[int] = None, kv_dtype: torch.dtype = torch.float16,
                 exact_linears: bool = False, comm=None):
        self.file = path_or_file if isinstance(path_or_file, GgufFile) else GgufFile.open(path_or_file)
        self.cfg = Qwen2Config.from_gguf(self.file)
        self.device = torch.device(device)
        self.ctx = Context.for_device(self.device)
        self.L = _lib.lib()
        # tensor parallelism (one process per GPU, runtimed_b200.tp.TpComm): this rank's
        # query / kv heads and FFN rows; o_proj and ffn_down reduce over the ranks
        self.comm = comm
        self.rank, self.world = (comm.rank, comm.world) if comm is not None else (0, 1)
        cfg = self.cfg
        if cfg.n_head % self.world or cfg.n_kv % self.world or cfg.ffn % self.world:
            raise ConfigError(f"{cfg.n_head} heads / {cfg.n_kv} kv heads / FFN {cfg.ffn} do not split over "
                              f"{self.world} ranks")
        self.n_head_l, self.n_kv_l, self.ffn_l = cfg.n_head // self.world, cfg.n_kv // self.world, cfg.ffn // self.world
        self.weights = self._load()
        blocks = kv_blocks if kv_blocks is not None else max_seqs * (-(-max_ctx // KV_BLOCK))
        local = Qwen2Config(**{**cfg.__dict__, "n_kv": self.n_kv_l})
        self.cache = PagedKvCache(local, blocks, max_seqs, max_ctx, self.device, kv_dtype)
        self.max_ctx = int(max_ctx)
        self.exact_linears = bool(exact_linears)

    # ---- load (crates/runtimed-model/src/weights/load_gguf.rs:47-120)
    FUSE = (("qkv", ("attn_q", "attn_k", "attn_v")), ("gate_up", ("ffn_gate", "ffn_up")))

    def _shard(self, name: str, t) -> tuple:
        """(raw bytes, N, K) of this rank's part of a tensor: column-parallel linears keep
        their rows of this rank's heads / FFN rows, row-parallel ones (attn_output,
        ffn_down) their input columns (runtimed_b200.tp, crates/runtimed-model/src/tp/*)."""
        from . import tp

        raw = self.file.tensor_bytes(t)
        k, n = int(t.dims[0]), int(t.dims[1])
        if self.world == 1 or not name.startswith("blk."):
            return raw, n, k
        kind = name.split(".")[2]
        if kind in ("attn_q", "attn_k", "attn_v", "ffn_gate", "ffn_up"):
            return tp.shard_rows(raw, t.dtype, n, k, self.rank, self.world), n // self.world, k
        if kind in ("attn_output", "ffn_down"):
            return tp.shard_cols(raw, t.dtype, n, k, self.rank, self.world), n, k // self.world
        return raw, n, k

    def _bias(self, name: str) -> Optional[np.ndarray]:
        t = self.file.tensor(name)
        if t is None:
            return None
        b = self.file.tensor_bytes(t).view(np.float32)
        if self.world > 1:  # column-parallel bias: this rank's rows
            per = b.size // self.world
            b = b[self.rank * per:(self.rank + 1) * per]
        return b

    def _load(self) -> Weights:
        """Every tensor (this rank's part of it) to the device.  The linears of a layer that
        read the same input and share a format (q / k / v; gate / up) are uploaded as one
        row-concatenated matrix -- one launch serves them -- and ``q_map`` holds a row view
        of it under each name."""
        q_map: Dict[str, QMatMul] = {}
        dense: Dict[str, torch.Tensor] = {}
        infos = {t.name: t for t in self.file.tensors}
        self.fused: Dict[tuple, tuple] = {}
        for i in range(self.cfg.n_layer):
            for key, parts in self.FUSE:
                ts = [infos.get(f"blk.{i}.{p}.weight") for p in parts]
                if any(t is None or len(t.dims) != 2 for t in ts):
                    continue
                if len({t.dtype for t in ts}) != 1 or len({int(t.dims[0]) for t in ts}) != 1:
                    continue
                shards = [self._shard(t.name, t) for t in ts]
                if any(n % 16 for _, n, _ in shards[:-1]):  # views start on 16-row tiles
                    continue
                n_tot, k = sum(n for _, n, _ in shards), shards[0][2]
                fused = QMatMul(ts[0].dtype, np.concatenate([r for r, _, _ in shards]), n_tot, k, device=self.device)
                row, biases = 0, []
                for p, t, (_, n, _) in zip(parts, ts, shards):
                    q_map[t.name] = fused.rows(row, n)
                    biases.append(self._bias(f"blk.{i}.{p}.bias"))
                    row += n
                bias = None
                if all(b is not None for b in biases):
                    bias = torch.from_numpy(np.concatenate(biases)).to(self.device)
                self.fused[(i, key)] = (fused, bias, [n for _, n, _ in shards])
        for t in self.file.tensors:
            if t.name in q_map:
                continue
            if t.dtype == 0:
                if t.name.endswith(".bias") and t.name.split(".")[2] in ("attn_q", "attn_k", "attn_v"):
                    dense[t.name] = torch.from_numpy(self._bias(t.name).copy()).to(self.device)
                else:
                    dense[t.name] = torch.from_numpy(self.file.tensor_bytes(t).view(np.float32).copy()).to(self.device)
            elif len(t.dims) == 2:
                raw, n, k = self._shard(t.name, t)  # GGUF [K, N] -> [N, K] (load_gguf.rs:35)
                q_map[t.name] = QMatMul(t.dtype, raw, n, k, device=self.device)
            else:
                raise ConfigError(f"{t.name}: {len(t.dims)}-D tensor of type {t.dtype} is not on this path")
        return Weights(device=self.device, map=dense, q_map=q_map)

    def _check(self, st: int) -> None:
        _raise(st, self.ctx.handle)

    def _lin(self, x: torch.Tensor, ldx: int, m: int, qm: QMatMul, bias: Optional[torch.Tensor]) -> torch.Tensor:
        """y[m, N] (f32) = x . W^T (+ bias), x f32 rows ldx elements apart."""
        y = torch.empty((m, qm.n), dtype=torch.float32, device=self.device)
        b = None if bias is None else bias.data_ptr()
        step = 3 if self.exact_linears else m
        for m0 in range(0, m, step):
            mc = min(step, m - m0)
            self._check(self.L.rtd_qlinear(self.ctx.handle, qm.handle, x.data_ptr() + 4 * m0 * ldx, _lib.DT_F32, ldx,
                                           mc, b, y[m0].data_ptr(), _lib.DT_F32, qm.n, _stream_ptr(self.device)))
        return y

    def _row(self, x: torch.Tensor, ldx: int, m: int, qm: QMatMul) -> torch.Tensor:
        """A row-parallel linear: y[m, N] summed over the ranks, on every rank (the exchange
        fused into the GEMV up to three tokens, the GEMM + all-reduce from four)."""
        if self.world == 1:
            return self._lin(x, ldx, m, qm, None)
        y = torch.empty((m, qm.n), dtype=torch.float32, device=self.device)
        step = 3 if self.exact_linears else m
        for m0 in range(0, m, step):
            mc = min(step, m - m0)
            self._check(self.L.rtd_tp_qlinear_row(self.comm.handle, qm.handle, x.data_ptr() + 4 * m0 * ldx,
                                                  _lib.DT_F32, ldx, mc, None, y[m0].data_ptr(), _lib.DT_F32, qm.n,
                                                  _stream_ptr(self.device)))
        return y

    def _linear(self, x: torch.Tensor, name: str, bias: Optional[str] = None) -> torch.Tensor:
        qm = self.weights.q_map.get(name)
        if qm is None:
            raise MissingWeight(name)
        return self._lin(x, qm.k, x.shape[0], qm, self.weights.map[bias] if bias else None)

    # ---- one call over T tokens, each with its own (sequence, position)
    def _run(self, ids: torch.Tensor, tok_seq: torch.Tensor, tok_pos: torch.Tensor, max_ctx: int,
             logits_rows: Optional[torch.Tensor] = None, trace: Optional[list] = None,
             head_ids: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        """Logits of the call's tokens (rows `logits_rows` only, when given); with `head_ids`
        (int32 [rows]) the greedy ids are written there instead, the pick fused into the LM
        head (rtd_qlinear_argmax: no logits written below four rows), and None is returned."""
        cfg, L, st = self.cfg, self.L, _stream_ptr(self.device)
        T = int(ids.shape[0])
        c = self.ctx.handle
        emb = self.weights.q_map["token_embd.weight"]
        h = torch.empty((T, cfg.hidden), dtype=torch.float32, device=self.device)
        self._check(L.rtd_qembed(c, emb.handle, ids.data_ptr(), T, h.data_ptr(), st))
        n = torch.empty_like(h)
        nh, nkv = self.n_head_l, self.n_kv_l  # this rank's heads
        qr = torch.empty((T, nh * cfg.head_dim), dtype=torch.float32, device=self.device)
        att = torch.empty_like(qr)
        scale = float(np.float32(1.0) / np.sqrt(np.float32(cfg.head_dim)))
        delta = None
        for i in range(cfg.n_layer):
            p = f"blk.{i}"
            self._check(L.rtd_rmsnorm(c, h.data_ptr(), cfg.hidden, None if delta is None else delta.data_ptr(),
                                      _lib.DT_F32, cfg.hidden, self.weights.map[f"{p}.attn_norm.weight"].data_ptr(),
                                      cfg.eps, T, cfg.hidden, n.data_ptr(), _lib.DT_F32, cfg.hidden, st))
            fq = self.fused.get((i, "qkv"))
            if fq is not None:  # q | k | v from one launch: column slices of one output
                qkv = self._lin(n, cfg.hidden, T, fq[0], fq[1])
                w = qkv.shape[1]
                qp, kp = qkv.data_ptr(), qkv.data_ptr() + 4 * fq[2][0]
                vp = kp + 4 * fq[2][1]
                ldq = ldk = ldv = w
            else:
                bias = cfg.has_qkv_bias
                q = self._linear(n, f"{p}.attn_q.weight", f"{p}.attn_q.bias" if bias else None)
                k = self._linear(n, f"{p}.attn_k.weight", f"{p}.attn_k.bias" if bias else None)
                v = self._linear(n, f"{p}.attn_v.weight", f"{p}.attn_v.bias" if bias else None)
                qp, kp, vp, ldq, ldk, ldv = q.data_ptr(), k.data_ptr(), v.data_ptr(), q.shape[1], k.shape[1], v.shape[1]
            self._check(L.rtd_rope_kv_append(c, qp, ldq, kp, ldk, vp, ldv, T, nh, nkv, cfg.head_dim,
                                             cfg.head_dim, cfg.rope_theta, tok_seq.data_ptr(), tok_pos.data_ptr(),
                                             self.cache.table.data_ptr(), self.cache.max_blocks,
                                             self.cache.k[i].data_ptr(), self.cache.v[i].data_ptr(),
                                             self.cache.abi_dtype, qr.data_ptr(), st))
            self._check(L.rtd_attention_paged(c, qr.data_ptr(), T, nh, nkv, cfg.head_dim, scale,
                                              tok_seq.data_ptr(), tok_pos.data_ptr(), self.cache.table.data_ptr(),
                                              self.cache.max_blocks, max_ctx, self.cache.k[i].data_ptr(),
                                              self.cache.v[i].data_ptr(), self.cache.abi_dtype, att.data_ptr(),
                                              _lib.DT_F32, att.shape[1], st))
            o = self._row(att, att.shape[1], T, self.weights.q_map[f"{p}.attn_output.weight"])
            self._check(L.rtd_rmsnorm(c, h.data_ptr(), cfg.hidden, o.data_ptr(), _lib.DT_F32, cfg.hidden,
                                      self.weights.map[f"{p}.ffn_norm.weight"].data_ptr(), cfg.eps, T, cfg.hidden,
                                      n.data_ptr(), _lib.DT_F32, cfg.hidden, st))
            fg = self.fused.get((i, "gate_up"))
            if fg is not None:  # gate | up from one launch; silu(gate) * up written over gate
                gu = self._lin(n, cfg.hidden, T, fg[0], None)
                F, ld = fg[2][0], gu.shape[1]
                self._check(L.rtd_silu_mul(c, gu.data_ptr(), _lib.DT_F32, ld, gu.data_ptr() + 4 * F, _lib.DT_F32, ld,
                                           T, F, gu.data_ptr(), _lib.DT_F32, ld, st))
                delta = self._row(gu, ld, T, self.weights.q_map[f"{p}.ffn_down.weight"])
            else:
                g = self._linear(n, f"{p}.ffn_gate.weight")
                u = self._linear(n, f"{p}.ffn_up.weight")
                self._check(L.rtd_silu_mul(c, g.data_ptr(), _lib.DT_F32, g.shape[1], u.data_ptr(), _lib.DT_F32,
                                           u.shape[1], T, g.shape[1], g.data_ptr(), _lib.DT_F32, g.shape[1], st))
                delta = self._row(g, g.shape[1], T, self.weights.q_map[f"{p}.ffn_down.weight"])
            if trace is not None:  # the residual stream after layer i (a diagnostic copy)
                trace.append((h + delta).clone())
        self._check(L.rtd_rmsnorm(c, h.data_ptr(), cfg.hidden, delta.data_ptr(), _lib.DT_F32, cfg.hidden,
                                  self.weights.map["output_norm.weight"].data_ptr(), cfg.eps, T, cfg.hidden,
                                  n.data_ptr(), _lib.DT_F32, cfg.hidden, st))
        rows = n if logits_rows is None else n.index_select(0, logits_rows)
        if head_ids is not None:
            qm = self.weights.q_map.get("output.weight")
            if qm is None:
                raise MissingWeight("output.weight")
            m = int(rows.shape[0])
            lg = None if m < 4 else torch.empty((m, qm.n), dtype=torch.float32, device=self.device)
            self._check(L.rtd_qlinear_argmax(c, qm.handle, rows.data_ptr(), _lib.DT_F32, cfg.hidden, m, None,
                                             None if lg is None else lg.data_ptr(), _lib.DT_F32, qm.n,
                                             head_ids.data_ptr(), st))
            return None
        return self._linear(rows, "output.weight")

    def _tokens(self, values: Sequence[int]) -> torch.Tensor:
        return torch.tensor(np.asarray(values, dtype=np.int32), device=self.device)

    def forward(self, ids: Sequence[int], q0: int, seq: int = 0, last_only: bool = False,
                trace: Optional[list] = None) -> torch.Tensor:
        """Logits [t, vocab] (f32) of `ids` at positions q0 .. q0 + t - 1 of sequence `seq`
        (qwen2.rs:217-229); `last_only` computes the LM head for the last position only."""
        t = len(ids)
        if t == 0:
            raise ConfigError("forward of no tokens")
        self.cache.reserve(seq, q0 + t)
        self.cache.sync_table()
        ids_d = self._tokens(ids)
        seq_d = self._tokens([seq] * t)
        pos_d = self._tokens(range(q0, q0 + t))
        rows = self._tokens([t - 1]) if last_only else None
        return self._run(ids_d, seq_d, pos_d, q0 + t, rows, trace)

    def decode_batch(self, ids: Sequence[int], seqs: Sequence[int], positions: Sequence[int]) -> torch.Tensor:
        """One token for each of several sequences (batched decode); logits [b, vocab]."""
        for s, p in zip(seqs, positions):
            self.cache.reserve(int(s), int(p) + 1)
        self.cache.sync_table()
        return self._run(self._tokens(ids), self._tokens(seqs), self._tokens(positions), int(max(positions)) + 1)

    def greedy_graph(self, prompt: Sequence[int], steps: int, seq: int = 0):
        """Greedy decode of `steps` tokens after the prompt with one decode step captured as
        a CUDA graph: the step reads its token and position from device tensors, and its
        last kernel (the LM head with the greedy pick in its epilogue, rtd_qlinear_argmax:
        no logits are written) puts the next token where the next replay reads it, so no
        step waits for the host.  Returns (ids on the device [steps], the graph, a
        replay function) -- the timing target of the bench's decode figure."""
        logits = self.forward(list(prompt), 0, seq=seq, last_only=True)
        total = len(prompt) + steps
        self.cache.reserve(seq, total)
        self.cache.sync_table()
        tok = self.argmax(logits[-1:])
        pos = torch.tensor([len(prompt)], dtype=torch.int32, device=self.device)
        seq_d = torch.tensor([seq], dtype=torch.int32, device=self.device)
        out = torch.empty((steps,), dtype=torch.int32, device=self.device)

        def step():
            self._run(tok, seq_d, pos, total, head_ids=tok)
            pos.add_(1)

        # one eager step first (kernel attributes are configured outside capture); the
        # graph's first replay recomputes the same position from the same token
        tok0 = tok.clone()
        step()
        torch.cuda.synchronize(self.device)
        tok.copy_(tok0)
        pos.fill_(len(prompt))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            step()
        state = {"i": 0}

        def replay():
            g.replay()
            out[state["i"]:state["i"] + 1].copy_(tok)
            state["i"] += 1

        return out, g, replay

    def argmax(self, logits: torch.Tensor) -> torch.Tensor:
        """Greedy ids of the rows of `logits` (SubstratePort::argmax, decode/sample.rs:11-18)."""
        x = logits.contiguous()
        out = torch.empty((x.shape[0],), dtype=torch.int32, device=self.device)
        self._check(self.L.rtd_argmax(self.ctx.handle, x.data_ptr(), x.shape[1], x.shape[0], x.shape[1],
                                      out.data_ptr(), _stream_ptr(self.device)))
        return out


class Session:
    """Greedy generation for one sequence (crates/runtimed-model/src/decode/session.rs:157-166)."""

    def __init__(self, model: Qwen2Model, seq: int = 0):
        self.model, self.seq, self.pos = model, seq, 0

    def prefill(self, prompt: Sequence[int]) -> torch.Tensor:
        self.model.cache.release(self.seq)
        logits = self.model.forward(list(prompt), 0, seq=self.seq, last_only=True)
        self.pos = len(prompt)
        return logits[-1]

    def step(self, token: int) -> torch.Tensor:
        logits = self.model.forward([int(token)], self.pos, seq=self.seq)
        self.pos += 1
        return logits[-1]

    def truncate(self, length: int) -> None:
        self.model.cache.truncate(self.seq, length)
        self.pos = length

    def greedy(self, prompt: Sequence[int], steps: int):
        """(ids, logits rows) of `steps` greedy tokens after the prompt."""
        logits = self.prefill(prompt)
        out, per = [], [logits]
        for _ in range(steps):
            nxt = int(self.model.argmax(logits[None, :])[0])
            out.append(nxt)
            logits = self.step(nxt)
            per.append(logits)
        return out, per
