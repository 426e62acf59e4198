"""Tensor-parallel quantized linears (one process per GPU).

Mirrors the reference's Megatron-style layers:

- `ColumnParallelLinear`: crates/runtimed-model/src/tp/column_linear.rs:20-61. It splits
  the N output rows, so every rank holds whole GGUF rows and no data is re-quantized.
  Its forward needs no exchange.
- `RowParallelLinear`: crates/runtimed-model/src/tp/row_linear.rs:20-66. It splits K on
  superblock boundaries. The reduction that the reference runs as a separate
  `ring_all_reduce` (crates/runtimed-model/src/tp/ring_reduce.rs:7-65) runs inside
  `rtd_tp_qlinear_row`: fused into the GEMV epilogue for decode-sized M (tile partials
  cross NVLink as peer stores), a two-shot all-reduce kernel after the tensor-core GEMM
  from four tokens on; every rank writes the full y.

`forward_nccl` computes the same result with an NCCL all-reduce, as the measured
comparison; `forward_ar` runs the unfused GEMV followed by this library's all-reduce.

- `VocabParallelHead`: the LM head (qwen2.rs:224-228) split by vocabulary rows, with the
  greedy pick (decode/sample.rs:11-18) distributed: every rank picks in its GEMV epilogue
  and outputs one packed 8-byte key per token, and the keys of all ranks are gathered and
  combined by an unsigned maximum (`combine_keys`), so no logits cross NVLink.
The shard helpers work on raw GGUF bytes and are plain numpy, so the host side can be
tested without a GPU.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from . import _lib
from .errors import ConfigError, ShapeError

BLOCK = {8: (32, 34), 12: (256, 144), 14: (256, 210)}  # ggml type -> (elements, bytes)


def _geometry(ggml_type: int):
    if ggml_type not in BLOCK:
        raise ConfigError(f"ggml type {ggml_type} has no tensor-parallel shard layout")
    return BLOCK[ggml_type]


def shard_rows(raw, ggml_type: int, n: int, k: int, rank: int, world: int) -> np.ndarray:
    """Bytes of output rows [rank*n/world, (rank+1)*n/world) (column-parallel shard)."""
    if world == 0:
        raise ConfigError("TP size cannot be zero")
    if n % world:
        raise ConfigError(f"Output dimension {n} not divisible by TP size {world}")
    elems, bb = _geometry(ggml_type)
    row = (k // elems) * bb
    raw = np.asarray(raw, dtype=np.uint8).reshape(-1)
    if raw.size != n * row:
        raise ShapeError("tp_weight", [n * row], [raw.size])
    rows = n // world
    return raw[rank * rows * row:(rank + 1) * rows * row].copy()


def shard_cols(raw, ggml_type: int, n: int, k: int, rank: int, world: int) -> np.ndarray:
    """Bytes of input columns [rank*k/world, (rank+1)*k/world) of every row (row-parallel
    shard).  The split must fall on superblock boundaries."""
    if world == 0:
        raise ConfigError("TP size cannot be zero")
    if k % world:
        raise ConfigError(f"Input dimension {k} not divisible by TP size {world}")
    elems, bb = _geometry(ggml_type)
    ks = k // world
    if ks % elems:
        raise ConfigError(f"Input shard {ks} is not a multiple of the {elems}-element block")
    raw = np.asarray(raw, dtype=np.uint8).reshape(-1)
    nb = k // elems
    if raw.size != n * nb * bb:
        raise ShapeError("tp_weight", [n * nb * bb], [raw.size])
    blocks = raw.reshape(n, nb, bb)
    per = ks // elems
    return np.ascontiguousarray(blocks[:, rank * per:(rank + 1) * per, :]).reshape(-1)


class TpComm:
    """Row-reduction communicator of one rank: `rtd_tp_comm_create` on every rank, the
    IPC handles gathered over torch.distributed (rank order), then `rtd_tp_comm_open`."""

    HANDLE_BYTES = 64

    def __init__(self, ctx, rank: int, world: int, max_n: int, group=None):
        import torch.distributed as dist

        self.ctx, self.rank, self.world, self.max_n = ctx, rank, world, int(max_n)
        L = _lib.lib()
        self.handle = ctypes.c_void_p()
        h = (ctypes.c_ubyte * self.HANDLE_BYTES)()
        _lib.check(L.rtd_tp_comm_create(ctx.handle, rank, world, self.max_n, ctypes.byref(self.handle), h),
                   ctx.handle)
        mine = bytes(h)
        everyone = [None] * world
        dist.all_gather_object(everyone, mine, group=group)
        allh = (ctypes.c_ubyte * (self.HANDLE_BYTES * world)).from_buffer_copy(b"".join(everyone))
        _lib.check(L.rtd_tp_comm_open(self.handle, allh), ctx.handle)

    def allreduce(self, partial, bias=None, out_dtype=None):
        """Sum of every rank's f32 partial [M, N] (+ bias once), on every rank
        (rtd_tp_allreduce: two-shot over NVLink; replaces ring_all_reduce,
        crates/runtimed-model/src/tp/ring_reduce.rs:7-34)."""
        import torch
        from .weights import _DT, _stream_ptr

        p = partial.to(torch.float32)
        n = int(p.shape[-1])
        p2 = p.reshape(-1, n).contiguous()
        m = int(p2.shape[0])
        out_dtype = out_dtype or torch.float32
        y = torch.empty((m, n), dtype=out_dtype, device=p2.device)
        b = None
        if bias is not None:
            b = bias.to(device=p2.device, dtype=torch.float32).contiguous()
        st = _lib.lib().rtd_tp_allreduce(self.handle, p2.data_ptr(), n, m, n, None if b is None else b.data_ptr(),
                                         y.data_ptr(), _DT[out_dtype], n, _stream_ptr(p2.device))
        _lib.check(st, self.ctx.handle)
        return y.reshape(*partial.shape[:-1], n)

    def close(self) -> None:
        if getattr(self, "handle", None):
            _lib.lib().rtd_tp_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ColumnParallelLinear:
    """Output rows split across ranks; y_rank = x . W_rank^T + b_rank."""

    def __init__(self, weight, bias, rank: int, tp_size: int):
        self.weight, self.bias, self.rank, self.tp_size = weight, bias, rank, tp_size

    @classmethod
    def from_full_weight(cls, raw, ggml_type: int, n: int, k: int, full_bias, rank: int, tp_size: int,
                         device="cuda:0") -> "ColumnParallelLinear":
        from .weights import QMatMul

        shard = shard_rows(raw, ggml_type, n, k, rank, tp_size)
        rows = n // tp_size
        qm = QMatMul(ggml_type, shard, rows, k, device=device)
        bias = None
        if full_bias is not None:
            import torch

            b = torch.as_tensor(np.asarray(full_bias, dtype=np.float32))
            bias = b[rank * rows:(rank + 1) * rows].contiguous().to(qm.device)
        return cls(qm, bias, rank, tp_size)

    def forward(self, x):
        return self.weight.forward(x, bias=self.bias)


class RowParallelLinear:
    """Input columns split across ranks.  With a communicator, forward returns the
    full reduced y on every rank (bias added once); without one it returns the rank's
    partial with the bias on rank 0 only, as the reference does."""

    def __init__(self, weight, bias, rank: int, tp_size: int, comm: Optional[TpComm] = None):
        self.weight, self.bias, self.rank, self.tp_size, self.comm = weight, bias, rank, tp_size, comm

    @classmethod
    def from_full_weight(cls, raw, ggml_type: int, n: int, k: int, full_bias, rank: int, tp_size: int,
                         comm: Optional[TpComm] = None, device="cuda:0") -> "RowParallelLinear":
        from .weights import QMatMul

        shard = shard_cols(raw, ggml_type, n, k, rank, tp_size)
        qm = QMatMul(ggml_type, shard, n, k // tp_size, device=device)
        bias = None
        if full_bias is not None:
            import torch

            bias = torch.as_tensor(np.asarray(full_bias, dtype=np.float32)).contiguous().to(qm.device)
        return cls(qm, bias, rank, tp_size, comm)

    def _flat(self, x):
        import torch

        if x.shape[-1] != self.weight.k:
            raise ShapeError("row_parallel_linear", [self.weight.k], list(x.shape))
        m = 1
        for d in x.shape[:-1]:
            m *= int(d)
        return x.reshape(m, self.weight.k).contiguous().to(self.weight.device), m

    def forward(self, x):
        import torch
        from .weights import _DT, _stream_ptr

        if self.comm is None or self.tp_size == 1:
            b = self.bias if (self.rank == 0 or self.tp_size == 1) else None
            return self.weight.forward(x, bias=b)
        x2, m = self._flat(x)
        if x2.dtype not in _DT:
            x2 = x2.to(torch.float32)
        y = torch.empty((m, self.weight.n), dtype=x2.dtype, device=self.weight.device)
        bp = None if self.bias is None else self.bias.data_ptr()
        st = _lib.lib().rtd_tp_qlinear_row(self.comm.handle, self.weight.handle, x2.data_ptr(), _DT[x2.dtype],
                                           self.weight.k, m, bp, y.data_ptr(), _DT[y.dtype], self.weight.n,
                                           _stream_ptr(self.weight.device))
        _lib.check(st, self.weight.ctx.handle)
        return y.reshape(*x.shape[:-1], self.weight.n)

    def forward_ar(self, x):
        """Local partial GEMV (f32), then this library's two-shot all-reduce kernel."""
        import torch

        y = self.weight.forward(x, out_dtype=torch.float32)
        out = x.dtype if x.dtype in (torch.float16, torch.bfloat16, torch.float32) else torch.float32
        return self.comm.allreduce(y, bias=self.bias, out_dtype=out)

    def forward_nccl(self, x, group=None):
        """The comparison path: local partial GEMV, then an NCCL all-reduce."""
        import torch
        import torch.distributed as dist

        y = self.weight.forward(x, out_dtype=torch.float32)
        dist.all_reduce(y, group=group)
        if self.bias is not None:
            y = y + self.bias
        return y.to(x.dtype) if x.dtype in (torch.float16, torch.bfloat16) else y


# ---- the vocabulary-parallel LM head and its distributed greedy pick
_TOP = -(1 << 63)  # XOR with this maps unsigned 64-bit order onto signed order


def pack_key(value: float, row: int) -> int:
    """The packed key of output `value` at global row `row`, as the GEMV epilogue forms it
    (u64 as a Python int): the f32 order mapped onto unsigned order (-0 as +0) in the high
    word, 0xFFFFFFFF - row in the low word, so the larger key is the larger value and,
    among equal values, the lower row.  NaN has no key (0)."""
    v = np.float32(value)
    if np.isnan(v):
        return 0
    u = int(np.float32(0.0 if v == 0 else v).view(np.uint32))
    u = (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)
    return (u << 32) | (0xFFFFFFFF - int(row))


def combine_keys(keys):
    """Greedy ids (int32 [M]) from every rank's keys ([world, M] int64 holding u64 bit
    patterns): the unsigned maximum per token, its row decoded; 0 where every key is 0."""
    import torch

    k = torch.as_tensor(keys, dtype=torch.int64)
    if k.dim() == 1:
        k = k[None, :]
    best = (k ^ _TOP).max(dim=0).values ^ _TOP
    ids = torch.where(best == 0, torch.zeros_like(best), 0xFFFFFFFF - (best & 0xFFFFFFFF))
    return ids.to(torch.int32)


class VocabParallelHead:
    """output.weight split by vocabulary rows: rank r holds rows [r V / world, (r + 1) V /
    world).  `greedy` returns the whole head's greedy ids on every rank: the local pick as
    keys (rtd_qlinear_argmax_keys), an all-gather of M keys per rank, `combine_keys`."""

    def __init__(self, weight, row0: int, rank: int, tp_size: int, group=None):
        self.weight, self.row0, self.rank, self.tp_size, self.group = weight, int(row0), rank, tp_size, group

    @classmethod
    def from_full_weight(cls, raw, ggml_type: int, n: int, k: int, rank: int, tp_size: int, device="cuda:0",
                         group=None) -> "VocabParallelHead":
        from .weights import QMatMul

        shard = shard_rows(raw, ggml_type, n, k, rank, tp_size)
        rows = n // tp_size
        return cls(QMatMul(ggml_type, shard, rows, k, device=device), rank * rows, rank, tp_size, group)

    def local_keys(self, x):
        return self.weight.greedy_keys(x, row0=self.row0)

    def greedy(self, x):
        return gather_greedy(self.local_keys(x), self.tp_size, self.group)


def gather_greedy(keys, tp_size: int, group=None):
    """Every rank's keys [M] gathered (torch.distributed, M int64 a rank) and combined:
    the whole head's greedy ids on every rank."""
    if tp_size == 1:
        return combine_keys(keys)
    import torch
    import torch.distributed as dist

    everyone = [torch.empty_like(keys) for _ in range(tp_size)]
    dist.all_gather(everyone, keys.contiguous(), group=group)
    return combine_keys(torch.stack(everyone))
