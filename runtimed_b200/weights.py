"""Host-side operator surface: the reference's Weights / QMatMul / Fp8Weight, on the C ABI.

Mirrors, with the same names, argument meaning and error behaviour:
  * ``QMatMul``  -- candle's QMatMul::QTensor as built by load_quantized_tensor
                    (crates/runtimed-model/src/weights/load_gguf.rs:28-38): forward,
                    embedding, dequantize, storage size;
  * ``Fp8Weight`` -- crates/runtimed-model/src/weights/fp8_weight.rs:9-97;
  * ``Weights``  -- crates/runtimed-model/src/weights/store.rs:12-101 (map / q_map,
                    q_matmul, resident_bytes, get) with linear / linear_bias
                    (linear_layer.rs:45-118) and embed (embed_layer.rs:16-57).

Tensors are torch tensors (device memory, streams); every byte of arithmetic runs
in libruntimed_b200.so.  There is no CPU path: a CPU tensor handed to a device
weight is moved to the weight's device first, as the reference does with
``x.to_device(dev)`` (linear_layer.rs:49).
"""
from __future__ import annotations

import ctypes
from typing import Dict, Optional

import numpy as np
import torch

from . import _lib
from ._lib import check
from .errors import ConfigError, GgufError, MissingWeight, ShapeError

_DT = {torch.float32: _lib.DT_F32, torch.float16: _lib.DT_F16, torch.bfloat16: _lib.DT_BF16}
_BLOCK = {_lib.TYPE_Q8_0: (32, 34), _lib.TYPE_Q4_K: (256, 144), _lib.TYPE_Q6_K: (256, 210)}


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _raise(status: int, ctx_handle) -> None:
    """Map an rtd_status to the reference's ModelError variants."""
    if status == _lib.RTD_OK:
        return
    msg = _lib.lib().rtd_last_error(ctx_handle)
    text = msg.decode() if msg else ""
    if status in (_lib.RTD_ERR_UNSUPPORTED, _lib.RTD_ERR_TRUNCATED):
        raise GgufError(text)
    if status == _lib.RTD_ERR_SHAPE:
        raise ShapeError("rtd", [], [])  # callers check shapes first; this is a backstop
    raise ConfigError(f"rtd status {status}: {text}")


class Context:
    """One CUDA device bound to the library (rtd_init); owns the kernels' workspace."""

    _by_device: Dict[int, "Context"] = {}

    def __init__(self, device: int = 0):
        h = ctypes.c_void_p()
        check(_lib.lib().rtd_init(device, ctypes.byref(h)))
        self.handle = h
        self.device = torch.device("cuda", device)

    @classmethod
    def for_device(cls, device) -> "Context":
        idx = torch.device(device).index
        idx = torch.cuda.current_device() if idx is None else idx
        ctx = cls._by_device.get(idx)
        if ctx is None:
            ctx = cls(idx)
            cls._by_device[idx] = ctx
        return ctx

    def check_device_status(self, stream: Optional[int] = None) -> None:
        s = _stream_ptr(self.device) if stream is None else stream
        _raise(_lib.lib().rtd_check_device_status(self.handle, s), self.handle)

    def close(self) -> None:
        if self.handle:
            _lib.lib().rtd_destroy(self.handle)
            self.handle = None


class QMatMul:
    """A quantized [N, K] matrix resident on one device (candle QMatMul::QTensor)."""

    def __init__(self, ggml_type: int, raw, n: int, k: int, device="cuda:0"):
        if ggml_type not in _BLOCK:
            raise GgufError(f"unsupported ggml type {ggml_type} for QMatMul on this path")
        self.ctx = Context.for_device(device)
        self.ggml_type = int(ggml_type)
        self.n, self.k = int(n), int(k)
        buf = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if isinstance(raw, (bytes, bytearray))
                                   else np.asarray(raw, dtype=np.uint8).reshape(-1))
        h = ctypes.c_void_p()
        st = _lib.lib().rtd_qweight_upload(self.ctx.handle, self.ggml_type, buf.ctypes.data_as(ctypes.c_void_p),
                                           buf.size, self.n, self.k, ctypes.byref(h))
        if st == _lib.RTD_ERR_SHAPE:
            elems = _BLOCK[self.ggml_type][0]
            raise GgufError(f"{self.k} not a multiple of {elems}")
        _raise(st, self.ctx.handle)
        self.handle = h
        raw_b, dev_b = ctypes.c_size_t(), ctypes.c_size_t()
        check(_lib.lib().rtd_qweight_info(h, None, None, None, ctypes.byref(raw_b), ctypes.byref(dev_b)))
        self._raw_bytes, self._dev_bytes = raw_b.value, dev_b.value

    # -- candle QTensor surface
    @property
    def shape(self):
        return (self.n, self.k)

    @property
    def device(self) -> torch.device:
        return self.ctx.device

    def storage_size_in_bytes(self) -> int:
        return self._raw_bytes

    def device_bytes(self) -> int:
        return self._dev_bytes

    def forward(self, x: torch.Tensor, bias: Optional[torch.Tensor] = None,
                out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """y = x . W^T (+ bias); leading dims of x are kept, the last becomes N."""
        if x.dim() == 0 or x.shape[-1] != self.k:
            raise ShapeError("qmatmul", [self.k], list(x.shape))
        if x.dtype not in _DT:
            x = x.to(torch.float32)
        if x.device != self.device:
            x = x.to(self.device)
        m = 1
        for d in x.shape[:-1]:
            m *= int(d)
        x2 = x.reshape(m, self.k)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        out_dtype = out_dtype or x.dtype
        y = torch.empty((m, self.n), dtype=out_dtype, device=self.device)
        b = None
        if bias is not None:
            b = bias.to(device=self.device, dtype=torch.float32).contiguous()
            if b.numel() != self.n:
                raise ShapeError("bias", [self.n], list(bias.shape))
        st = _lib.lib().rtd_qlinear(self.ctx.handle, self.handle, x2.data_ptr(), _DT[x2.dtype], self.k, m,
                                    None if b is None else b.data_ptr(), y.data_ptr(), _DT[out_dtype], self.n,
                                    _stream_ptr(self.device))
        _raise(st, self.ctx.handle)
        return y.reshape(*x.shape[:-1], self.n)

    __call__ = forward

    def greedy(self, x: torch.Tensor, bias: Optional[torch.Tensor] = None,
               logits: Optional[torch.Tensor] = None) -> torch.Tensor:
        """int32 ids [m] of the largest output of each row of x: the LM head followed by
        the greedy pick (qwen2.rs:224-228, sample.rs:11-18) in one call.  Below four rows
        the pick runs in the GEMV's epilogue and the logits are written only into
        `logits` ([m, N] f32) when it is given; from four rows they are required."""
        if x.dim() != 2 or x.shape[1] != self.k:
            raise ShapeError("qmatmul_greedy", [-1, self.k], list(x.shape))
        if x.dtype not in _DT:
            x = x.to(torch.float32)
        x2 = x.to(self.device).contiguous()
        m = x2.shape[0]
        if logits is not None and (logits.dtype != torch.float32 or tuple(logits.shape) != (m, self.n)
                                   or not logits.is_contiguous()):
            raise ShapeError("logits", [m, self.n], list(logits.shape))
        b = None
        if bias is not None:
            b = bias.to(device=self.device, dtype=torch.float32).contiguous()
            if b.numel() != self.n:
                raise ShapeError("bias", [self.n], list(bias.shape))
        ids = torch.empty((m,), dtype=torch.int32, device=self.device)
        st = _lib.lib().rtd_qlinear_argmax(self.ctx.handle, self.handle, x2.data_ptr(), _DT[x2.dtype], self.k, m,
                                           None if b is None else b.data_ptr(),
                                           None if logits is None else logits.data_ptr(), _lib.DT_F32, self.n,
                                           ids.data_ptr(), _stream_ptr(self.device))
        _raise(st, self.ctx.handle)
        return ids

    def greedy_keys(self, x: torch.Tensor, row0: int = 0, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Packed greedy keys [m] (int64 holding the u64 bit patterns) of the rows of x against
        this matrix, its rows numbered from `row0` -- one vocabulary shard's share of a
        distributed greedy pick (rtd_qlinear_argmax_keys; combine with tp.combine_keys)."""
        if x.dim() != 2 or x.shape[1] != self.k:
            raise ShapeError("qmatmul_greedy", [-1, self.k], list(x.shape))
        if x.dtype not in _DT:
            x = x.to(torch.float32)
        x2 = x.to(self.device).contiguous()
        b = None
        if bias is not None:
            b = bias.to(device=self.device, dtype=torch.float32).contiguous()
            if b.numel() != self.n:
                raise ShapeError("bias", [self.n], list(bias.shape))
        keys = torch.empty((x2.shape[0],), dtype=torch.int64, device=self.device)
        st = _lib.lib().rtd_qlinear_argmax_keys(self.ctx.handle, self.handle, x2.data_ptr(), _DT[x2.dtype], self.k,
                                                x2.shape[0], None if b is None else b.data_ptr(), int(row0),
                                                keys.data_ptr(), _stream_ptr(self.device))
        _raise(st, self.ctx.handle)
        return keys

    def embedding(self, ids: torch.Tensor) -> torch.Tensor:
        """f32 rows ids of the dequantized matrix (QMatMul::embedding)."""
        ids_d = ids.to(device=self.device, dtype=torch.int32).reshape(-1).contiguous()
        y = torch.empty((ids_d.numel(), self.k), dtype=torch.float32, device=self.device)
        st = _lib.lib().rtd_qembed(self.ctx.handle, self.handle, ids_d.data_ptr(), ids_d.numel(), y.data_ptr(),
                                   _stream_ptr(self.device))
        _raise(st, self.ctx.handle)
        return y

    def dequantize(self) -> torch.Tensor:
        """The whole matrix as f32 [N, K], bit-exact with the reference decoders."""
        y = torch.empty((self.n, self.k), dtype=torch.float32, device=self.device)
        st = _lib.lib().rtd_qdequant(self.ctx.handle, self.handle, y.data_ptr(), _stream_ptr(self.device))
        _raise(st, self.ctx.handle)
        return y

    def to_device(self, device) -> "QMatMul":
        """A copy on `device` (the same device gives a second, distinct device copy),
        made without a host round trip (rtd_qweight_to_device)."""
        ctx = Context.for_device(device)
        h = ctypes.c_void_p()
        _raise(_lib.lib().rtd_qweight_to_device(self.handle, ctx.handle, ctypes.byref(h)), ctx.handle)
        out = QMatMul.__new__(QMatMul)
        out.ctx, out.ggml_type, out.n, out.k = ctx, self.ggml_type, self.n, self.k
        out.handle = h
        out._raw_bytes, out._dev_bytes = self._raw_bytes, self._dev_bytes
        return out

    def rows(self, row0: int, n: int) -> "QMatMul":
        """Rows [row0, row0 + n) as a QMatMul sharing this one's device memory (row0 a
        multiple of 16; rtd_qweight_rows).  The view keeps a reference to its parent."""
        h = ctypes.c_void_p()
        _raise(_lib.lib().rtd_qweight_rows(self.handle, int(row0), int(n), ctypes.byref(h)), self.ctx.handle)
        out = QMatMul.__new__(QMatMul)
        out.ctx, out.ggml_type, out.n, out.k = self.ctx, self.ggml_type, int(n), self.k
        out.handle = h
        out._raw_bytes = self._raw_bytes // max(self.n, 1) * int(n)
        out._dev_bytes = 0  # shares the parent's memory
        out._parent = self
        return out

    def free(self) -> None:
        if getattr(self, "handle", None):
            _lib.lib().rtd_qweight_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class Fp8Weight:
    """FP8 E4M3 weight [out, in] with a per-channel (or per-tensor) f32 scale."""

    def __init__(self, weight, scale, in_dim: int, out_dim: int, device="cuda:0"):
        w = np.ascontiguousarray(np.asarray(weight, dtype=np.uint8))
        s = np.ascontiguousarray(np.asarray(scale, dtype=np.float32))
        if list(w.shape) != [out_dim, in_dim]:
            raise ShapeError("fp8_weight", [out_dim, in_dim], list(w.shape))
        if list(s.shape) not in ([out_dim], [out_dim, 1]) and s.size != 1:
            raise ShapeError("fp8_scale", [out_dim], list(s.shape))
        self.in_dim, self.out_dim = int(in_dim), int(out_dim)
        self.ctx = Context.for_device(device)
        h = ctypes.c_void_p()
        s = s.reshape(-1)
        _raise(_lib.lib().rtd_fp8weight_upload(self.ctx.handle, w.ctypes.data_as(ctypes.c_void_p),
                                               s.ctypes.data_as(ctypes.c_void_p), s.size, out_dim, in_dim,
                                               ctypes.byref(h)), self.ctx.handle)
        self.handle = h
        self._bytes = w.size + 4 * s.size

    @property
    def device(self) -> torch.device:
        return self.ctx.device

    def resident_bytes(self) -> int:
        return self._bytes

    def forward(self, x: torch.Tensor, mode: str = "w8a16") -> torch.Tensor:
        """y = x . (E4M3(W) * s)^T.  mode "w8a8" first encodes x to E4M3 like the
        reference CUDA path; output is f16 for f16 input, else f32 (fp8_gemm.rs:106)."""
        if x.shape[-1] != self.in_dim:
            raise ShapeError("fp8_gemm", [self.in_dim], list(x.shape))
        if x.dtype not in _DT:
            x = x.to(torch.float32)
        x = x.to(self.device)
        m = 1
        for d in x.shape[:-1]:
            m *= int(d)
        x2 = x.reshape(m, self.in_dim).contiguous()
        out_dtype = torch.float16 if x.dtype == torch.float16 else torch.float32
        y = torch.empty((x2.shape[0], self.out_dim), dtype=out_dtype, device=self.device)
        m = {"w8a16": _lib.FP8_W8A16, "w8a8": _lib.FP8_W8A8}[mode]
        st = _lib.lib().rtd_fp8_linear(self.ctx.handle, self.handle, x2.data_ptr(), _DT[x2.dtype], self.in_dim,
                                       x2.shape[0], y.data_ptr(), _DT[out_dtype], self.out_dim, m,
                                       _stream_ptr(self.device))
        _raise(st, self.ctx.handle)
        return y.reshape(*x.shape[:-1], self.out_dim)

    def free(self) -> None:
        if getattr(self, "handle", None):
            _lib.lib().rtd_fp8weight_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _round_half_away(v: np.ndarray) -> np.ndarray:
    """f32::round: halves go away from zero (numpy's round goes to even)."""
    return (np.sign(v) * np.floor(np.abs(v) + np.float32(0.5))).astype(np.float32)


def repack_marlin_tiles(weight, scales):
    """Dense [out, in] weight and per-row scales -> (packed u32 [ceil(in / 32), out, 4],
    scales), as repack_marlin_tiles does (crates/runtimed-model/src/ops/marlin_gemv.rs:64-97):
    q = clamp(round(w / s) + 8, 0, 15) in f32 (1 / s taken as 1 when |s| <= 1e-12), eight
    nibbles to a word, k past `in` padded with 8.  Host-side packing, as in the reference."""
    w = np.asarray(weight, dtype=np.float32)
    if w.ndim != 2:
        raise ConfigError(f"weight must be 2D, got {list(w.shape)}")
    out_dim, in_dim = w.shape
    s = np.asarray(scales, dtype=np.float32).reshape(-1)
    if s.size != out_dim:
        raise ShapeError("scales", [out_dim], [int(s.size)])
    inv = np.where(np.abs(s) > np.float32(1e-12), np.float32(1.0) / s, np.float32(1.0)).astype(np.float32)
    kc = (in_dim + 31) // 32
    q = np.full((out_dim, kc * 32), 8, dtype=np.uint32)
    if in_dim:
        q[:, :in_dim] = np.clip(_round_half_away(w * inv[:, None]) + np.float32(8.0), 0.0, 15.0).astype(np.uint32)
    nib = q.reshape(out_dim, kc, 4, 8)
    words = np.zeros((out_dim, kc, 4), dtype=np.uint32)
    for i in range(8):
        words |= nib[..., i] << np.uint32(4 * i)
    return np.ascontiguousarray(words.transpose(1, 0, 2)), s


class MarlinWeight(QMatMul):
    """INT4 Marlin weight (crates/runtimed-model/src/ops/marlin_gemv.rs:11-62): packed u32
    [ceil(in / 32), out, 4] and f32 scales [out] (or [out, 1]); value (q - 8) * s[n].
    forward runs the library's tensor-core paths (rtd_qlinear on an rtd_marlin_upload
    handle) for any token count; dequantize is bit-exact with MarlinWeight::dequantize."""

    def __init__(self, packed, scales, in_dim: int, out_dim: int, device="cuda:0"):
        p = np.asarray(packed)
        if p.dtype != np.uint32:
            raise ConfigError(f"marlin packed must be U32, got {p.dtype}")
        s = np.asarray(scales, dtype=np.float32)
        if list(s.shape) not in ([out_dim], [out_dim, 1]):
            raise ShapeError("marlin_scales", [out_dim], list(s.shape))
        kc = (int(in_dim) + 31) // 32
        if p.size < kc * out_dim * 4:
            raise ShapeError("marlin_packed", [kc, out_dim, 4], list(p.shape))
        self.ctx = Context.for_device(device)
        self.ggml_type = _lib.TYPE_INT4_MARLIN
        self.n, self.k = int(out_dim), int(in_dim)
        p = np.ascontiguousarray(p.reshape(-1)[: kc * out_dim * 4])
        s = np.ascontiguousarray(s.reshape(-1))
        h = ctypes.c_void_p()
        _raise(_lib.lib().rtd_marlin_upload(self.ctx.handle, p.ctypes.data_as(ctypes.c_void_p),
                                            s.ctypes.data_as(ctypes.c_void_p), self.n, self.k, ctypes.byref(h)),
               self.ctx.handle)
        self.handle = h
        raw_b, dev_b = ctypes.c_size_t(), ctypes.c_size_t()
        check(_lib.lib().rtd_qweight_info(h, None, None, None, ctypes.byref(raw_b), ctypes.byref(dev_b)))
        self._raw_bytes, self._dev_bytes = raw_b.value, dev_b.value
        self.packed, self.scales = p.reshape(kc, self.n, 4), s  # the struct's host tensors

    @property
    def in_dim(self) -> int:
        return self.k

    @property
    def out_dim(self) -> int:
        return self.n

    def resident_bytes(self) -> int:
        return self._raw_bytes

    def forward(self, x: torch.Tensor, bias: Optional[torch.Tensor] = None,
                out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        if x.shape[-1] != self.k:
            raise ShapeError("marlin_gemv", [self.k], list(x.shape))
        return super().forward(x, bias, out_dtype)

    __call__ = forward

    def embedding(self, ids: torch.Tensor) -> torch.Tensor:
        raise ConfigError("INT4 Marlin weights are not an embedding format")


def marlin_gemv(x: torch.Tensor, w: MarlinWeight) -> torch.Tensor:
    """y = x @ (w * scale)^T (marlin_gemv.rs:112-119), in x's dtype."""
    return w.forward(x)


def fp8_encode(x: torch.Tensor) -> torch.Tensor:
    """Device E4M3 encoding of f32 x with the reference rounding (uint8 codes)."""
    x = x.to(torch.float32).contiguous()
    ctx = Context.for_device(x.device)
    out = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    _raise(_lib.lib().rtd_fp8_encode(ctx.handle, x.data_ptr(), x.numel(), out.data_ptr(), _stream_ptr(x.device)),
           ctx.handle)
    return out


def _is_u32(t) -> bool:
    return (torch.is_tensor(t) and t.dtype == torch.uint32) or (isinstance(t, np.ndarray) and t.dtype == np.uint32)


class Weights:
    """The reference's weight store: dense tensors in ``map``, quantized in ``q_map``."""

    def __init__(self, device="cuda:0", map: Optional[dict] = None, q_map: Optional[dict] = None,
                 fp8_map: Optional[dict] = None):
        self.dev = torch.device(device)
        self.map: Dict[str, torch.Tensor] = dict(map or {})
        self.q_map: Dict[str, QMatMul] = dict(q_map or {})
        self.fp8_map: Dict[str, Fp8Weight] = dict(fp8_map or {})

    @classmethod
    def from_parts(cls, device, map: dict) -> "Weights":
        """Weights::from_parts (store.rs:22-29): dense tensors only."""
        return cls(device=device, map=map)

    @classmethod
    def from_quantized(cls, device, map: dict, q_map: dict) -> "Weights":
        """Weights::from_quantized (store.rs:31-43): dense and quantized entries."""
        return cls(device=device, map=map, q_map=q_map)

    def device(self) -> torch.device:
        return self.dev

    @staticmethod
    def cuda_available(ordinal: int) -> bool:
        """Weights::cuda_available (store.rs:116-126)."""
        return torch.cuda.is_available() and 0 <= int(ordinal) < torch.cuda.device_count()

    def q_matmul(self, name: str) -> Optional[QMatMul]:
        return self.q_map.get(name)

    def resident_bytes(self) -> int:
        dense = sum(t.numel() * t.element_size() for t in self.map.values())
        seen, quant = set(), 0
        for qm in self.q_map.values():
            if id(qm) not in seen:
                seen.add(id(qm))
                quant += qm.storage_size_in_bytes()
        fp8 = sum(w.resident_bytes() for w in {id(w): w for w in self.fp8_map.values()}.values())
        return dense + quant + fp8

    def get(self, name: str) -> torch.Tensor:
        if name in self.map:
            return self.map[name].to(torch.float32)
        if name in self.q_map:
            return self.q_map[name].dequantize()
        raise MissingWeight(name)

    def to_device(self, target) -> int:
        """Weights::to_device (store.rs:170-205): dense entries move to `target` in its store
        dtype (f16 on a GPU, f32 on the CPU; E4M3 stays E4M3 on a GPU); quantized entries stay
        where they are, as the reference leaves its QTensors.  Integer entries (Marlin's
        packed words) keep their dtype here -- a cast would change the words.  Returns the
        resident bytes."""
        dev = torch.device(target)
        store = torch.float16 if dev.type == "cuda" else torch.float32
        for name, t in list(self.map.items()):
            t = t.to(dev)
            if t.dtype == torch.float8_e4m3fn:
                if dev.type != "cuda":
                    t = t.to(store)
            elif t.dtype != store and t.dtype.is_floating_point:
                t = t.to(store)
            self.map[name] = t
        self.dev = dev
        return self.resident_bytes()

    def get_raw(self, name: str) -> torch.Tensor:
        """The dense entry itself (store.rs:103-107)."""
        t = self.map.get(name)
        if t is None:
            raise MissingWeight(name)
        return t

    def contains_key(self, name: str) -> bool:
        return name in self.map or name in self.q_map

    def replace(self, name: str, tensor: torch.Tensor) -> None:
        """Weights::replace (store.rs:147-162): a dense entry is overwritten; a quantized
        one is dropped from q_map and the dense tensor takes its name; else MissingWeight."""
        if name in self.map:
            self.map[name] = tensor
            return
        if self.q_map.pop(name, None) is not None:
            self.map[name] = tensor
            return
        raise MissingWeight(name)

    def candidate_weights(self, name: str, ids) -> torch.Tensor:
        """Rows `ids` of a vocabulary matrix, [len(ids), hidden] (embed_layer.rs:59-82): f32
        dequantized rows of a q_map entry (rtd_qembed), else rows of the dense entry in its
        own dtype."""
        ids_t = torch.as_tensor(np.asarray(ids, dtype=np.int64) if not torch.is_tensor(ids) else ids).reshape(-1)
        qm = self.q_map.get(name)
        if qm is not None:
            if ids_t.numel() == 0:
                return torch.zeros((0, qm.k), dtype=torch.float32, device=qm.device)
            return qm.embedding(ids_t)
        w = self.get_raw(name)
        if ids_t.numel() == 0:
            return torch.zeros((0, int(w.shape[1])), dtype=torch.float32, device=w.device)
        return w.index_select(0, ids_t.to(device=w.device, dtype=torch.int64))

    def linear(self, x: torch.Tensor, name: str) -> torch.Tensor:
        qm = self.q_map.get(name)
        if qm is not None:
            return qm.forward(x)
        if self.find_marlin(name) is not None:
            return self._marlin_linear(x, name)
        fw = self.fp8_map.get(name)
        if fw is not None:
            return fw.forward(x).to(x.dtype)
        if name in self.map:
            return self.linear_dense(x, name)
        raise MissingWeight(name)

    # -- INT4 Marlin entries (linear_layer.rs:17-66): packed / scales tensors in ``map``
    MARLIN_PACKED_KEYS = ("{name}.marlin_packed", "{stem}.marlin_packed", "{name}.packed", "{stem}.packed")
    MARLIN_SCALE_KEYS = ("{name}.marlin_scales", "{stem}.marlin_scales", "{name}.scales", "{stem}.scales",
                         "{name}.scale", "{stem}.scale", "{name}.weight.scale", "{stem}.weight.scale")

    def insert_marlin(self, name: str, mw: "MarlinWeight") -> None:
        """Weights::insert_marlin (linear_layer.rs:17-22): the packed words under ``name``
        and ``{stem}.marlin_packed``, the scales under ``{stem}.marlin_scales``; the device
        handle is kept for the linears that use it."""
        stem = name[:-len(".weight")] if name.endswith(".weight") else name
        packed = torch.from_numpy(np.ascontiguousarray(mw.packed, dtype=np.uint32))
        self.map[name] = packed
        self.map[f"{stem}.marlin_packed"] = packed
        self.map[f"{stem}.marlin_scales"] = torch.from_numpy(np.asarray(mw.scales, dtype=np.float32).copy())
        self.__dict__.setdefault("_marlin_dev", {})[(stem, mw.in_dim)] = mw

    def find_marlin(self, name: str):
        """(packed, scales) of a Marlin entry, found as Weights::find_marlin does
        (linear_layer.rs:24-43): the suffixed keys first, then a U32 tensor under the name or
        its stem; None when either half is missing."""
        stem = name[:-len(".weight")] if name.endswith(".weight") else name
        packed = None
        for key in self.MARLIN_PACKED_KEYS:
            packed = self.map.get(key.format(name=name, stem=stem))
            if packed is not None:
                break
        if packed is None:
            for key in (name, stem):
                t = self.map.get(key)
                if t is not None and _is_u32(t):
                    packed = t
                    break
        if packed is None:
            return None
        for key in self.MARLIN_SCALE_KEYS:
            scales = self.map.get(key.format(name=name, stem=stem))
            if scales is not None:
                return packed, scales
        return None

    def _marlin_linear(self, x: torch.Tensor, name: str, check: bool = True) -> torch.Tensor:
        """The Marlin branch of Weights::linear (linear_layer.rs:53-63): in_dim from x, the
        packed chunk count bounding it (`check`; linear_dense's branch, :69-74, skips the
        bound), then marlin_gemv."""
        packed, scales = self.find_marlin(name)
        x_in = int(x.shape[-1]) if x.dim() else 0
        out_dim = int(scales.numel()) if torch.is_tensor(scales) else int(np.asarray(scales).size)
        ndim = packed.dim() if torch.is_tensor(packed) else np.asarray(packed).ndim
        kc = int(packed.shape[0]) if ndim >= 2 else (x_in + 31) // 32
        max_k, min_k = kc * 32, ((kc - 1) * 32 if kc > 1 else 0)
        if check and (x_in > max_k or (kc > 1 and x_in <= min_k)):
            raise ShapeError(name, [max_k], list(x.shape))
        stem = name[:-len(".weight")] if name.endswith(".weight") else name
        cache = self.__dict__.setdefault("_marlin_dev", {})
        mw = cache.get((stem, x_in))
        if mw is None:
            p = packed.cpu().numpy() if torch.is_tensor(packed) else np.asarray(packed)
            sc = scales.cpu().numpy() if torch.is_tensor(scales) else np.asarray(scales)
            mw = MarlinWeight(p.astype(np.uint32, copy=False), sc.astype(np.float32).reshape(-1), x_in, out_dim,
                              device=self.dev)
            cache[(stem, x_in)] = mw
        return mw.forward(x)

    FP8_SCALE_SUFFIXES = (".scale", "_scale", ".weight_scale_inv")

    def fp8_scale(self, name: str, out_dim: int) -> torch.Tensor:
        """The scale of an E4M3 weight in ``map``: the first of ``{name}.scale``,
        ``{name}_scale`` and ``{name}.weight_scale_inv`` that exists, else ones
        (crates/runtimed-model/src/weights/linear_layer.rs:78-86)."""
        for suffix in self.FP8_SCALE_SUFFIXES:
            s = self.map.get(name + suffix)
            if s is not None:
                return s.to(torch.float32)
        return torch.ones(out_dim, dtype=torch.float32)

    def linear_dense(self, x: torch.Tensor, name: str, mode: str = "w8a8") -> torch.Tensor:
        """Weights::linear_dense (linear_layer.rs:68-101) for E4M3 entries of ``map``
        (torch.float8_e4m3fn, [out, in]): the scale by key lookup, then the FP8 linear
        with the reference CUDA semantics (W8A8: x encoded to E4M3 first,
        fp8_gemm.rs:96-101); the device weight is built once per entry."""
        if self.find_marlin(name) is not None:  # linear_layer.rs:68-75: Marlin entries first
            return self._marlin_linear(x, name, check=False)
        w = self.map.get(name)
        if w is None:
            raise MissingWeight(name)
        if w.dtype != torch.float8_e4m3fn:
            raise ConfigError(f"{name}: dense {w.dtype} weights are not on this path")
        if w.dim() != 2:
            raise ShapeError(name, [2], list(w.shape))
        out_dim, in_dim = int(w.shape[0]), int(w.shape[1])
        if x.shape[-1] != in_dim:
            raise ShapeError(name, [in_dim], list(x.shape))
        cache = self.__dict__.setdefault("_fp8_dense", {})
        fw = cache.get(name)
        if fw is None:
            scale = self.fp8_scale(name, out_dim).reshape(-1).cpu().numpy()
            codes = w.detach().cpu().view(torch.uint8).numpy()
            fw = Fp8Weight(codes, scale, in_dim, out_dim, device=self.dev)
            cache[name] = fw
        return fw.forward(x, mode=mode).to(x.dtype)

    def linear_bias(self, x: torch.Tensor, name: str, bias: Optional[str] = None) -> torch.Tensor:
        if bias is None:
            return self.linear(x, name)
        b = self.get(bias)
        qm = self.q_map.get(name)
        if qm is not None:
            return qm.forward(x, bias=b)
        y = self.linear(x, name)
        return y + b.to(device=y.device, dtype=y.dtype)

    def embed(self, name: str, ids) -> torch.Tensor:
        """Weights::embed (embed_layer.rs:16-57): rows `ids` as f32 [1, len(ids), hidden] --
        dequantized rows of a q_map entry (rtd_qembed), else rows of the dense entry."""
        qm = self.q_map.get(name)
        ids_t = torch.as_tensor(np.asarray(ids, dtype=np.int64) if not torch.is_tensor(ids) else ids).reshape(-1)
        if qm is None:
            w = self.map.get(name)
            if w is None:
                raise MissingWeight(name)
            if ids_t.numel() == 0:
                return torch.zeros((1, 0, int(w.shape[1])), dtype=torch.float32, device=w.device)
            if int(ids_t.max()) >= int(w.shape[0]) or int(ids_t.min()) < 0:
                raise ConfigError(f"embedding id out of range for {name} with {int(w.shape[0])} rows")
            return w.index_select(0, ids_t.to(device=w.device, dtype=torch.int64)).unsqueeze(0).to(torch.float32)
        if ids_t.numel() == 0:
            return torch.zeros((1, 0, qm.k), dtype=torch.float32, device=qm.device)
        if int(ids_t.max()) >= qm.n or int(ids_t.min()) < 0:
            raise ConfigError(f"embedding id out of range for {name} with {qm.n} rows")
        return qm.embedding(ids_t).unsqueeze(0)
