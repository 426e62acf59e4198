"""GGUF v3 container parsing, mirroring crates/runtimed-gguf/src/header.rs.

``GgufFile.open(path)`` maps the file read-only and parses it the way
``GgufFile::parse`` (header.rs:130-184) does: magic ``GGUF``, version 3, tensor and
metadata counts (u64), the metadata entries (the 13 value types of ``Cursor::value``,
header.rs:80-107, arrays included), the tensor infos (name, dims fast-first, ggml type
id, offset relative to the data start), then the data start rounded up to
``general.alignment`` (a U32; 32 when absent).  ``tensor_bytes`` (header.rs:191-205)
returns the bounds-checked raw block bytes of a tensor -- exactly what
``rtd_qweight_upload`` takes, with the GGUF dims ``[K, N]`` read as ``[N, K]``
(crates/runtimed-model/src/weights/load_gguf.rs:35).

Errors mirror ``GgufError`` (crates/runtimed-gguf/src/error.rs): the exception's
``kind`` is one of BadMagic, Version, Truncated, MetaType, Range, Overflow,
Unsupported.  All parsing is host-side byte work; no device is involved.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass
from typing import Dict, List, Optional

import numpy as np

from .errors import GgufError as _GgufError

# GgmlDtype::block (crates/runtimed-gguf/src/quant/dtype.rs:49-64): id -> (elements, bytes)
BLOCK = {0: (1, 4), 1: (1, 2), 30: (1, 2), 2: (32, 18), 6: (32, 22), 8: (32, 34), 10: (256, 84), 11: (256, 110),
         12: (256, 144), 13: (256, 176), 14: (256, 210)}
TYPE_NAMES = {0: "F32", 1: "F16", 30: "BF16", 2: "Q4_0", 6: "Q5_0", 8: "Q8_0", 10: "Q2_K", 11: "Q3_K", 12: "Q4_K",
              13: "Q5_K", 14: "Q6_K"}


class GgufError(_GgufError):
    """GgufError::{BadMagic, Version, Truncated, MetaType, Range, Overflow, Unsupported}."""

    def __init__(self, kind: str, detail=None):
        msg = {
            "BadMagic": "bad magic: not a GGUF file",
            "Version": f"unsupported GGUF version: {detail} (want 3)",
            "Truncated": f"truncated file at offset {detail}",
            "MetaType": f"unknown metadata type id: {detail}",
            "Range": f"tensor '{detail}': byte range out of bounds",
            "Overflow": f"tensor '{detail}': element count overflows",
            "Unsupported": f"decode of {detail} not implemented",
        }[kind]
        super().__init__(msg)
        self.kind, self.detail = kind, detail


@dataclass
class TensorInfo:
    name: str
    dims: List[int]       # GGUF order: fastest dimension first
    dtype: int            # ggml type id
    offset: int           # absolute file offset of the tensor's bytes
    n_elements: int


class _Cursor:
    """header.rs:41-107: a bounds-checked little-endian reader."""

    def __init__(self, buf):
        self.buf, self.pos = buf, 0

    def take(self, n: int) -> bytes:
        end = self.pos + n
        if n < 0 or end > len(self.buf):
            raise GgufError("Truncated", self.pos)
        out = self.buf[self.pos:end]
        self.pos = end
        return out

    def u8(self) -> int:
        return self.take(1)[0]

    def u16(self) -> int:
        return struct.unpack("<H", self.take(2))[0]

    def u32(self) -> int:
        return struct.unpack("<I", self.take(4))[0]

    def u64(self) -> int:
        return struct.unpack("<Q", self.take(8))[0]

    def string(self) -> str:
        n = self.u64()
        raw = self.take(n)
        try:
            return bytes(raw).decode("utf-8")
        except UnicodeDecodeError:
            raise GgufError("Truncated", self.pos) from None

    def value(self, ty: int):
        if ty == 0:
            return self.u8()
        if ty == 1:
            return struct.unpack("<b", self.take(1))[0]
        if ty == 2:
            return self.u16()
        if ty == 3:
            return struct.unpack("<h", self.take(2))[0]
        if ty == 4:
            return self.u32()
        if ty == 5:
            return struct.unpack("<i", self.take(4))[0]
        if ty == 6:
            return struct.unpack("<f", self.take(4))[0]
        if ty == 7:
            return self.u8() != 0
        if ty == 8:
            return self.string()
        if ty == 9:
            elem = self.u32()
            n = self.u64()
            return [self.value(elem) for _ in range(n)]
        if ty == 10:
            return self.u64()
        if ty == 11:
            return struct.unpack("<q", self.take(8))[0]
        if ty == 12:
            return struct.unpack("<d", self.take(8))[0]
        raise GgufError("MetaType", ty)


class GgufFile:
    """A parsed GGUF file backed by a read-only mapping; tensor access is bounds-checked."""

    def __init__(self, buf, metadata: Dict[str, object], meta_types: Dict[str, int], tensors: List[TensorInfo]):
        self._buf = buf
        self.metadata = metadata
        self.meta_types = meta_types
        self.tensors = tensors
        self._by_name = {t.name: t for t in tensors}

    @classmethod
    def open(cls, path: str) -> "GgufFile":
        with open(path, "rb") as f:
            size = f.seek(0, 2)
            buf = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) if size > 0 else b""
        return cls.parse(buf)

    @classmethod
    def parse(cls, buf) -> "GgufFile":
        """header.rs:130-184."""
        cur = _Cursor(buf)
        if bytes(cur.take(4)) != b"GGUF":
            raise GgufError("BadMagic")
        version = cur.u32()
        if version != 3:
            raise GgufError("Version", version)
        n_tensors, n_meta = cur.u64(), cur.u64()
        metadata, types = {}, {}
        for _ in range(n_meta):
            key = cur.string()
            ty = cur.u32()
            metadata[key] = cur.value(ty)
            types[key] = ty
        raw = []
        for _ in range(n_tensors):
            name = cur.string()
            n_dims = cur.u32()
            if n_dims > 8:
                raise GgufError("Truncated", cur.pos)
            dims = [cur.u64() for _ in range(n_dims)]
            dtype = cur.u32()
            offset = cur.u64()
            raw.append((name, dims, dtype, offset))
        align = metadata.get("general.alignment") if types.get("general.alignment") == 4 else 32
        align = max(int(align), 1)
        data_start = -(-cur.pos // align) * align
        tensors = []
        for name, dims, dtype, rel in raw:
            n = 1
            for d in dims:
                n *= d
                if n >= 1 << 64:
                    raise GgufError("Overflow", name)
            offset = data_start + rel
            if offset > len(buf):
                raise GgufError("Range", name)
            tensors.append(TensorInfo(name, dims, dtype, offset, n))
        return cls(buf, metadata, types, tensors)

    def tensor(self, name: str) -> Optional[TensorInfo]:
        return self._by_name.get(name)

    def meta_str(self, key: str) -> Optional[str]:
        v = self.metadata.get(key)
        return v if isinstance(v, str) else None

    def tensor_bytes(self, info: TensorInfo) -> np.ndarray:
        """Raw bytes of a tensor (header.rs:191-205), a read-only view of the mapping."""
        geo = BLOCK.get(info.dtype)
        if geo is None:
            raise GgufError("Unsupported", TYPE_NAMES.get(info.dtype, info.dtype))
        elems, bb = geo
        length = -(-info.n_elements // elems) * bb
        end = info.offset + length
        if end > len(self._buf):
            raise GgufError("Range", info.name)
        return np.frombuffer(self._buf, dtype=np.uint8, count=length, offset=info.offset)

    def close(self) -> None:
        if isinstance(self._buf, mmap.mmap):
            self._buf.close()
