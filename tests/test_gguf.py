"""GGUF container parsing (runtimed_b200.gguf, mirroring crates/runtimed-gguf/src/header.rs)
and the Qwen2 fixture writer, checked on the CPU.

Files are written by gguf-py's GGUFWriter (an independent implementation) and read back
by the parser: metadata values and types, tensor dims / types / offsets, the data start
on the alignment boundary, and tensor_bytes against gguf-py's own reader.  The error
cases follow GgufError: bad magic, version, truncation, unknown metadata type, a tensor
past the end of the file, and an undecodable type.  The restated Qwen2 forward's
operations are pinned by the reference's own unit tests (ops/norm.rs, ops/rope.rs).
"""
import os
import struct

import numpy as np
import pytest

from runtimed_b200 import fixtures, gguf as G


@pytest.fixture(scope="module")
def small_file(tmp_path_factory):
    path = str(tmp_path_factory.mktemp("gguf") / "small.gguf")
    types = fixtures.write_qwen2_gguf(path, fixtures.small_shape(n_layer=2, vocab=300), seed=1)
    return path, types


def test_parse_matches_gguf_py_reader(small_file):
    import gguf

    path, types = small_file
    f = G.GgufFile.open(path)
    r = gguf.GGUFReader(path)
    assert f.metadata["general.architecture"] == "qwen2"
    assert f.metadata["qwen2.block_count"] == 2 and f.meta_types["qwen2.block_count"] == 4
    assert f.metadata["qwen2.attention.head_count_kv"] == 2
    assert abs(f.metadata["qwen2.attention.layer_norm_rms_epsilon"] - 1e-6) < 1e-12
    assert [t.name for t in f.tensors] == [t.name for t in r.tensors]
    for t, rt in zip(f.tensors, r.tensors):
        assert t.dims == [int(d) for d in rt.shape]
        assert t.dtype == int(rt.tensor_type)
        assert t.offset == int(rt.data_offset)
        got = f.tensor_bytes(t)
        assert np.array_equal(got, np.asarray(rt.data).reshape(-1).view(np.uint8))
        if t.name in types:
            assert t.dtype == types[t.name]
    # data starts on the 32-byte boundary; GGUF [K, N] dims of a linear
    assert min(t.offset for t in f.tensors) % 32 == 0
    assert f.tensor("blk.0.ffn_gate.weight").dims == [256, 512]


def test_config0_formats_fall_back_to_q8_0_on_k_896():
    # K-quant superblocks need K % 256 == 0: hidden 896 takes Q8_0, ffn_down (K = 4864) keeps Q6_K
    s = fixtures.CONFIGS["config0"]
    got = {kind: fixtures.tensor_format(s, kind, k) for kind, n, k in fixtures.layer_tensors(s)}
    assert got == {"attn_q": 8, "attn_k": 8, "attn_v": 8, "attn_output": 8, "ffn_gate": 8, "ffn_up": 8, "ffn_down": 14}
    assert fixtures.tensor_format(s, "token_embd", s.hidden) == 8


def _header(version=3, n_tensors=0, n_meta=0):
    return b"GGUF" + struct.pack("<IQQ", version, n_tensors, n_meta)


def _s(x: str) -> bytes:
    return struct.pack("<Q", len(x)) + x.encode()


def test_errors_mirror_gguf_error():
    with pytest.raises(G.GgufError) as e:
        G.GgufFile.parse(b"GGML" + bytes(20))
    assert e.value.kind == "BadMagic"
    with pytest.raises(G.GgufError) as e:
        G.GgufFile.parse(_header(version=2))
    assert e.value.kind == "Version" and e.value.detail == 2
    with pytest.raises(G.GgufError) as e:
        G.GgufFile.parse(_header(n_meta=1) + _s("a.b"))  # the value type is missing
    assert e.value.kind == "Truncated"
    with pytest.raises(G.GgufError) as e:
        G.GgufFile.parse(_header(n_meta=1) + _s("a.b") + struct.pack("<I", 13))
    assert e.value.kind == "MetaType" and e.value.detail == 13
    # one Q8_0 tensor [32] whose data lies past the end of the file
    body = _header(n_tensors=1) + _s("w") + struct.pack("<IQIQ", 1, 32, 8, 4096)
    with pytest.raises(G.GgufError) as e:
        G.GgufFile.parse(body)
    assert e.value.kind == "Range"
    # in range but shorter than its blocks: tensor_bytes refuses
    body = _header(n_tensors=1) + _s("w") + struct.pack("<IQIQ", 1, 64, 8, 0)
    body += bytes((-len(body)) % 32) + bytes(34)
    f = G.GgufFile.parse(body)
    with pytest.raises(G.GgufError) as e:
        f.tensor_bytes(f.tensor("w"))
    assert e.value.kind == "Range"
    # an undecodable type id
    body = _header(n_tensors=1) + _s("w") + struct.pack("<IQIQ", 1, 32, 7, 0)
    body += bytes((-len(body)) % 32) + bytes(64)
    f = G.GgufFile.parse(body)
    with pytest.raises(G.GgufError) as e:
        f.tensor_bytes(f.tensor("w"))
    assert e.value.kind == "Unsupported"


def test_alignment_from_metadata_and_arrays():
    # general.alignment (U32) moves the data start; arrays and every scalar type parse
    meta = _s("general.alignment") + struct.pack("<II", 4, 64)
    meta += _s("x.arr") + struct.pack("<IIQ", 9, 5, 3) + struct.pack("<iii", -1, 2, 3)
    meta += _s("x.f64") + struct.pack("<Id", 12, 0.25) + _s("x.b") + struct.pack("<IB", 7, 1)
    meta += _s("x.s") + struct.pack("<I", 8) + _s("hi")
    body = _header(n_tensors=1, n_meta=5) + meta + _s("w") + struct.pack("<IQIQ", 1, 4, 0, 0)
    pad = (-len(body)) % 64
    body += bytes(pad) + struct.pack("<4f", 1, 2, 3, 4)
    f = G.GgufFile.parse(body)
    assert f.metadata["x.arr"] == [-1, 2, 3] and f.metadata["x.f64"] == 0.25
    assert f.metadata["x.b"] is True and f.metadata["x.s"] == "hi"
    assert f.tensor("w").offset % 64 == 0
    assert np.array_equal(f.tensor_bytes(f.tensor("w")).view(np.float32), [1, 2, 3, 4])


def test_qwen2_config_parse_and_refusal(small_file, tmp_path):
    torch = pytest.importorskip("torch")  # noqa: F841 (the model module imports torch)
    from runtimed_b200.errors import ConfigError
    from runtimed_b200.qwen2 import Qwen2Config

    path, _ = small_file
    cfg = Qwen2Config.from_gguf(G.GgufFile.open(path))
    assert (cfg.n_layer, cfg.hidden, cfg.n_head, cfg.n_kv, cfg.head_dim, cfg.ffn, cfg.vocab) == (2, 256, 4, 2, 64, 512, 300)
    assert cfg.has_qkv_bias and abs(cfg.rope_theta - 1e6) < 1
    # a file without output.weight is refused (parse_gguf.rs:220-222)
    import gguf

    p2 = str(tmp_path / "no_output.gguf")
    w = gguf.GGUFWriter(p2, "qwen2")
    w.add_block_count(1)
    w.add_embedding_length(32)
    w.add_head_count(1)
    w.add_head_count_kv(1)
    w.add_feed_forward_length(64)
    w.add_layer_norm_rms_eps(1e-6)
    w.add_rope_freq_base(1e6)
    w.add_tensor("token_embd.weight", np.zeros((4, 32), np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(ConfigError, match="output.weight"):
        Qwen2Config.from_gguf(G.GgufFile.open(p2))


def test_restated_ops_pinned_by_reference_unit_tests():
    from oracle import qwen2_ref as R

    # ops/norm.rs:29-38: x = [3, 4], w = [2, 0.5], eps = 0
    y = R._rmsnorm(np.array([[3.0, 4.0]], np.float32), np.array([2.0, 0.5], np.float32), 0.0)[0]
    rms = np.sqrt(np.float32(12.5))
    assert abs(y[0] - 3 / rms * 2) < 1e-6 and abs(y[1] - 4 / rms * 0.5) < 1e-6
    # ops/rope.rs:103-121: x = [1, 0, 0, 1]; position 0 is the identity, position 1
    # rotates the first pair by one radian
    x = np.array([[[1.0, 0.0, 0.0, 1.0]]], np.float32)  # [heads=1, t=1, d=4]
    y0 = R._rope(x, np.array([0]), 10000.0, 4)[0, 0]
    assert abs(y0[0] - 1.0) < 1e-6 and abs(y0[3] - 1.0) < 1e-6
    y1 = R._rope(x, np.array([1]), 10000.0, 4)[0, 0]
    assert abs(y1[0] - np.cos(np.float32(1.0))) < 1e-6 and abs(y1[2] - np.sin(np.float32(1.0))) < 1e-6
