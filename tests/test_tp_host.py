"""Host-side tensor-parallel logic on the CPU: the shard byte layouts, the
reference's divisibility errors, and a two-rank gloo run of the row-parallel
reduction (restated oracle partials summed by all_reduce) against the unsharded GEMV.

Reference: crates/runtimed-model/src/tp/{column_linear,row_linear,mod}.rs
(the mod.rs:18-34 test checks that column shards concatenate to the full output).
"""
import os

import numpy as np
import pytest

import oracle
from runtimed_b200 import synth
from runtimed_b200.errors import ConfigError
from runtimed_b200.tp import shard_cols, shard_rows


def _dequant(t, raw, n, k):
    rc, y = oracle.dequant_tensor(t, raw, n * k)
    assert rc == oracle.OK
    return y.reshape(n, k)


@pytest.mark.parametrize("t", [12, 14, 8])
@pytest.mark.parametrize("world", [2, 4])
def test_shards_are_exact_slices(t, world):
    n, k = 32, 2048
    raw = synth.quant_matrix(t, n, k, seed=3, stream=t)
    full = _dequant(t, raw, n, k)
    for r in range(world):
        rows = _dequant(t, shard_rows(raw, t, n, k, r, world), n // world, k)
        assert np.array_equal(rows.view(np.uint32), full[r * n // world:(r + 1) * n // world].view(np.uint32))
        cols = _dequant(t, shard_cols(raw, t, n, k, r, world), n, k // world)
        assert np.array_equal(cols.view(np.uint32), full[:, r * k // world:(r + 1) * k // world].view(np.uint32))


def test_column_and_row_parallel_recombine():
    """Column shards concatenate to the full output; row-shard partials sum to it."""
    t, n, k, world = 12, 48, 1024, 4
    raw = synth.quant_matrix(t, n, k, seed=9)
    x = synth.activations(3, k, seed=9)
    full = oracle.qgemv_f64(t, raw, n, k, x)
    cat = np.concatenate([oracle.qgemv_f64(t, shard_rows(raw, t, n, k, r, world), n // world, k, x)
                          for r in range(world)], axis=1)
    assert np.allclose(cat, full, rtol=0, atol=1e-12)
    ks = k // world
    part = sum(oracle.qgemv_f64(t, shard_cols(raw, t, n, k, r, world), n, ks, x[:, r * ks:(r + 1) * ks])
               for r in range(world))
    assert np.allclose(part, full, rtol=1e-12, atol=1e-12)


def test_reference_divisibility_errors():
    raw = synth.quant_matrix(12, 6, 512, seed=1)
    with pytest.raises(ConfigError, match="TP size cannot be zero"):
        shard_rows(raw, 12, 6, 512, 0, 0)
    with pytest.raises(ConfigError, match="Output dimension 6 not divisible by TP size 4"):
        shard_rows(raw, 12, 6, 512, 0, 4)
    with pytest.raises(ConfigError, match="Input dimension 512 not divisible by TP size 3"):
        shard_cols(raw, 12, 6, 512, 0, 3)
    with pytest.raises(ConfigError, match="not a multiple of the 256-element block"):
        shard_cols(raw, 12, 6, 512, 0, 4)  # 128-element shards split a Q4_K superblock


def _gloo_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        t, n, k = 14, 40, 1024
        raw = synth.quant_matrix(t, n, k, seed=21)
        x = synth.activations(2, k, seed=21)
        ks = k // world
        part = oracle.qgemv_f64(t, shard_cols(raw, t, n, k, rank, world), n, ks, x[:, rank * ks:(rank + 1) * ks])
        y = torch.from_numpy(part)
        dist.all_reduce(y)
        # the communicator's handle exchange: every rank receives every rank's bytes in rank order
        got = [None] * world
        dist.all_gather_object(got, bytes([rank]) * 64)
        ok_handles = got == [bytes([r]) * 64 for r in range(world)]
        full = oracle.qgemv_f64(t, raw, n, k, x)
        q.put((rank, bool(np.allclose(y.numpy(), full, rtol=1e-12, atol=1e-12)), ok_handles))
    finally:
        dist.destroy_process_group()


def test_row_parallel_reduction_over_gloo():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert sorted(r for r, _, _ in res) == [0, 1]
    assert all(ok and hok for _, ok, hok in res)


def test_fp8_scale_key_order_and_default():
    # the lookup order of linear_layer.rs:78-86, on the host side of the mirror
    torch = pytest.importorskip("torch")
    from runtimed_b200.weights import Weights

    W = Weights.__new__(Weights)
    W.map = {"a.weight_scale_inv": torch.full((3,), 3.0), "a_scale": torch.full((3,), 2.0)}
    assert float(W.fp8_scale("a", 3)[0]) == 2.0  # "_scale" before ".weight_scale_inv"
    W.map["a.scale"] = torch.full((3,), 1.5)
    assert float(W.fp8_scale("a", 3)[0]) == 1.5  # ".scale" first
    assert torch.equal(W.fp8_scale("b", 4), torch.ones(4))  # none: ones of out_dim


def test_decoder_shards_reassemble_the_full_tensors(tmp_path):
    # Qwen2Model._shard (the TP decoder's per-rank weights): column-parallel linears keep
    # their rows, attn_output / ffn_down their input columns, everything else is whole
    pytest.importorskip("torch")
    from types import SimpleNamespace

    from runtimed_b200 import fixtures
    from runtimed_b200.gguf import GgufFile
    from runtimed_b200.qwen2 import Qwen2Model

    shape = fixtures.Qwen2Shape(hidden=512, n_layer=1, n_head=8, n_kv=4, ffn=1024, vocab=300,
                                formats={k: 8 for k in fixtures.DEFAULT_FORMATS})
    path = str(tmp_path / "m.gguf")
    fixtures.write_qwen2_gguf(path, shape, seed=2)
    f = GgufFile.open(path)
    for world in (2, 4):
        for t in f.tensors:
            if len(t.dims) != 2:
                continue
            k, n = int(t.dims[0]), int(t.dims[1])
            rc, full = oracle.dequant_tensor(t.dtype, np.asarray(f.tensor_bytes(t)), n * k)
            full = full.reshape(n, k)
            parts = []
            for r in range(world):
                raw, ns, ks = Qwen2Model._shard(SimpleNamespace(file=f, rank=r, world=world), t.name, t)
                rc, v = oracle.dequant_tensor(t.dtype, np.asarray(raw), ns * ks)
                parts.append(v.reshape(ns, ks))
            kind = t.name.split(".")[2] if t.name.startswith("blk.") else t.name
            if kind in ("attn_q", "attn_k", "attn_v", "ffn_gate", "ffn_up"):
                assert np.array_equal(np.concatenate(parts, axis=0), full), t.name
            elif kind in ("attn_output", "ffn_down"):
                assert np.array_equal(np.concatenate(parts, axis=1), full), t.name
            else:
                assert all(np.array_equal(p, full) for p in parts), t.name


def _np_greedy(v):
    """The greedy pick over f32 values as the reference's argmax makes it: the largest
    value, the lowest row among equal ones (-0 == +0), NaN never chosen, 0 if all are NaN."""
    v = np.asarray(v, np.float32)
    if np.isnan(v).all():
        return 0
    return int(np.nanargmax(v))


def _shard_keys(v, world):
    import ctypes

    from runtimed_b200.tp import pack_key

    rows = len(v) // world
    out = []
    for r in range(world):
        part = v[r * rows:(r + 1) * rows]
        best = max([pack_key(x, r * rows + i) for i, x in enumerate(part)] + [0])
        out.append(ctypes.c_int64(best).value)  # the u64 bit pattern, as int64
    return out


def test_vocab_parallel_keys_combine_to_the_greedy_pick():
    import torch

    from runtimed_b200.tp import combine_keys, pack_key

    # the packing orders values, then prefers the lower row; -0 equals +0; NaN has no key
    assert pack_key(1.0, 5) > pack_key(0.5, 0) > pack_key(0.0, 9) > pack_key(-1.0, 0) > pack_key(-np.inf, 0) > 0
    assert pack_key(2.0, 3) > pack_key(2.0, 4)
    assert pack_key(-0.0, 7) == pack_key(0.0, 7)
    assert pack_key(float("nan"), 1) == 0
    rng = np.random.default_rng(3)
    cases = []
    v = rng.normal(0, 1, 4096).astype(np.float32)
    cases.append(v)
    t = v.copy()
    t[[100, 3000]] = 9.0  # a tie across shards: the lower global row
    cases.append(t)
    n = v.copy()
    n[::3] = np.nan
    n[2] = np.nan
    cases.append(n)
    cases.append(np.full(4096, np.nan, np.float32))  # every value NaN: row 0
    z = np.zeros(4096, np.float32)
    z[::2] = -0.0
    cases.append(z)  # all zeros of either sign: row 0
    neg = -np.abs(v) - 1.0
    neg[2049] = -0.5
    cases.append(neg)
    for world in (1, 2, 4, 8):
        keys = torch.tensor([_shard_keys(c, world) for c in cases], dtype=torch.int64).T  # [world, cases]
        got = combine_keys(keys).tolist()
        assert got == [_np_greedy(c) for c in cases], world


def _gloo_vocab_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from runtimed_b200.tp import gather_greedy

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        logits = rng.normal(0, 1, (3, 1200)).astype(np.float32)  # 3 tokens, vocabulary 1200
        logits[1, [40, 900]] = 7.0
        mine = torch.tensor([_shard_keys(row, world)[rank] for row in logits], dtype=torch.int64)
        ids = gather_greedy(mine, world)
        q.put((rank, ids.tolist() == [_np_greedy(r) for r in logits]))
    finally:
        dist.destroy_process_group()


def test_vocab_parallel_greedy_over_gloo():
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_vocab_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert sorted(r for r, _ in res) == [0, 1]
    assert all(ok for _, ok in res)


def test_vocab_keys_property_random_values():
    # any f32 values (NaN, infinities, signed zeros, subnormals, duplicates) split into any
    # number of equal shards: the combined keys pick what the reference's argmax picks
    import torch
    from hypothesis import given, settings
    from hypothesis import strategies as st

    from runtimed_b200.tp import combine_keys

    special = st.sampled_from([0.0, -0.0, float("inf"), float("-inf"), float("nan"), 1e-45, -1e-45, 3.0, -3.0])
    value = st.one_of(special, st.floats(width=32, allow_nan=True, allow_infinity=True))

    @settings(max_examples=200, deadline=None)
    @given(st.lists(value, min_size=1, max_size=12), st.sampled_from([1, 2, 3, 4]))
    def check(vals, world):
        v = np.array(vals * world, dtype=np.float32)  # length divisible by world, duplicates
        keys = torch.tensor([_shard_keys(v, world)], dtype=torch.int64).T
        assert combine_keys(keys).tolist() == [_np_greedy(v)]

    check()


def test_weights_store_helpers_on_dense_entries():
    # store.rs:103-107,147-168 and embed_layer.rs:74-81 on dense entries (no device work)
    import torch

    from runtimed_b200.errors import MissingWeight
    from runtimed_b200.weights import Weights

    emb = torch.arange(12, dtype=torch.float32).reshape(4, 3)
    W = Weights(device="cuda:0", map={"tok.weight": emb}, q_map={"q.weight": object()})
    assert W.get_raw("tok.weight") is emb
    with pytest.raises(MissingWeight):
        W.get_raw("nope")
    assert W.contains_key("tok.weight") and W.contains_key("q.weight") and not W.contains_key("nope")
    assert W.candidate_weights("tok.weight", [3, 0, 3]).tolist() == [[9, 10, 11], [0, 1, 2], [9, 10, 11]]
    assert tuple(W.candidate_weights("tok.weight", []).shape) == (0, 3)
    with pytest.raises(MissingWeight):
        W.candidate_weights("nope", [0])
    W.replace("tok.weight", emb * 2)
    assert W.get_raw("tok.weight")[1, 1] == 8
    W.replace("q.weight", emb)  # a quantized entry gives way to the dense tensor
    assert "q.weight" not in W.q_map and W.get_raw("q.weight") is emb
    with pytest.raises(MissingWeight):
        W.replace("nope", emb)
    W2 = Weights.from_quantized("cuda:0", {"a": emb}, {"b.weight": object()})
    assert W2.contains_key("a") and W2.contains_key("b.weight")
    assert Weights.from_parts("cuda:0", {"a": emb}).q_map == {}
    assert Weights.cuda_available(0) == torch.cuda.is_available()
    assert not Weights.cuda_available(1 << 20)


def test_reference_tensor_parallel_known_answer():
    # tp/mod.rs:18-38: W = [[1, 2], [3, 4]] split by output rows over two ranks; x = [1, 1]
    # gives [3] and [7], concatenated [3, 7].  Here W is a Q8_0 matrix (d = 1, the codes the
    # values, K padded to one 32-wide block with zeros) and each rank's shard is its byte
    # slice; the partial outputs come from the oracle.
    from runtimed_b200.tp import shard_rows

    blocks = np.zeros((2, 34), np.uint8)
    blocks[:, 0:2] = np.array([0x3C00], np.uint16).view(np.uint8)  # d = 1.0 (f16)
    blocks[0, 2:4] = [1, 2]
    blocks[1, 2:4] = [3, 4]
    raw = blocks.reshape(-1)
    x = np.zeros((1, 32), np.float32)
    x[0, :2] = 1.0
    ys = [oracle.qgemv_f64(8, shard_rows(raw, 8, 2, 32, r, 2), 1, 32, x) for r in range(2)]
    assert np.concatenate(ys, axis=1).tolist() == [[3.0, 7.0]]
    # the reduction of two equal partials (ring_all_reduce over [y0, y0]): every rank gets 2 y0
    assert (ys[0] + ys[0]).tolist() == [[6.0]]


def test_reference_embed_dense_known_answer():
    # embed_layer.rs:90-124 (embed_dense_and_quantized), the dense half: a 4 x 3 table,
    # ids [1, 3] -> [1, 2, 3] rows [3, 4, 5] and [9, 10, 11]; candidate_weights -> [2, 3]
    # (the quantized half runs rtd_qembed and is checked bit-exact on the GPU)
    import torch

    from runtimed_b200.errors import ConfigError, MissingWeight
    from runtimed_b200.weights import Weights

    table = torch.arange(12, dtype=torch.float32).reshape(4, 3)
    W = Weights.from_parts("cuda:0", {"dense_embd": table})
    out = W.embed("dense_embd", [1, 3])
    assert tuple(out.shape) == (1, 2, 3)
    assert out.flatten().tolist() == [3.0, 4.0, 5.0, 9.0, 10.0, 11.0]
    assert tuple(W.candidate_weights("dense_embd", [1, 3]).shape) == (2, 3)
    assert tuple(W.embed("dense_embd", []).shape) == (1, 0, 3)
    assert W.embed("dense_embd", [2]).dtype == torch.float32
    with pytest.raises(ConfigError):
        W.embed("dense_embd", [4])
    with pytest.raises(MissingWeight):
        W.embed("nope", [0])


def _gloo_mlp_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        h, inter = 256, 512
        gate = synth.quant_matrix(12, inter, h, seed=31)
        up = synth.quant_matrix(12, inter, h, seed=32)
        down = synth.quant_matrix(14, h, inter, seed=33)
        x = synth.activations(2, h, seed=34).astype(np.float64)
        # this rank: gate / up rows (column parallel), down columns (row parallel)
        fr = inter // world
        g = oracle.qgemv_f64(12, shard_rows(gate, 12, inter, h, rank, world), fr, h, x)
        u = oracle.qgemv_f64(12, shard_rows(up, 12, inter, h, rank, world), fr, h, x)
        act = g / (1.0 + np.exp(-g)) * u
        part = oracle.qgemv_f64(14, shard_cols(down, 14, h, inter, rank, world), h, fr, act)
        y = torch.from_numpy(part)
        dist.all_reduce(y)
        # the unsharded MLP
        G = oracle.qgemv_f64(12, gate, inter, h, x)
        U = oracle.qgemv_f64(12, up, inter, h, x)
        full = oracle.qgemv_f64(14, down, h, inter, G / (1.0 + np.exp(-G)) * U)
        mine = y.numpy().copy()
        got = [torch.zeros_like(y) for _ in range(world)]
        dist.all_gather(got, y)
        q.put((rank, float(np.abs(mine - full).max() / np.abs(full).max()),
               all(torch.equal(got[0], t) for t in got)))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_mlp_ranks_agree_over_gloo():
    # tp/dual_gpu.rs:192-205 (test_dual_gpu_mlp_and_block, the MLP half) with quantized
    # shards: gate / up split by rows, down by columns, SwiGLU on each rank's slice, the
    # partial outputs summed over two gloo ranks; every rank holds the same y, equal to
    # the unsharded MLP (the reference's bar: ranks within 1e-4)
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gloo_mlp_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert sorted(r for r, _, _ in res) == [0, 1]
    assert all(err < 1e-12 and same for _, err, same in res)


def test_weights_to_device_store_dtypes():
    # store.rs:170-205 toward the CPU: dense entries become f32 (E4M3 included), integer
    # entries keep their dtype, and the resident bytes follow
    import torch

    from runtimed_b200.weights import Weights

    W = Weights.from_parts("cuda:0", {"a": torch.ones(4, 3, dtype=torch.float16),
                                      "e": torch.ones(2, 2).to(torch.float8_e4m3fn),
                                      "packed": torch.zeros(3, dtype=torch.uint32)})
    n = W.to_device("cpu")
    assert W.map["a"].dtype == torch.float32 and W.map["e"].dtype == torch.float32
    assert W.map["packed"].dtype == torch.uint32
    assert W.device() == torch.device("cpu")
    assert n == 4 * 3 * 4 + 2 * 2 * 4 + 3 * 4
