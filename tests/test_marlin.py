"""INT4 Marlin weights (crates/runtimed-model/src/ops/marlin_gemv.rs): the oracle against the
reference's own test values, the host repack against the oracle, and (GPU) the library's
rtd_marlin_upload handle through rtd_qdequant and rtd_qlinear."""
import numpy as np
import pytest

import oracle


def _case(n, k, seed):
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((n, k)).astype(np.float32) * np.float32(0.02)
    s = (np.abs(w).max(axis=1) / np.float32(7.0)).astype(np.float32)
    return w, s


def test_oracle_reference_known_answer():
    # marlin_gemv.rs:216-233 (marlin_gemv_cpu_matches_dequant): the 2 x 4 weight, scales
    # 0.5 / 0.25 and x = [2, 1, -1, 3]; resident bytes 2*4*4 + 2*4
    w = np.array([[1.0, -2.0, 3.0, 0.0], [0.5, 1.5, -0.5, 2.0]], np.float32)
    s = np.array([0.5, 0.25], np.float32)
    p = oracle.marlin_repack(w, s)
    assert p.nbytes + s.nbytes == 2 * 4 * 4 + 2 * 4
    deq = oracle.marlin_dequant(p, s, 2, 4)
    # row 1's 2.0 / 0.25 = 8 clamps to code 15 -> 1.75
    assert np.array_equal(deq, np.array([[1.0, -2.0, 3.0, 0.0], [0.5, 1.5, -0.5, 1.75]], np.float32))
    y = oracle.marlin_gemv_f64(np.array([[2.0, 1.0, -1.0, 3.0]]), p, s, 2, 4)
    assert np.allclose(y, [[-3.0, 8.25]])


def test_host_repack_matches_oracle():
    from runtimed_b200.weights import repack_marlin_tiles

    for n, k in [(2, 4), (32, 50), (17, 256), (8, 100)]:
        w, s = _case(n, k, n + k)
        w[0, 0] = s[0] * np.float32(2.5)  # a half: rounds away from zero
        p, s2 = repack_marlin_tiles(w, s)
        assert p.dtype == np.uint32 and p.shape == ((k + 31) // 32, n, 4)
        assert np.array_equal(p, oracle.marlin_repack(w, s))
        assert np.array_equal(s2, s)


@pytest.mark.gpu
@pytest.mark.parametrize("n,k", [(32, 50), (300, 4096), (64, 1000)])
def test_marlin_dequant_bit_exact(n, k):
    from runtimed_b200.weights import MarlinWeight, repack_marlin_tiles

    w, s = _case(n, k, 7)
    p, s = repack_marlin_tiles(w, s)
    mw = MarlinWeight(p, s, k, n)
    got = mw.dequantize().cpu().numpy()
    want = oracle.marlin_dequant(p, s, n, k)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert mw.resident_bytes() == p.nbytes + s.nbytes


@pytest.mark.gpu
@pytest.mark.parametrize("n,k", [(32, 50), (2048, 4096), (300, 1000)])
@pytest.mark.parametrize("m", [1, 2, 5, 64, 130])
def test_marlin_linear_matches_oracle(n, k, m):
    # M <= 3: the decode GEMV (exact products: 2e-5 with f32 out); 4 <= M <= 64 the skinny
    # tensor-memory GEMM and above it the shared-memory GEMM (weights exact in f16: codes
    # q - 8, the f32 row scale in the epilogue; activations rounded to f16: 1e-3)
    import torch

    from runtimed_b200.weights import MarlinWeight, marlin_gemv, repack_marlin_tiles

    w, s = _case(n, k, 3)
    p, s = repack_marlin_tiles(w, s)
    mw = MarlinWeight(p, s, k, n)
    x = np.random.default_rng(m).standard_normal((m, k)).astype(np.float32)
    y = marlin_gemv(torch.from_numpy(x).cuda(), mw).cpu().numpy()
    want = oracle.marlin_gemv_f64(x, p, s, n, k)
    err = np.linalg.norm(y - want) / np.linalg.norm(want)
    assert err <= (2e-5 if m <= 3 else 1e-3), err
    assert y.dtype == np.float32 and y.shape == (m, n)


@pytest.mark.gpu
def test_marlin_shape_errors_and_refusals():
    import torch

    from runtimed_b200.errors import ConfigError, ShapeError
    from runtimed_b200.weights import MarlinWeight, repack_marlin_tiles

    w, s = _case(16, 64, 1)
    p, s = repack_marlin_tiles(w, s)
    with pytest.raises(ConfigError):
        MarlinWeight(p.astype(np.int32), s, 64, 16)
    with pytest.raises(ShapeError):
        MarlinWeight(p, s[:8], 64, 16)
    with pytest.raises(ShapeError):
        MarlinWeight(p[:1, :8], s, 64, 16)
    mw = MarlinWeight(p, s.reshape(16, 1), 64, 16)
    with pytest.raises(ShapeError):
        mw.forward(torch.zeros(1, 63, device="cuda"))
    with pytest.raises(ConfigError):
        mw.embedding(torch.zeros(1, dtype=torch.int32))
    assert mw.forward(torch.zeros(0, 64, device="cuda")).shape == (0, 16)


def test_weights_find_marlin_keys_and_bounds_on_cpu():
    # Weights::find_marlin's key order (linear_layer.rs:24-43) and Weights::linear's bound on
    # the activation width (:55-59), both decided before any device work
    import torch

    from runtimed_b200.errors import ShapeError
    from runtimed_b200.weights import Weights, repack_marlin_tiles

    w, s = _case(2, 4, 3)
    p, s = repack_marlin_tiles(w, s)
    pt, st = torch.from_numpy(p), torch.from_numpy(s)
    W = Weights(device="cuda:0", map={"a.weight": pt, "a.scale": st})
    assert W.find_marlin("a.weight") is not None  # a U32 tensor under the name, ".scale" of the stem
    W = Weights(device="cuda:0", map={"b.weight": pt.to(torch.int64), "b.scales": st})
    assert W.find_marlin("b.weight") is None  # not U32, no packed key
    W = Weights(device="cuda:0", map={"c.packed": pt, "c.weight.marlin_scales": st, "c.scales": st * 2})
    got = W.find_marlin("c.weight")
    assert got is not None and got[1] is W.map["c.weight.marlin_scales"]  # "{name}.marlin_scales" first
    W = Weights(device="cuda:0", map={"d.marlin_packed": pt})
    assert W.find_marlin("d.weight") is None  # scales missing
    # one 32-wide chunk: any in_dim up to 32; more than 32 is a shape error
    W = Weights(device="cuda:0", map={"e.marlin_packed": pt, "e.marlin_scales": st})
    with pytest.raises(ShapeError):
        W.linear(torch.zeros(1, 80), "e.weight")
    # two chunks: in_dim must exceed 32 (the first chunk alone would do)
    w2, s2 = _case(2, 40, 4)
    p2, s2 = repack_marlin_tiles(w2, s2)
    W = Weights(device="cuda:0", map={"f.marlin_packed": torch.from_numpy(p2), "f.marlin_scales": torch.from_numpy(s2)})
    with pytest.raises(ShapeError):
        W.linear(torch.zeros(1, 32), "f.weight")
    with pytest.raises(ShapeError):
        W.linear(torch.zeros(1, 65), "f.weight")


@pytest.mark.gpu
def test_weights_linear_marlin_reference_known_answer():
    # linear_layer.rs:142-158 (linear_marlin_cpu): W = [[1, 2, 3, 4], [2, 3, 4, 5]], scales 1,
    # repacked, inserted under blk.0.attn_q; x = ones(4) gives [10, 14]; an 80-wide x is an error
    import torch

    from runtimed_b200.errors import ShapeError
    from runtimed_b200.weights import MarlinWeight, Weights, repack_marlin_tiles

    w = np.array([[1.0, 2.0, 3.0, 4.0], [2.0, 3.0, 4.0, 5.0]], np.float32)
    p, s = repack_marlin_tiles(w, np.ones(2, np.float32))
    W = Weights(device="cuda:0")
    W.insert_marlin("blk.0.attn_q", MarlinWeight(p, s, 4, 2))
    y = W.linear(torch.ones(1, 4, device="cuda"), "blk.0.attn_q.weight")
    assert tuple(y.shape) == (1, 2)
    assert y.flatten().cpu().tolist() == [10.0, 14.0]
    with pytest.raises(ShapeError):
        W.linear(torch.ones(1, 80, device="cuda"), "blk.0.attn_q.weight")
    # linear_dense reaches the same entry first
    assert W.linear_dense(torch.ones(1, 4, device="cuda"), "blk.0.attn_q.weight").flatten().cpu().tolist() == [10.0, 14.0]
