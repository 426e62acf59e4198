"""The decoder-layer kernels (rtd_rmsnorm, rtd_rope_kv_append, rtd_attention_paged,
rtd_silu_mul, rtd_argmax) on the GPU against float64 numpy statements of the reference
operations (crates/runtimed-model/src/ops/{norm,rope,attention,activation}.rs,
decode/sample.rs) on identical inputs.

The KV cache is paged: 16-token blocks from one pool, the block table shuffled by seed,
several sequences of different lengths in one call; long contexts take the split path
(partial softmax states merged in order).  Tolerances are f32 rounding bounds (the
cache holds f16, so keys and values are compared after the same f16 rounding).
"""
import numpy as np
import pytest

from runtimed_b200 import _lib

pytestmark = pytest.mark.gpu


def rel_l2(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))


def _ctx():
    from runtimed_b200.weights import Context

    return Context.for_device("cuda:0")


def _st():
    import torch

    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("H,T,with_delta,ydt", [(896, 3, True, "f32"), (8192, 2, False, "bf16"), (100, 5, True, "f16")])
def test_rmsnorm_with_residual_add(H, T, with_delta, ydt):
    import torch

    rng = np.random.default_rng(H)
    h = rng.normal(0, 3, (T, H)).astype(np.float32)
    d = rng.normal(0, 1, (T, H)).astype(np.float32)
    w = rng.normal(1, 0.1, H).astype(np.float32)
    hd, dd, wd = (torch.from_numpy(a).cuda() for a in (h, d, w))
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[ydt]
    y = torch.empty((T, H), dtype=tdt, device="cuda")
    L = _lib.lib()
    rc = L.rtd_rmsnorm(_ctx().handle, hd.data_ptr(), H, dd.data_ptr() if with_delta else None, _lib.DT_F32, H,
                       wd.data_ptr(), 1e-6, T, H, y.data_ptr(), {"f32": 0, "f16": 1, "bf16": 2}[ydt], H, _st())
    assert rc == 0
    hh = h.astype(np.float64) + (d if with_delta else 0)
    want = hh / np.sqrt((hh * hh).mean(-1, keepdims=True) + 1e-6) * w
    tol = {"f32": 1e-6, "f16": 1e-3, "bf16": 4e-3}[ydt]
    assert rel_l2(y.float().cpu().numpy(), want) <= tol
    assert rel_l2(hd.cpu().numpy(), hh) <= 1e-7  # the residual add is written back


def _rope_np(x, pos, theta, rot):
    half = rot // 2
    i = np.arange(half, dtype=np.float64)
    ang = pos[:, None, None] * theta ** (-2.0 * i / rot)[None, None, :]
    c, s = np.cos(ang), np.sin(ang)
    x1, x2 = x[..., :half], x[..., half:rot]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s, x[..., rot:]], axis=-1)


def _paged(n_seq, lens, max_blocks, n_blocks, seed):
    """A shuffled block pool: table[s][j] = block of tokens 16j .. 16j + 15 of sequence s."""
    rng = np.random.default_rng(seed)
    perm = rng.permutation(n_blocks)
    table = np.zeros((n_seq, max_blocks), np.int32)
    k = 0
    for s, n in enumerate(lens):
        for j in range(-(-n // 16)):
            table[s, j] = perm[k]
            k += 1
    return table


@pytest.mark.parametrize("n_head,n_kv,hd,kv", [(14, 2, 64, "f16"), (64, 8, 128, "f16"), (28, 4, 128, "f16"),
                                                (14, 2, 64, "f32"), (64, 8, 128, "f32")])
def test_rope_kv_append_and_paged_attention(n_head, n_kv, hd, kv):
    import torch

    cdt, npdt = (torch.float16, np.float16) if kv == "f16" else (torch.float32, np.float32)
    abi = _lib.DT_F16 if kv == "f16" else _lib.DT_F32
    rng = np.random.default_rng(n_head)
    lens = [37, 5, 300]  # three sequences; tokens are appended at the last positions
    n_seq, max_blocks, n_blocks = 3, 32, 64
    table = _paged(n_seq, lens, max_blocks, n_blocks, seed=hd)
    # this call: the last 3 tokens of seq 0 (a prefill chunk), the last of seq 1 and 2
    tok_seq = np.array([0, 0, 0, 1, 2], np.int32)
    tok_pos = np.array([34, 35, 36, 4, 299], np.int32)
    T = len(tok_seq)
    kc = torch.zeros((n_blocks, n_kv, 16, hd), dtype=cdt, device="cuda")
    vc = torch.zeros_like(kc)
    # earlier positions of every sequence already in the cache
    K = {s: rng.normal(0, 1, (lens[s], n_kv, hd)).astype(npdt) for s in range(n_seq)}
    V = {s: rng.normal(0, 1, (lens[s], n_kv, hd)).astype(npdt) for s in range(n_seq)}
    kch, vch = kc.cpu().numpy(), vc.cpu().numpy()
    for s in range(n_seq):
        for p in range(lens[s]):
            kch[table[s, p // 16], :, p % 16] = K[s][p]
            vch[table[s, p // 16], :, p % 16] = V[s][p]
    kc.copy_(torch.from_numpy(kch))
    vc.copy_(torch.from_numpy(vch))
    q = rng.normal(0, 1, (T, n_head * hd)).astype(np.float32)
    k = rng.normal(0, 1, (T, n_kv * hd)).astype(np.float32)
    v = rng.normal(0, 1, (T, n_kv * hd)).astype(np.float32)
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, k, v))
    sd, pd, td = (torch.from_numpy(a).cuda() for a in (tok_seq, tok_pos, table))
    qo = torch.empty((T, n_head * hd), dtype=torch.float32, device="cuda")
    L, c = _lib.lib(), _ctx().handle
    theta = 1e6
    rc = L.rtd_rope_kv_append(c, qd.data_ptr(), n_head * hd, kd.data_ptr(), n_kv * hd, vd.data_ptr(), n_kv * hd, T,
                              n_head, n_kv, hd, hd, theta, sd.data_ptr(), pd.data_ptr(), td.data_ptr(), max_blocks,
                              kc.data_ptr(), vc.data_ptr(), abi, qo.data_ptr(), _st())
    assert rc == 0
    qr = _rope_np(q.reshape(T, n_head, hd).astype(np.float64), tok_pos.astype(np.float64), theta, hd)
    kr = _rope_np(k.reshape(T, n_kv, hd).astype(np.float64), tok_pos.astype(np.float64), theta, hd)
    assert rel_l2(qo.cpu().numpy().reshape(T, n_head, hd), qr) <= 4e-6
    kch, vch = kc.cpu().numpy(), vc.cpu().numpy()
    for t in range(T):
        s, p = tok_seq[t], tok_pos[t]
        got_k = kch[table[s, p // 16], :, p % 16].astype(np.float64)
        assert rel_l2(got_k, kr[t]) <= (1e-3 if kv == "f16" else 4e-6)
        assert np.array_equal(vch[table[s, p // 16], :, p % 16], v[t].reshape(n_kv, hd).astype(npdt))
        K[s][p], V[s][p] = kch[table[s, p // 16], :, p % 16], vch[table[s, p // 16], :, p % 16]
    # attention over every visible position, from the cache contents
    scale = 1.0 / np.sqrt(hd)
    o = torch.empty((T, n_head * hd), dtype=torch.float32, device="cuda")
    rc = L.rtd_attention_paged(c, qo.data_ptr(), T, n_head, n_kv, hd, np.float32(scale), sd.data_ptr(), pd.data_ptr(),
                               td.data_ptr(), max_blocks, int(tok_pos.max()) + 1, kc.data_ptr(), vc.data_ptr(), abi,
                               o.data_ptr(), _lib.DT_F32, n_head * hd, _st())
    assert rc == 0
    G = n_head // n_kv
    qq = qo.cpu().numpy().reshape(T, n_head, hd).astype(np.float64)
    want = np.zeros((T, n_head, hd))
    for t in range(T):
        s, p = tok_seq[t], tok_pos[t]
        Ks = K[s][:p + 1].astype(np.float64)
        Vs = V[s][:p + 1].astype(np.float64)
        for h in range(n_head):
            sc = Ks[:, h // G] @ qq[t, h] * scale
            e = np.exp(sc - sc.max())
            want[t, h] = (e / e.sum()) @ Vs[:, h // G]
    assert rel_l2(o.cpu().numpy().reshape(T, n_head, hd), want) <= 1e-5


def test_attention_long_context_splits():
    # one decode token over 4000 positions: the context is split across CTAs and merged
    import torch

    n_head, n_kv, hd, n = 8, 1, 128, 4000
    max_blocks = -(-n // 16)
    table = _paged(1, [n], max_blocks, max_blocks + 3, seed=2)
    rng = np.random.default_rng(11)
    K = rng.normal(0, 1, (n, n_kv, hd)).astype(np.float16)
    V = rng.normal(0, 1, (n, n_kv, hd)).astype(np.float16)
    kc = np.zeros((max_blocks + 3, n_kv, 16, hd), np.float16)
    vc = np.zeros_like(kc)
    for p in range(n):
        kc[table[0, p // 16], :, p % 16] = K[p]
        vc[table[0, p // 16], :, p % 16] = V[p]
    q = rng.normal(0, 0.3, (1, n_head * hd)).astype(np.float32)
    kd, vd, qd = torch.from_numpy(kc).cuda(), torch.from_numpy(vc).cuda(), torch.from_numpy(q).cuda()
    sd = torch.zeros(1, dtype=torch.int32, device="cuda")
    pd = torch.full((1,), n - 1, dtype=torch.int32, device="cuda")
    td = torch.from_numpy(table).cuda()
    o = torch.empty((1, n_head * hd), dtype=torch.float32, device="cuda")
    scale = np.float32(1 / np.sqrt(hd))
    rc = _lib.lib().rtd_attention_paged(_ctx().handle, qd.data_ptr(), 1, n_head, n_kv, hd, scale, sd.data_ptr(),
                                        pd.data_ptr(), td.data_ptr(), max_blocks, n, kd.data_ptr(), vd.data_ptr(),
                                        _lib.DT_F16, o.data_ptr(), _lib.DT_F32, n_head * hd, _st())
    assert rc == 0
    Kf, Vf = K[:, 0].astype(np.float64), V[:, 0].astype(np.float64)
    want = []
    for h in range(n_head):
        sc = Kf @ q[0, h * hd:(h + 1) * hd].astype(np.float64) * float(scale)
        e = np.exp(sc - sc.max())
        want.append((e / e.sum()) @ Vf)
    assert rel_l2(o.cpu().numpy().reshape(-1), np.concatenate(want)) <= 1e-5


def test_silu_mul_and_argmax():
    import torch

    rng = np.random.default_rng(0)
    g = rng.normal(0, 4, 10000).astype(np.float32)
    g[:3] = [-100.0, 100.0, 0.0]  # exp overflow -> -0, large -> x
    u = rng.normal(0, 1, 10000).astype(np.float32)
    gd, ud = torch.from_numpy(g).cuda(), torch.from_numpy(u).cuda()
    y = torch.empty_like(gd)
    L, c = _lib.lib(), _ctx().handle
    assert L.rtd_silu_mul(c, gd.data_ptr(), 0, g.size, ud.data_ptr(), 0, g.size, 1, g.size, y.data_ptr(), 0, g.size,
                          _st()) == 0
    gg = g.astype(np.float64)
    assert rel_l2(y.cpu().numpy(), gg / (1 + np.exp(-gg)) * u) <= 1e-6
    # rows of a fused [gate | up] output, written in place over gate
    gu = np.concatenate([g.reshape(4, 2500), u.reshape(4, 2500)], axis=1)
    gud = torch.from_numpy(gu).cuda()
    assert L.rtd_silu_mul(c, gud.data_ptr(), 0, 5000, gud.data_ptr() + 4 * 2500, 0, 5000, 4, 2500, gud.data_ptr(), 0,
                          5000, _st()) == 0
    got = gud.cpu().numpy()[:, :2500].reshape(-1)
    assert rel_l2(got, gg / (1 + np.exp(-gg)) * u) <= 1e-6
    # argmax: the lowest index among equal maxima, per row
    x = rng.normal(0, 1, (3, 151936)).astype(np.float32)
    x[1, [5, 70000, 151935]] = 9.0
    x[2, :] = -1.0
    xd = torch.from_numpy(x).cuda()
    out = torch.empty(3, dtype=torch.int32, device="cuda")
    assert L.rtd_argmax(c, xd.data_ptr(), x.shape[1], 3, x.shape[1], out.data_ptr(), _st()) == 0
    assert out.cpu().tolist() == [int(np.argmax(x[0])), 5, 0]
