"""rtd_qlinear_argmax: the LM head and the greedy pick in one call (qwen2::forward's
`linear(h, "output.weight")`, crates/runtimed-model/src/arch/qwen2.rs:224-228, followed by
SubstratePort::argmax, crates/runtimed-model/src/decode/sample.rs:11-18).

Below four tokens the pick runs in the decode GEMV's epilogue: each lane keeps a packed
(value, row) key per token, one atomic per warp and token meets in the context's key
words, and the launch's last CTA writes the ids and clears the keys.  Checked on the GPU:
  * ids identical to rtd_argmax over the logits the same call writes, with and without
    the logits written, in whole-mode (LM-head-sized) and split-mode launches, for bf16
    and f32 activations (f32 rows run two tokens a launch, so M = 3 is two launches);
  * the chosen row's float64 oracle value equals the oracle's maximum within the
    linear's own error (a near-tie certificate, as the reference's differential test
    accepts at a divergence);
  * ties go to the lowest row (duplicated weight rows give bit-identical outputs), NaN
    rows never win, all-zero outputs give row 0, a bias alone decides when x is zero;
  * from four tokens the call writes f32 logits and runs rtd_argmax after them;
  * rtd_qlinear_argmax_keys on vocabulary shards (rows numbered from the shard's first
    row): the shards' keys combined by an unsigned maximum give the unsharded ids.
"""
import numpy as np
import pytest

import oracle
from runtimed_b200 import synth

pytestmark = pytest.mark.gpu


def _qm(t, raw, N, K):
    from runtimed_b200.weights import QMatMul

    return QMatMul(t, raw, N, K, device="cuda:0")


def _argmax_rows(y):
    import torch
    from runtimed_b200 import _lib
    from runtimed_b200.weights import Context

    out = torch.empty((y.shape[0],), dtype=torch.int32, device=y.device)
    rc = _lib.lib().rtd_argmax(Context.for_device("cuda:0").handle, y.data_ptr(), y.shape[1], y.shape[0], y.shape[1],
                               out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    return out.cpu().tolist()


def _x(M, K, xdt, seed):
    import torch

    x = synth.bf16_round(synth.activations(M, K, seed=seed))
    return x, torch.from_numpy(x).to(xdt).cuda()


@pytest.mark.parametrize("name,t,N,K,M,xdt", [
    ("Q8_0", 8, 151936, 896, 1, "bf16"),   # config-0 LM head, whole mode, x staged by every CTA
    ("Q8_0", 8, 151936, 896, 1, "f32"),    # whole mode, f32 x through the prep kernel
    ("Q6_K", 14, 5000, 1024, 3, "bf16"),   # split mode, three tokens in one launch
    ("Q4_K", 12, 4096, 2048, 3, "f32"),    # split mode, f32 x: two launches (2 + 1 tokens)
    ("Q8_0", 8, 40000, 512, 2, "bf16"),
])
def test_fused_argmax_matches_logits_argmax(name, t, N, K, M, xdt):
    import torch

    raw = synth.quant_matrix(t, N, K, seed=31, stream=t)
    qm = _qm(t, raw, N, K)
    x, xd = _x(M, K, {"bf16": torch.bfloat16, "f32": torch.float32}[xdt], seed=32)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ids = qm.greedy(xd, logits=y).cpu().tolist()
    ids_nolog = qm.greedy(xd).cpu().tolist()
    assert ids == _argmax_rows(y), name
    assert ids_nolog == ids
    plain = qm.forward(xd, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert float((plain - y).abs().max()) <= 1e-6 * float(plain.abs().max())  # the same logits
    if N * K <= 151936 * 896:
        want = oracle.qgemv_f64(t, raw, N, K, x)
        for r in range(M):
            top = float(want[r].max())
            assert float(want[r, ids[r]]) >= top - 1e-4 * float(np.abs(want[r]).max()), (name, r)


@pytest.mark.parametrize("N", [151936, 5000])
def test_fused_argmax_ties_nan_and_zero_rows(N):
    import torch

    t, K = synth.Q8_0, 256
    nb = K // 32
    raw = synth.quant_matrix(t, N, K, seed=41, stream=3).reshape(N, nb * 34).copy()
    x, xd = _x(1, K, torch.bfloat16, seed=42)
    r = int(_qm(t, raw.reshape(-1), N, K).greedy(xd).cpu()[0])
    lo, mid = (3, 4000) if r not in (3, 4000) else (5, 4001)
    # the winning row copied to two more rows: bit-identical outputs, the lowest row wins
    tied = raw.copy()
    tied[lo] = raw[r]
    tied[mid] = raw[r]
    qm = _qm(t, tied.reshape(-1), N, K)
    y = torch.empty((1, N), dtype=torch.float32, device="cuda")
    got = int(qm.greedy(xd, logits=y).cpu()[0])
    yc = y.cpu().numpy()[0]
    assert yc[lo] == yc[mid] == yc[r]
    assert got == min(lo, mid, r) == _argmax_rows(y)[0]
    # NaN rows (a NaN block scale) never win: the pick is the largest of the others
    nanned = tied.copy()
    for row in (lo, mid, r):
        nanned[row, 0:2] = np.array([0x7E00], dtype=np.uint16).view(np.uint8)
    qm = _qm(t, nanned.reshape(-1), N, K)
    got = int(qm.greedy(xd, logits=y).cpu()[0])
    yc = y.cpu().numpy()[0]
    assert np.isnan(yc[[lo, mid, r]]).all()
    assert got == int(np.nanargmax(yc)) == _argmax_rows(y)[0]
    # zero activations: every finite output is zero (either sign), row 0 wins; a bias
    # decides, and two equal bias values tie exactly (the lower row wins)
    z = torch.zeros((1, K), dtype=torch.bfloat16, device="cuda")
    assert int(qm.greedy(z).cpu()[0]) == 0
    bias = torch.zeros(N, dtype=torch.float32, device="cuda")
    bias[N - 7] = 0.5
    assert int(qm.greedy(z, bias=bias).cpu()[0]) == N - 7
    b1, b2 = [v for v in (10, 11, 12, 13) if v not in (lo, mid, r)][:2]
    bias[b2] = bias[b1] = 0.75
    assert int(qm.greedy(z, bias=bias).cpu()[0]) == b1
    # back-to-back calls start from cleared keys
    assert int(_qm(t, raw.reshape(-1), N, K).greedy(xd).cpu()[0]) == r


def test_fused_argmax_prompt_sizes_and_errors():
    import torch
    from runtimed_b200.errors import ConfigError

    t, N, K, M = synth.Q4_K, 3000, 1024, 6
    raw = synth.quant_matrix(t, N, K, seed=51, stream=1)
    qm = _qm(t, raw, N, K)
    _, xd = _x(M, K, torch.bfloat16, seed=52)
    y = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ids = qm.greedy(xd, logits=y).cpu().tolist()
    assert ids == _argmax_rows(y)
    with pytest.raises(ConfigError):
        qm.greedy(xd)  # four or more tokens need the logits


@pytest.mark.parametrize("world", [2, 8])
def test_vocab_parallel_shards_combine_to_the_unsharded_pick(world):
    # config 0's head split by vocabulary rows over `world` ranks (151936 / 8 = 18992 rows a
    # shard), each shard uploaded on its own with its first row as row0: the shards' keys,
    # combined by an unsigned maximum, give the unsharded head's ids -- five f32 tokens,
    # so three GEMV launches of at most two tokens each, and a tie across shards
    import torch
    from runtimed_b200.tp import VocabParallelHead, combine_keys

    t, N, K, M = synth.Q8_0, 151936, 896, 5
    nb = K // 32
    raw = synth.quant_matrix(t, N, K, seed=61, stream=8).reshape(N, nb * 34).copy()
    _, xd = _x(M, K, torch.float32, seed=62)
    full = _qm(t, raw.reshape(-1), N, K)
    want = full.greedy(xd[:3]).cpu().tolist() + full.greedy(xd[3:]).cpu().tolist()

    def sharded(w):
        keys = [VocabParallelHead.from_full_weight(w.reshape(-1), t, N, K, r, world).local_keys(xd)
                for r in range(world)]
        return combine_keys(torch.stack(keys).cpu()).tolist()

    assert sharded(raw) == want
    r = want[0]
    lo = 1 if r != 1 else 2
    tied = raw.copy()
    tied[lo] = raw[r]  # token 0's winner also in shard 0's row lo: the lower row wins
    full = _qm(t, tied.reshape(-1), N, K)
    want_t = full.greedy(xd[:3]).cpu().tolist() + full.greedy(xd[3:]).cpu().tolist()
    assert want_t[0] == min(lo, r)
    assert sharded(tied) == want_t


def test_reference_greedy_known_answers():
    # decode/sample.rs:173-195: greedy([0.1, 5.0, 2.0]) = 1, and 151646 zeros with 100.0 at
    # row 19 give 19 (the reference's multi-device case; here on cuda:0).  Through
    # rtd_argmax on the logits, and through the fused pick of a head whose outputs are
    # those values (zero activations, the values as the bias; 151646 rows end in a ragged
    # tile of 14), one to three tokens a call
    import torch

    big = np.zeros(151646, np.float32)
    big[19] = 100.0
    for vals, want in ((np.array([0.1, 5.0, 2.0], np.float32), 1), (big, 19)):
        logits = torch.from_numpy(vals[None, :]).cuda()
        assert _argmax_rows(logits) == [want]
        N, K = vals.size, 256
        qm = _qm(synth.Q8_0, synth.quant_matrix(synth.Q8_0, N, K, seed=71), N, K)
        bias = torch.from_numpy(vals).cuda()
        for M in (1, 2, 3):
            z = torch.zeros((M, K), dtype=torch.bfloat16, device="cuda")
            assert qm.greedy(z, bias=bias).cpu().tolist() == [want] * M
