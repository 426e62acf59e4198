"""Greedy speculative decoding's host logic (runtimed_b200/speculate.py, after
crates/runtimed-model/src/decode/speculate.rs:17-199) on stub decoders, CPU only.

A stub decoder is a deterministic next-token rule over its cached tokens, with a KV cache
that insists every forward start exactly where the cache ends -- so each rollback
(truncate) and each re-feed of a correction, bonus or unseen proposal is checked, as the
reference checks its decode loop with canned-logit stubs (decode/generate.rs:130-151).
The speculative tokens must equal the target's own greedy decode for any draft.

The paged KV cache's block bookkeeping (PagedKvCache, after cache/paged/table.rs:57-145)
is checked on the CPU too: blocks spanned, rollback returning blocks to the pool, the
block table, and the limits.
"""
import numpy as np
import pytest
import torch

from runtimed_b200.speculate import speculative_generate

V = 97


class _Cache:
    def __init__(self):
        self.seqs = {}

    def release(self, seq):
        self.seqs[seq] = []

    def truncate(self, seq, n):
        assert n <= len(self.seqs[seq])
        self.seqs[seq] = self.seqs[seq][:n]


class _Stub:
    def __init__(self, rule):
        self.rule, self.cache, self.forwards = rule, _Cache(), 0

    def forward(self, ids, q0, seq=0, last_only=False):
        toks = self.cache.seqs.setdefault(seq, [])
        assert len(toks) == q0, f"forward at {q0} with {len(toks)} cached tokens"
        self.forwards += 1
        rows = []
        for t in ids:
            toks.append(int(t))
            row = torch.full((V,), -1.0)
            row[self.rule(toks)] = 1.0
            rows.append(row)
        out = torch.stack(rows)
        return out[-1:] if last_only else out

    def argmax(self, rows):
        return torch.argmax(rows, dim=1).to(torch.int32)


def _target_rule(toks):
    return (3 * toks[-1] + len(toks)) % V


def _greedy(rule, prompt, n):
    toks = list(prompt)
    out = []
    for _ in range(n):
        t = rule(toks)
        out.append(t)
        toks.append(t)
    return out


@pytest.mark.parametrize("k", [1, 2, 4, 7])
@pytest.mark.parametrize("agree", [1.0, 0.7, 0.0])
def test_speculative_tokens_equal_the_target_greedy(k, agree):
    rng = np.random.default_rng(int(k * 10 + agree * 100))
    flips = set(int(v) for v in rng.integers(0, V, int((1.0 - agree) * V)))

    def draft_rule(toks):  # the target's rule, wrong where the last token is in `flips`
        t = _target_rule(toks)
        return (t + 5) % V if toks[-1] in flips else t

    prompt = [int(v) for v in rng.integers(0, V, 9)]
    target, draft = _Stub(_target_rule), _Stub(draft_rule)
    st = speculative_generate(draft, target, prompt, 40, k=k)
    assert st.tokens == _greedy(_target_rule, prompt, 40)
    assert st.accepted <= st.proposed
    if agree == 1.0:  # the draft always agrees: every proposal accepted, a bonus each round
        assert st.accepted == st.proposed
        assert st.target_forwards <= -(-40 // (k + 1)) + 1


def test_speculative_stops_at_eos():
    prompt = [3, 1, 4, 1, 5]
    want = _greedy(_target_rule, prompt, 60)
    eos = want[17]
    st = speculative_generate(_Stub(_target_rule), _Stub(_target_rule), prompt, 60, k=4, eos=[eos])
    assert st.tokens == want[:want.index(eos) + 1]


def _cache(num_blocks=8, max_seqs=3, max_ctx=128):
    from runtimed_b200.qwen2 import PagedKvCache, Qwen2Config

    cfg = Qwen2Config(n_layer=1, hidden=64, n_head=2, n_kv=2, head_dim=4, ffn=128, vocab=V, eps=1e-6,
                      rope_theta=1e6, has_qkv_bias=False)
    return PagedKvCache(cfg, num_blocks, max_seqs, max_ctx, "cpu", dtype=torch.float32)


def test_paged_cache_spans_blocks_and_rolls_back():
    # cache/paged/table.rs:169-215: 25 tokens span two 16-token blocks and one more token
    # stays in the second; 35 tokens take three, a rollback to 20 keeps two, and two more
    # tokens after it make 22 in the same two blocks
    from runtimed_b200.errors import ConfigError

    c = _cache()
    c.reserve(0, 25)
    assert len(c._blocks[0]) == 2 and c.lengths[0] == 25
    c.reserve(0, 26)
    assert len(c._blocks[0]) == 2 and c.lengths[0] == 26
    c.reserve(1, 35)
    assert len(c._blocks[1]) == 3
    third = c._blocks[1][2]
    c.truncate(1, 20)
    assert len(c._blocks[1]) == 2 and c.lengths[1] == 20
    assert third in c._free  # the rolled-back block returns to the pool
    c.reserve(1, 22)
    assert len(c._blocks[1]) == 2 and c.lengths[1] == 22
    # the device table holds each sequence's blocks in order, after sync
    c.sync_table()
    assert c.table[0, :2].tolist() == c._blocks[0] and c.table[1, :2].tolist() == c._blocks[1]
    # no block is owned twice; release returns them all
    owned = c._blocks[0] + c._blocks[1]
    assert len(set(owned)) == len(owned) and not set(owned) & set(c._free)
    c.release(0)
    c.release(1)
    assert sorted(c._free) == list(range(8))
    # limits: the pool, the context length, the sequence slots
    c.reserve(2, 8 * 16)
    with pytest.raises(ConfigError):
        c.reserve(0, 1)  # out of blocks
    c.release(2)
    with pytest.raises(ConfigError):
        c.reserve(0, 129)  # past max_ctx
    with pytest.raises(ConfigError):
        c.reserve(3, 1)  # no such sequence slot


def test_session_greedy_and_truncate_on_a_stub():
    # Session (decode/session.rs:157-166): prefill, one forward per step at the next
    # position, and truncate to roll back -- on the stub, every forward starts where the
    # cache ends
    from runtimed_b200.qwen2 import Session

    prompt = [7, 11, 13]
    stub = _Stub(_target_rule)
    s = Session(stub, seq=0)
    ids, rows = s.greedy(prompt, 12)
    assert ids == _greedy(_target_rule, prompt, 12)
    assert len(rows) == 13 and s.pos == len(prompt) + 12
    s.truncate(len(prompt) + 4)  # keep four generated tokens
    logits = s.step(ids[4])
    assert int(torch.argmax(logits)) == ids[5]
