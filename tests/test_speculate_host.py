"""Greedy speculative decoding's host logic (runtimed_b200/speculate.py, after
crates/runtimed-model/src/decode/speculate.rs:17-199) on stub decoders, CPU only.

A stub decoder is a deterministic next-token rule over its cached tokens, with a KV cache
that insists every forward start exactly where the cache ends -- so each rollback
(truncate) and each re-feed of a correction, bonus or unseen proposal is checked, as the
reference checks its decode loop with canned-logit stubs (decode/generate.rs:130-151).
The speculative tokens must equal the target's own greedy decode for any draft.
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
