"""Greedy speculative decoding over two decoders (draft and target).

Mirrors ``speculative_step`` at temperature 0 (crates/runtimed-model/src/decode/speculate.rs:17-199):
  1. the draft proposes up to k tokens greedily from its head row, one M = 1 forward each;
  2. the target verifies them in ONE forward of the k tokens at the current position
     (the k + 1 positions the configs count: its head row plus the k new rows);
  3. candidates are accepted while they equal the target's argmax; the first mismatch is
     replaced by the target's token; if all k are accepted the target's last row gives a
     bonus token;
  4. both KV caches are rolled back to the accepted length (a paged-cache truncation) and
     the next head rows come from forwarding the correction / bonus token.
With greedy acceptance the output equals the target's own greedy decode.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Sequence

from .qwen2 import Qwen2Model


@dataclass
class SpeculativeStats:
    tokens: List[int] = field(default_factory=list)
    proposed: int = 0
    accepted: int = 0
    target_forwards: int = 0


def _argmax(model: Qwen2Model, row) -> int:
    return int(model.argmax(row[None, :])[0])


def speculative_generate(draft: Qwen2Model, target: Qwen2Model, prompt: Sequence[int], n_tokens: int, k: int = 4,
                         seq: int = 0, eos: Sequence[int] = ()) -> SpeculativeStats:
    """Generate `n_tokens` after `prompt` (greedy); returns the tokens and acceptance counts."""
    k = max(1, int(k))
    draft.cache.release(seq)
    target.cache.release(seq)
    d_head = draft.forward(list(prompt), 0, seq=seq, last_only=True)[-1]
    t_head = target.forward(list(prompt), 0, seq=seq, last_only=True)[-1]
    pos = len(prompt)
    st = SpeculativeStats()
    while len(st.tokens) < n_tokens:
        # 1. draft proposals
        cand, row = [], d_head
        for j in range(k):
            tok = _argmax(draft, row)
            cand.append(tok)
            if tok in eos or j + 1 == k:
                break
            row = draft.forward([tok], pos + j, seq=seq)[-1]
        # 2. one target forward over the candidates
        t_logits = target.forward(cand, pos, seq=seq)
        st.target_forwards += 1
        st.proposed += len(cand)
        # 3. greedy acceptance
        accepted, n_acc, hit_eos, head = [], 0, False, t_head
        for i, c in enumerate(cand):
            t_tok = _argmax(target, head)
            if c == t_tok:
                accepted.append(c)
                n_acc += 1
                if c in eos:
                    hit_eos = True
                    break
                head = t_logits[i]
            else:
                accepted.append(t_tok)
                hit_eos = t_tok in eos
                break
        all_acc = n_acc == len(cand)
        if all_acc and not hit_eos:
            accepted.append(_argmax(target, t_logits[len(cand) - 1]))  # the bonus token
            hit_eos = accepted[-1] in eos
        st.accepted += n_acc
        # 4. rollback and the next head rows
        if not all_acc:
            corr, corr_pos = accepted[-1], pos + n_acc
            target.cache.truncate(seq, corr_pos)
            draft.cache.truncate(seq, corr_pos)
            if not hit_eos:
                t_head = target.forward([corr], corr_pos, seq=seq)[-1]
                d_head = draft.forward([corr], corr_pos, seq=seq)[-1]
        elif not hit_eos:
            bonus, p_last = accepted[-1], pos + len(cand)
            t_head = target.forward([bonus], p_last, seq=seq)[-1]
            # the draft has not seen its own last proposal yet: feed it and the bonus
            d_head = draft.forward([cand[-1], bonus], p_last - 1, seq=seq)[-1]
        st.tokens.extend(accepted)
        pos += len(accepted)
        if hit_eos:
            break
    st.tokens = st.tokens[:n_tokens]
    return st
