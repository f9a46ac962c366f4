"""The batched grammar verifier on the GPU (one spec_verify launch through the C ABI) on the
full 32 x 5 x 151,936 bf16 verify workload, against the oracle's speculative verify.

Each batch entry walks its own chain grammar whose state at position i admits exactly the
workload's mask of (entry, i). Some entries are changed so that every outcome occurs: a
draft the grammar does not allow (the walk stops there and the later masks stay empty), an
empty valid set inside the proposal (no-decision) and in the final row."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from onyx_b200 import bitmask, grammar_verify, workloads
from tests.gpu_util import requires_cuda, to_device

pytestmark = [pytest.mark.gpu, requires_cuda]


class ChainGrammar:
    """State (b, i) admits the ids of mask (b, i); every admitted id leads to (b, i + 1)."""

    vocab_size = 151936
    grammar_type = "regex"

    def __init__(self, masks: np.ndarray) -> None:
        self.masks = masks
        self.live: dict[int, tuple[int, int]] = {}
        self.next_key = 0

    def _new(self, b: int, i: int) -> int:
        self.next_key += 1
        self.live[self.next_key] = (b, i)
        return self.next_key

    def get_valid_token_ids(self, s, /):
        b, i = self.live[s]
        if i >= self.masks.shape[1]:
            return ()
        return tuple(np.flatnonzero(bitmask.unpack(self.masks[b, i], self.vocab_size)).tolist())

    def advance_state(self, s, t, /):
        b, i = self.live[s]
        if not (self.masks[b, i, t >> 5] >> (t & 31)) & 1:
            raise ValueError("token not allowed")
        return self._new(b, i + 1)

    def is_match_state(self, s, /):
        return self.live[s][1] == self.masks.shape[1]

    def is_dead_state(self, s, /):
        return False

    def release_state(self, s, /):
        del self.live[s]


def test_full_verify_workload_through_the_grammar_walk(cuda_lib):
    w = workloads.spec_verify(lambda x, m: oracle.masked_argmax(x, m, dtype="bf16")[0])
    x, masks, drafts = w["logits_bf16"], w["masks"].copy(), w["drafts"].copy()
    masks[3, 2] = 0           # no valid token at position 2 of entry 3, reached by
    drafts[3, :2] = oracle.masked_argmax(x[3, :2], masks[3, :2], dtype="bf16")[0]
    drafts[3, 2:] = 0         # accepting drafts 0 and 1
    masks[7, 4] = 0           # entry 7: the final row admits nothing
    drafts[7] = oracle.masked_argmax(x[7], masks[7], dtype="bf16")[0][:4]  # accepted in full
    bad = int(np.flatnonzero(~bitmask.unpack(masks[5, 1], 151936))[0])
    drafts[5, 1] = bad        # entry 5: a draft the grammar does not allow
    acc_ref, corr_ref, st_ref = oracle.spec_verify(x, masks, drafts, dtype="bf16")

    g = ChainGrammar(masks)
    starts = [g._new(b, 0) for b in range(x.shape[0])]
    verdicts = grammar_verify.verify_grammar_proposals(
        to_device(x, "bf16"), [tuple(int(t) for t in d) for d in drafts], g, starts,
        vocab_size=151936)
    gamma = drafts.shape[1]
    kinds = set()
    for b, v in enumerate(verdicts):
        assert v.accepted_count == acc_ref[b], b
        if st_ref[b] == oracle.STATUS_BITS["empty"]:
            assert v.no_decision_position == acc_ref[b], b
            kinds.add("no-decision" if acc_ref[b] < gamma else "final-row-empty")
        elif acc_ref[b] < gamma:
            assert st_ref[b] == 0 and v.replacement_token_id == corr_ref[b], b
            kinds.add("replacement")
        else:
            assert st_ref[b] == 0 and v.bonus_token_id == corr_ref[b], b
            kinds.add("bonus")
    assert kinds == {"no-decision", "final-row-empty", "replacement", "bonus"}
    assert verdicts[5].accepted_count <= 1
    # alive: the 32 starting states and one committed state per verdict that has one
    assert len(g.live) == 32 + sum(v.committed_state is not None for v in verdicts)
