"""Host logic of the batched grammar verifier (onyx_b200.grammar_verify) against whole
speculative iterations decided by the reference's own code.

``iteration_cases.json`` holds, for a branching scripted grammar, what the reference's
``decide_grammar_masked_target_acceptance`` + ``decide_grammar_masked_post_acceptance_
continuation`` returned (grammar_acceptance.py:166, grammar_continuation.py:102): the
accepted count, replacement, no-decision selections, committed states and match facts,
output tokens, and how many grammar states were left alive. Here the same grammar (a
test double of the GrammarConstraint protocol) is walked by the verifier; the one launch
it makes is replaced by the oracle's speculative verify on the host (the GPU run of the
same path is tests/test_gpu_grammar_verify.py).

When ``ONYX_REFERENCE_ROOT`` names a checkout of the reference, the drop-in entry point
is also driven with the reference's own FakeGrammarConstraint and its result objects are
compared with the reference pair's, field by field."""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from onyx_b200 import grammar_verify as gv
from tests.conftest import load_golden
from tests.grammar_double import ScriptedGrammar

CASES = load_golden("iteration_cases.json")["cases"]


def _host_verify(x, masks, drafts):
    """The launch's contract on the host: (accept_len, correction, status) per entry."""
    xs = np.ascontiguousarray(x.detach().cpu().numpy(), dtype=np.float32)
    return oracle.spec_verify(xs, masks, np.asarray(drafts, np.int32), bonus=True, dtype="f32")


def _grammar(case) -> ScriptedGrammar:
    return ScriptedGrammar(case["vocab_size"], [(n, ids) for n, ids in case["states"]],
                           [tuple(t) for t in case["transitions"]], case["match_states"], "q0")


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_verdict_matches_reference_iteration(case, oracle_lib):
    g = _grammar(case)
    start = g.init_state()
    rows = torch.tensor(case["rows_f32"], dtype=torch.float32)
    drafts = tuple(case["drafts"])
    v = gv.verify_grammar_proposals(rows, [drafts], g, [start], vocab_size=case["vocab_size"],
                                    _verify=_host_verify)[0]
    gamma = case["gamma"]
    assert v.accepted_count == case["accepted_count"]
    assert v.replacement_token_id == case["replacement_token_id"]
    cont = case["continuation"]
    if cont is None:  # a no-decision inside the proposal
        assert v.no_decision_position == v.accepted_count < gamma
        assert v.no_decision_is_match == case["no_decision_is_match"]
    else:
        final_empty = cont["final_row_no_decision_is_match"]
        if final_empty is not None:
            assert v.no_decision_position == gamma and v.no_decision_is_match == final_empty
            out = drafts
        elif v.replacement_token_id is not None:
            out = drafts[: v.accepted_count] + (v.replacement_token_id,)
        else:
            out = drafts + (v.bonus_token_id,)
        assert list(out) == cont["output_token_ids"]
        assert g.name(v.committed_state) == cont["committed_state"]
        assert v.committed_is_match == cont["committed_is_match"]
    # the acceptance step's committed state: its name was read before the continuation
    # could release it
    if case["acceptance_state"] is not None and v.bonus_token_id is None:
        assert g.name(v.acceptance_state) == case["acceptance_state"]
    assert v.acceptance_is_match == case["acceptance_is_match"]
    # alive afterwards: the starting state, plus the state handed to the caller
    assert g.active_state_count == case["active_states_after"]


def test_batch_of_proposals_in_one_call(oracle_lib):
    """Several proposals (each with its own grammar walk) decided by one launch give the
    same verdicts as one call per proposal."""
    picked = [c for c in CASES if c["gamma"] == 3 and c["vocab_size"] >= 16][:6]
    assert len(picked) >= 2
    vocab = max(c["vocab_size"] for c in picked)
    # one grammar holding every case's states under distinct names
    valid, trans, match = [], [], []
    for k, c in enumerate(picked):
        valid += [(f"c{k}{n}", ids) for n, ids in c["states"]]
        trans += [(f"c{k}{s}", t, f"c{k}{d}") for s, t, d in c["transitions"]]
        match += [f"c{k}{n}" for n in c["match_states"]]
    g = ScriptedGrammar(vocab, valid, trans, match, "c0q0")
    starts = [g._new(f"c{k}q0") for k in range(len(picked))]
    rows = torch.full((len(picked), 4, vocab), -1.0e30, dtype=torch.float32)
    for k, c in enumerate(picked):
        rows[k, :, : c["vocab_size"]] = torch.tensor(c["rows_f32"])
    verdicts = gv.verify_grammar_proposals(rows, [tuple(c["drafts"]) for c in picked], g, starts,
                                           vocab_size=vocab, _verify=_host_verify)
    for v, c in zip(verdicts, picked):
        assert v.accepted_count == c["accepted_count"]
        assert v.replacement_token_id == c["replacement_token_id"]
    assert g.active_state_count == len(picked) + sum(v.committed_state is not None for v in verdicts)


def test_rows_from_one_padded_buffer_are_a_view():
    raw = torch.randn(1, 5, 40)
    rows = tuple(raw[0, i, :33] for i in range(5))
    view = gv._rows_view(rows, 33)
    assert view.data_ptr() == raw.data_ptr() and view.stride() == (40, 1)
    assert torch.equal(view, raw[0, :, :33])
    shuffled = (rows[1], rows[0], rows[2], rows[3], rows[4])
    assert torch.equal(gv._rows_view(shuffled, 33), torch.stack(shuffled))


def test_walk_stops_at_the_first_disallowed_draft_and_releases_on_errors(oracle_lib):
    g = ScriptedGrammar(8, [("a", (1, 2)), ("b", (3,)), ("c", (4,))],
                        [("a", 1, "b"), ("a", 2, "c"), ("b", 3, "a"), ("c", 4, "a")], [], "a")
    start = g.init_state()
    w = gv.walk_proposal(g, start, (1, 3, 5, 1))
    assert [g.name(s) for s in w.states] == ["a", "b", "a"]
    assert w.valid == [(1, 2), (3,), (1, 2)]  # draft 5 is not allowed in "a": stop
    gv._release(g, w.states[1:])
    assert g.active_state_count == 1

    def failing_verify(x, masks, drafts):
        raise RuntimeError("launch failed")

    with pytest.raises(RuntimeError, match="launch failed"):
        gv.verify_grammar_proposals(torch.zeros(1, 5, 8), [(1, 3, 1, 3)], g, [start],
                                    vocab_size=8, _verify=failing_verify)
    assert g.active_state_count == 1  # every walked state was released


def test_status_at_the_deciding_row_raises_the_boundary_errors(oracle_lib):
    g = ScriptedGrammar(4, [("a", (0, 1, 2))], [("a", t, "a") for t in (0, 1, 2)], [], "a")
    start = g.init_state()
    rows = torch.zeros(1, 3, 4)
    rows[0, 0, :] = float("-inf")  # position 0: all valid values -inf
    with pytest.raises(gv.TorchGrammarMaskInvariantError, match="no logit support"):
        gv.verify_grammar_proposals(rows, [(0, 1)], g, [start], vocab_size=4, _verify=_host_verify)
    rows[0, 0, :] = 0.0
    rows[0, 0, 1] = float("nan")
    with pytest.raises(gv.TorchBackendInvariantError, match="NaN"):
        gv.verify_grammar_proposals(rows, [(0, 1)], g, [start], vocab_size=4, _verify=_host_verify)
    assert g.active_state_count == 1


# ---------------------------------------------------------------------------------------
# the drop-in entry point against the reference's own objects (needs its checkout)
# ---------------------------------------------------------------------------------------
def _reference_modules():
    root = os.environ.get("ONYX_REFERENCE_ROOT")
    if not root or not (Path(root) / "onyx_cuda" / "src").is_dir():
        pytest.skip("set ONYX_REFERENCE_ROOT to a checkout of the reference to run this test")
    src = str(Path(root) / "onyx_cuda" / "src")
    if src not in sys.path:
        sys.path.insert(0, src)
    import onyx_cuda.grammar_acceptance as acc
    import onyx_cuda.grammar_continuation as cont
    import onyx_cuda.testing as testing
    from onyx_cuda.generation import select_highest_logit
    return acc, cont, testing, select_highest_logit


class _ListMask:
    def __init__(self, vocab_size: int) -> None:
        self.vocab_size = vocab_size

    def apply(self, logits, valid_token_ids, /):
        keep = set(valid_token_ids)
        return tuple(x if i in keep else float("-inf") for i, x in enumerate(logits))


@pytest.mark.parametrize("case", CASES[:30], ids=[c["name"] for c in CASES[:30]])
def test_drop_in_returns_the_reference_result_objects(case, oracle_lib):
    acc_mod, cont_mod, testing, select_highest_logit = _reference_modules()
    program = testing.FakeGrammarProgram(
        initial_state="q0", transitions=tuple(tuple(t) for t in case["transitions"]),
        valid_token_ids=tuple((n, tuple(ids)) for n, ids in case["states"]),
        match_states=frozenset(case["match_states"]))
    vocab = tuple(f"t{i}".encode() for i in range(case["vocab_size"]))
    drafts = tuple(case["drafts"])
    rows_t = tuple(torch.tensor(r, dtype=torch.float32) for r in case["rows_f32"])
    rows_l = tuple(tuple(r) for r in case["rows_f32"])
    v = case["vocab_size"]

    ref_c = testing.FakeGrammarConstraint(vocab, grammar_type="regex", program=program)
    ref_start = ref_c.init_state()
    ref_a = acc_mod.decide_grammar_masked_target_acceptance(
        drafts, rows_l, ref_c, ref_start, _ListMask(v), vocab_size=v, select_token=select_highest_logit)
    ref_a_state = None if ref_a.committed_state is None else ref_c._states[ref_a.committed_state.value]
    ref_k = None
    if ref_a.decision_made:
        ref_k = cont_mod.decide_grammar_masked_post_acceptance_continuation(
            drafts, rows_l, ref_a, ref_c, _ListMask(v), vocab_size=v, select_token=select_highest_logit)

    our_c = testing.FakeGrammarConstraint(vocab, grammar_type="regex", program=program)
    our_start = our_c.init_state()
    our_a, our_k = gv.decide_grammar_masked_acceptance_and_continuation(
        drafts, rows_t, our_c, our_start, _ListMask(v), vocab_size=v, _verify=_host_verify)

    assert type(our_a) is type(ref_a)
    for f in ("proposal_token_ids", "accepted_count", "replacement_token_id",
              "no_decision_selection", "committed_state_is_match"):
        assert getattr(our_a, f) == getattr(ref_a, f), f
    assert (our_a.committed_state is None) == (ref_a.committed_state is None)
    if our_a.committed_state is not None and (our_k is None or our_k.uncached_next_token_id is None
                                              or our_a.replacement_token_id is not None):
        assert our_c._states[our_a.committed_state.value] == ref_a_state
    assert (our_k is None) == (ref_k is None)
    if ref_k is not None:
        assert type(our_k) is type(ref_k)
        for f in ("output_token_ids", "uncached_next_token_id", "final_row_no_decision_selection",
                  "committed_state_is_match"):
            assert getattr(our_k, f) == getattr(ref_k, f), f
        assert our_c._states[our_k.committed_state.value] == ref_c._states[ref_k.committed_state.value]
    assert our_c.active_state_count == ref_c.active_state_count
