"""Grammar-aware speculative verification of whole proposals in one launch.

The reference's speculative iteration (onyx_cuda/src/onyx_cuda/
grammar_speculative_iteration.py:429-517) decides a proposal in two calls:

* ``decide_grammar_masked_target_acceptance`` (grammar_acceptance.py:166-377) walks the
  positions in order; at each one it asks the grammar for the valid ids of the current
  state, masks the target row, selects (one device->host sync per position), and accepts
  while the selection equals the draft token, advancing the grammar state;
* ``decide_grammar_masked_post_acceptance_continuation`` (grammar_continuation.py:102-152)
  then emits the replacement, or on full acceptance selects the bonus token from the final
  row.

The selection at position i only ever runs under the state reached by accepting drafts
0..i-1, so every position's valid set is known before any row is selected. This module
builds those masks by walking the grammar along the drafts (stopping at the first draft
the grammar does not allow, where the decision is certain to fall), packs them, runs ONE
``spec_verify`` launch for all positions (and all proposals of a batch), reads back three
integers per proposal, and rebuilds the reference's outcome:

* :func:`verify_grammar_proposals` -- this package's own outcome type
  (:class:`ProposalVerdict`) for a batch, with the grammar states it committed;
* :func:`decide_grammar_masked_acceptance_and_continuation` -- the drop-in for the
  reference's pair: the same arguments, and the reference's own result objects
  (``GrammarMaskedTargetAcceptanceResult``, ``GrammarMaskedPostAcceptanceContinuationResult``
  or ``None`` after a no-decision), imported from the installed ``onyx_cuda`` package.

Grammar states follow the reference's ownership rules: the starting state is borrowed and
never released; every state the walk creates is released except the one committed to the
caller (after a bonus selection the acceptance's committed state is released, as the
reference's continuation does). A status at the deciding row raises the drop-in
boundary's errors, as ``mask.apply`` / ``select_cuda_argmax`` would have at that row.
"""

from __future__ import annotations

from bisect import bisect_left
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from typing import Any

import numpy as np
import torch

from . import bitmask as _bitmask
from . import masked_selection as _ms
from .torch_backend import TorchBackendExecutionError, TorchBackendInvariantError
from .torch_grammar_mask import TorchGrammarMaskInvariantError

__all__ = [
    "ProposalVerdict",
    "GrammarProposalWalk",
    "walk_proposal",
    "verify_grammar_proposals",
    "decide_grammar_masked_acceptance_and_continuation",
]


@dataclass(frozen=True)
class ProposalVerdict:
    """Outcome of one proposal of G draft tokens.

    ``accepted_count``: drafts accepted (0..G). Then exactly one of:
    ``replacement_token_id`` (the selection that differed from draft ``accepted_count``),
    ``bonus_token_id`` (full acceptance; the final row's selection), or
    ``no_decision_position`` (the valid set at that position was empty: < G stops inside
    the proposal, == G is a fully accepted proposal whose final row has no valid token).

    ``committed_state`` / ``committed_is_match``: the grammar state handed to the caller and
    its match fact (``None`` after a no-decision at position 0). ``acceptance_state`` /
    ``acceptance_is_match``: the state the acceptance step commits, as the reference's
    acceptance result reports it -- on full acceptance the state after the last draft,
    which a bonus selection supersedes (it is then released), otherwise the same as
    ``committed_state``. ``no_decision_is_match``: the match fact of the state whose valid
    set was empty (``None`` without a no-decision)."""

    accepted_count: int
    replacement_token_id: int | None
    bonus_token_id: int | None
    no_decision_position: int | None
    committed_state: Any
    committed_is_match: bool | None
    acceptance_state: Any
    acceptance_is_match: bool | None
    no_decision_is_match: bool | None


@dataclass
class GrammarProposalWalk:
    """The grammar walked along one proposal: ``states[i]`` is the state in which position
    i is selected (``states[0]`` the borrowed starting state), ``valid[i]`` its valid ids;
    the walk stops after the first position whose draft the grammar does not allow (or whose
    valid set is empty), since the decision falls there."""

    states: list[Any]
    valid: list[tuple[int, ...]]


def walk_proposal(constraint: Any, starting_state: Any, proposal: Sequence[int]) -> GrammarProposalWalk:
    """Walk the grammar along ``proposal`` from ``starting_state`` (see
    :class:`GrammarProposalWalk`). The created states belong to the caller."""
    states = [starting_state]
    valid: list[tuple[int, ...]] = []
    try:
        for i in range(len(proposal) + 1):
            ids = tuple(constraint.get_valid_token_ids(states[i]))
            valid.append(ids)
            if i == len(proposal):
                break
            k = bisect_left(ids, proposal[i])
            if k == len(ids) or ids[k] != proposal[i]:
                break  # position i decides (mismatch or no-decision): later rows are unused
            states.append(constraint.advance_state(states[i], proposal[i]))
    except BaseException:
        _release(constraint, states[1:])
        raise
    return GrammarProposalWalk(states=states, valid=valid)


def _release(constraint: Any, states: Sequence[Any]) -> None:
    for s in states:
        constraint.release_state(s)


def _logits_3d(target_logits: Any, batch: int, g1: int, vocab: int) -> torch.Tensor:
    """[B, G+1, V] view of the target rows: a tensor as is, or a sequence of B tuples of
    G+1 rows -- a strided view when each proposal's rows are evenly spaced slices of one
    buffer (the reference's ``raw_logits[0, i, :vocab]``), else a copy."""
    if isinstance(target_logits, torch.Tensor):
        x = target_logits
        if x.dim() == 2:
            x = x.unsqueeze(0)
        if tuple(x.shape) != (batch, g1, vocab):
            raise ValueError(f"target logits must have shape [{batch}, {g1}, {vocab}]; got {tuple(x.shape)}")
        return x
    per_entry = []
    for rows in target_logits:
        rows = tuple(rows)
        if len(rows) != g1:
            raise ValueError(f"each proposal needs {g1} target rows; got {len(rows)}")
        per_entry.append(_rows_view(rows, vocab))
    return torch.stack(per_entry) if batch > 1 else per_entry[0].unsqueeze(0)


def _rows_view(rows: tuple, vocab: int) -> torch.Tensor:
    first = rows[0]
    if not isinstance(first, torch.Tensor) or first.dim() != 1 or first.shape[0] != vocab:
        raise ValueError(f"target rows must be 1-D tensors of {vocab} logits")
    same = all(isinstance(r, torch.Tensor) and r.dim() == 1 and r.shape[0] == vocab and r.stride(0) == 1
               and r.dtype == first.dtype and r.device == first.device
               and r.untyped_storage().data_ptr() == first.untyped_storage().data_ptr() for r in rows)
    if same and first.stride(0) == 1:
        offs = [r.storage_offset() for r in rows]
        step = offs[1] - offs[0] if len(offs) > 1 else vocab
        if step >= vocab and all(offs[i + 1] - offs[i] == step for i in range(len(offs) - 1)):
            return first.as_strided((len(rows), vocab), (step, 1))
    return torch.stack(rows)


def verify_grammar_proposals(
    target_logits: Any,
    proposals: Sequence[Sequence[int]],
    constraint: Any,
    starting_states: Sequence[Any],
    *,
    vocab_size: int,
    _verify: Callable[..., Any] | None = None,
) -> list[ProposalVerdict]:
    """Decide B proposals of equal length G against their target rows in one launch.

    ``target_logits``: a CUDA tensor [B, G+1, V] (or [G+1, V] for one proposal), or B
    tuples of G+1 CUDA rows. ``proposals``: B sequences of G token ids. Each proposal is
    walked from its own starting state (borrowed). Returns one :class:`ProposalVerdict`
    per proposal; the caller owns each verdict's ``committed_state``.
    ``_verify`` replaces the launch in host-logic tests.
    """
    batch = len(proposals)
    if batch == 0:
        return []
    if len(starting_states) != batch:
        raise ValueError("one starting state per proposal")
    gamma = len(proposals[0])
    if gamma < 1 or any(len(p) != gamma for p in proposals):
        raise ValueError("proposals must be non-empty and of equal length")
    for p in proposals:
        for t in p:
            if isinstance(t, bool) or not isinstance(t, int) or not 0 <= t < vocab_size:
                raise ValueError(f"proposal token {t!r} is outside vocabulary range [0, {vocab_size})")
    x = _logits_3d(target_logits, batch, gamma + 1, vocab_size)
    words = _bitmask.words_for(vocab_size)
    masks = np.zeros((batch, gamma + 1, words), dtype=np.uint32)
    walks: list[GrammarProposalWalk] = []
    verdicts: list[ProposalVerdict] = []
    handed = 0  # walks passed to _verdict, which releases them on every path
    try:
        for b in range(batch):
            walk = walk_proposal(constraint, starting_states[b], proposals[b])
            walks.append(walk)
            for i, ids in enumerate(walk.valid):
                if ids:
                    _bitmask.pack_ids(np.asarray(ids, dtype=np.int64), vocab_size, out=masks[b, i])
        drafts = torch.tensor(np.asarray(proposals, dtype=np.int32))
        if _verify is None:
            dev = x.device
            res = _ms.spec_verify(
                x,
                torch.from_numpy(masks.view(np.int32)).pin_memory().to(dev, non_blocking=True),
                drafts.pin_memory().to(dev, non_blocking=True),
                bonus=True,
            )
            acc, corr, status = torch.stack((res.accept_len, res.correction, res.status)).cpu().numpy()
        else:
            acc, corr, status = _verify(x, masks, drafts.numpy())
        for b in range(batch):
            handed = b + 1
            verdicts.append(_verdict(constraint, walks[b], proposals[b], int(acc[b]), int(corr[b]),
                                     int(status[b]) & 0xFFFFFFFF))
        return verdicts
    except BaseException:
        # nothing is handed over when any proposal fails
        for w in walks[handed:]:
            _release(constraint, w.states[1:])
        _release(constraint, [v.committed_state for v in verdicts if v.committed_state is not None])
        raise


def _raise_for_status(status: int) -> None:
    if status & _ms.STATUS_WAIT_TIMEOUT:
        raise TorchBackendExecutionError("CUDA argmax failed: a bounded in-kernel wait gave up")
    if status & _ms.STATUS_NAN_IN_SUPPORT:
        raise TorchBackendInvariantError("CUDA logits cannot contain NaN")
    if status & _ms.STATUS_ALL_NEG_INF:
        raise TorchGrammarMaskInvariantError("valid token IDs have no logit support above -inf")
    raise TorchBackendExecutionError(f"speculative verify returned status {status:#x}")


def _verdict(constraint: Any, walk: GrammarProposalWalk, proposal: Sequence[int], acc: int,
             corr: int, status: int) -> ProposalVerdict:
    """Turn one proposal's (accept_len, correction, status) into its verdict, creating the
    committed state and releasing every walked state that is not handed over. The walk's
    states are released here on every path, errors included."""
    gamma = len(proposal)
    owned = walk.states[1:]  # states the walk created
    keep = None
    try:
        if status and status != _ms.STATUS_EMPTY_MASK:
            _raise_for_status(status)
        if acc > len(owned):  # the kernel cannot accept past the walk's last state
            raise TorchBackendExecutionError(f"speculative verify accepted {acc} drafts past the grammar walk")
        state = walk.states[acc]
        if status == _ms.STATUS_EMPTY_MASK:  # the valid set at position acc is empty
            match = bool(constraint.is_match_state(state))
            keep = state if acc > 0 else None
            return ProposalVerdict(acc, None, None, acc, keep, match if keep is not None else None,
                                   keep, match if keep is not None else None, match)
        if corr < 0 or (acc < gamma and corr == proposal[acc]):
            raise TorchBackendExecutionError("speculative verify returned an invalid selection")
        child = constraint.advance_state(state, corr)
        child_match = bool(constraint.is_match_state(child))
        if acc < gamma:
            return ProposalVerdict(acc, corr, None, None, child, child_match, child, child_match, None)
        # full acceptance and a bonus: the state after the last draft is superseded
        return ProposalVerdict(acc, None, corr, None, child, child_match, state,
                               bool(constraint.is_match_state(state)), None)
    finally:
        _release(constraint, [s for s in owned if s is not keep])


def decide_grammar_masked_acceptance_and_continuation(
    proposal_token_ids: tuple[int, ...],
    target_logit_rows: tuple[Any, ...],
    constraint: Any,
    starting_state: Any,
    logit_mask: Any = None,
    *,
    vocab_size: int,
    select_token: Callable[[Any], int] | None = None,
    _verify: Callable[..., Any] | None = None,
) -> tuple[Any, Any]:
    """Drop-in for the reference's pair ``decide_grammar_masked_target_acceptance`` +
    ``decide_grammar_masked_post_acceptance_continuation`` (same arguments; the mask and
    the selector are not called: one fused launch masks and selects every row).

    Returns ``(acceptance_result, continuation_result)`` as the reference's own types; the
    continuation is ``None`` after a no-decision inside the proposal, where the reference's
    coordinator does not call it (grammar_speculative_iteration.py:496-510). After a bonus
    selection the acceptance's committed state has been released, as the reference's
    continuation releases it; the continuation's committed state belongs to the caller."""
    from onyx_cuda.grammar_acceptance import GrammarMaskedTargetAcceptanceResult
    from onyx_cuda.grammar_continuation import GrammarMaskedPostAcceptanceContinuationResult
    from onyx_cuda.grammar_selection import GrammarMaskedSelectionResult

    if type(proposal_token_ids) is not tuple or not proposal_token_ids:
        raise ValueError("proposal_token_ids must be a non-empty tuple")
    if type(target_logit_rows) is not tuple or len(target_logit_rows) != len(proposal_token_ids) + 1:
        raise ValueError(f"target_logit_rows must hold {len(proposal_token_ids) + 1} rows")
    if logit_mask is not None and getattr(logit_mask, "vocab_size", vocab_size) != vocab_size:
        raise ValueError("logit_mask vocabulary size differs from vocab_size")
    gamma = len(proposal_token_ids)
    v = verify_grammar_proposals((target_logit_rows,), [proposal_token_ids], constraint,
                                 [starting_state], vocab_size=vocab_size, _verify=_verify)[0]
    acc = v.accepted_count
    inside = v.no_decision_position is not None and acc < gamma
    no_decision = (GrammarMaskedSelectionResult(valid_token_ids=(), is_match=v.no_decision_is_match,
                                                selected_token_id=None) if inside else None)
    acceptance = GrammarMaskedTargetAcceptanceResult(
        proposal_token_ids=proposal_token_ids,
        accepted_count=acc,
        replacement_token_id=v.replacement_token_id,
        no_decision_selection=no_decision,
        committed_state=v.acceptance_state,
        committed_state_is_match=v.acceptance_is_match,
    )
    if inside:
        return acceptance, None
    if v.replacement_token_id is not None:
        out, nxt, final_empty = proposal_token_ids[:acc] + (v.replacement_token_id,), v.replacement_token_id, None
    elif v.bonus_token_id is not None:
        out, nxt, final_empty = proposal_token_ids + (v.bonus_token_id,), v.bonus_token_id, None
    else:  # fully accepted, and the final row has no valid token
        out, nxt = proposal_token_ids, None
        final_empty = GrammarMaskedSelectionResult(valid_token_ids=(), is_match=v.no_decision_is_match,
                                                   selected_token_id=None)
    continuation = GrammarMaskedPostAcceptanceContinuationResult(
        output_token_ids=out,
        uncached_next_token_id=nxt,
        final_row_no_decision_selection=final_empty,
        committed_state=v.committed_state,
        committed_state_is_match=v.committed_is_match,
    )
    return acceptance, continuation
