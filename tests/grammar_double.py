"""A scripted grammar constraint for tests: the reference's GrammarConstraint protocol
(onyx_cuda/src/onyx_cuda/grammar.py:35-58) over an explicit state table.

States are named; each admits a sorted tuple of token ids, and each admitted id leads to a
named state. Handles are fresh objects per created state; releasing one removes it, and
``active_state_count`` counts the live ones, so tests can check state ownership."""

from __future__ import annotations

import itertools
from collections.abc import Iterable, Sequence


class ScriptedGrammar:
    def __init__(self, vocab_size: int, valid: Iterable[tuple[str, Sequence[int]]],
                 transitions: Iterable[tuple[str, int, str]], match_states: Iterable[str],
                 initial: str) -> None:
        self.vocab_size = vocab_size
        self.grammar_type = "regex"
        self._valid = {name: tuple(sorted(ids)) for name, ids in valid}
        self._next = {(s, t): d for s, t, d in transitions}
        self._match = frozenset(match_states)
        self._initial = initial
        self._live: dict[int, str] = {}
        self._keys = itertools.count(1)

    class Handle:
        __slots__ = ("key",)

        def __init__(self, key: int) -> None:
            self.key = key

    def _new(self, name: str) -> "ScriptedGrammar.Handle":
        h = ScriptedGrammar.Handle(next(self._keys))
        self._live[h.key] = name
        return h

    def name(self, state: "ScriptedGrammar.Handle | None") -> str | None:
        return None if state is None else self._live[state.key]

    def init_state(self):
        return self._new(self._initial)

    def advance_state(self, state, token_id: int, /):
        name = self._live[state.key]
        if (name, token_id) not in self._next:
            raise ValueError(f"token {token_id} is not valid in state {name}")
        return self._new(self._next[(name, token_id)])

    def get_valid_token_ids(self, state, /) -> tuple[int, ...]:
        return self._valid.get(self._live[state.key], ())

    def is_match_state(self, state, /) -> bool:
        return self._live[state.key] in self._match

    def is_dead_state(self, state, /) -> bool:
        return False

    def release_state(self, state, /) -> None:
        del self._live[state.key]

    def release_states(self, states, /) -> None:
        for s in states:
            self.release_state(s)

    @property
    def active_state_count(self) -> int:
        return len(self._live)

