"""Dense byte-DFA restatement of the reference's regex constraint -- TEST INFRASTRUCTURE ONLY.

This module is part of the oracle: only tests, the smoke check and the CPU-baseline
leg of the benchmark use it, as the checker.

The reference compiles a regex with ``regex-automata`` 0.4.15 (``regex-syntax`` 0.8.11;
onyx_cuda/rust/Cargo.lock:162-174) into an anchored dense DFA with
``MatchKind::LeftmostFirst`` (onyx_cuda/rust/src/regex_runtime.rs:71-85) and then:

* ``transition``      folds ``next_state`` over a token's bytes (regex_runtime.rs:197-201);
* ``get_valid_token_ids`` keeps every non-empty token whose walk does not end dead
  (regex_runtime.rs:129-145);
* ``is_match_state``  is false for dead, else the EOI transition's match flag (:147-156);
* ``is_dead_state``   is the DFA's dead test (:158-163).

That crate's source is not available here, so this file restates its published
determinisation algorithm for the pattern subset the workloads need:

1. Thompson NFA with prioritised alternation (``Union`` alternates in priority order;
   greedy repetition prefers another iteration, lazy prefers leaving).
2. Epsilon closure as a depth-first walk that visits the first alternate immediately and
   stacks the rest in reverse, recording states in first-visit order.
3. ``next(S, byte)`` walks S's NFA states in that order; a ``Match`` state marks the
   *next* DFA state as matching and, for leftmost-first, stops the walk (lower-priority
   threads are dropped); byte transitions that accept the byte contribute the closure of
   their target. Matches are therefore reported one byte late: after the last byte of a
   match any byte enters a non-dead "delayed match" state, and only the byte after that is
   dead. The EOI transition is the same walk with no byte accepted.
4. The dead state is the state with no NFA states and no match flag.

Supported syntax: literals, ``\\`` escapes of metacharacters, ``\\xHH`` and ``\\x{H..}``
(Unicode scalar encoded as UTF-8 bytes), non-negated ASCII classes ``[a-z0-9_]``,
``(...)``, ``(?:...)``, ``|``, ``*``, ``+``, ``?``, ``{n}``, ``{n,}``, ``{n,m}`` and their lazy
``?`` forms. Anything else raises ``ValueError`` rather than guessing.

Pinned by the reference's frozen black-box outcomes,
onyx_cuda/tests/regex_parity_fixtures.py:22-104 (committed as tests/golden/regex_parity.json).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

__all__ = ["ByteDFA", "compile_regex_dfa"]


# ---------------------------------------------------------------------------
# parser -> AST
# ---------------------------------------------------------------------------
# AST nodes: ("bytes", set_of_byte_values) | ("cat", [nodes]) | ("alt", [nodes])
#            ("rep", node, min, max_or_None, greedy) | ("empty",)

_META = set("\\.+*?()|[]{}^$")


class _Parser:
    def __init__(self, pattern: str) -> None:
        self.p = pattern
        self.i = 0

    def error(self, msg: str) -> ValueError:
        return ValueError(f"unsupported or invalid regex at {self.i}: {msg} in {self.p!r}")

    def peek(self) -> str | None:
        return self.p[self.i] if self.i < len(self.p) else None

    def take(self) -> str:
        if self.i >= len(self.p):
            raise self.error("unexpected end")
        ch = self.p[self.i]
        self.i += 1
        return ch

    def parse(self):
        node = self.parse_alt()
        if self.i != len(self.p):
            raise self.error("unbalanced ')'")
        return node

    def parse_alt(self):
        branches = [self.parse_cat()]
        while self.peek() == "|":
            self.i += 1
            branches.append(self.parse_cat())
        return branches[0] if len(branches) == 1 else ("alt", branches)

    def parse_cat(self):
        items = []
        while self.peek() is not None and self.peek() not in "|)":
            items.append(self.parse_repeat())
        if not items:
            return ("empty",)
        return items[0] if len(items) == 1 else ("cat", items)

    def parse_repeat(self):
        atom = self.parse_atom()
        while True:
            ch = self.peek()
            if ch == "*":
                self.i += 1
                lo, hi = 0, None
            elif ch == "+":
                self.i += 1
                lo, hi = 1, None
            elif ch == "?":
                self.i += 1
                lo, hi = 0, 1
            elif ch == "{":
                lo, hi = self.parse_counted()
            else:
                return atom
            greedy = True
            if self.peek() == "?":
                self.i += 1
                greedy = False
            atom = ("rep", atom, lo, hi, greedy)

    def parse_counted(self):
        start = self.i
        self.i += 1
        end = self.p.find("}", self.i)
        if end < 0:
            raise self.error("unterminated counted repetition")
        body = self.p[self.i : end]
        self.i = end + 1
        try:
            if "," in body:
                a, b = body.split(",", 1)
                lo = int(a)
                hi = int(b) if b.strip() else None
            else:
                lo = hi = int(body)
        except ValueError as exc:
            self.i = start
            raise self.error("bad counted repetition") from exc
        if hi is not None and hi < lo:
            raise self.error("counted repetition max below min")
        return lo, hi

    def parse_atom(self):
        ch = self.take()
        if ch == "(":
            if self.p.startswith("?:", self.i):
                self.i += 2
            elif self.peek() == "?":
                raise self.error("group flags")
            node = self.parse_alt()
            if self.take() != ")":
                raise self.error("expected ')'")
            return node
        if ch == "[":
            return ("bytes", self.parse_class())
        if ch == "\\":
            return self.literal(self.parse_escape())
        if ch in ".^$":
            raise self.error(f"'{ch}'")
        if ch in "*+?{)|]}":
            raise self.error(f"dangling '{ch}'")
        return self.literal(ord(ch))

    def parse_escape(self) -> int:
        ch = self.take()
        if ch == "x":
            if self.peek() == "{":
                end = self.p.find("}", self.i)
                if end < 0:
                    raise self.error("unterminated \\x{")
                cp = int(self.p[self.i + 1 : end], 16)
                self.i = end + 1
                return cp
            hexd = self.p[self.i : self.i + 2]
            self.i += 2
            return int(hexd, 16)
        if ch in _META or ch in "-/ ":
            return ord(ch)
        if ch == "n":
            return 10
        if ch == "t":
            return 9
        raise self.error(f"escape \\{ch}")

    def parse_class(self) -> set[int]:
        if self.peek() == "^":
            raise self.error("negated class")
        out: set[int] = set()
        first = True
        while True:
            ch = self.take()
            if ch == "]" and not first:
                return out
            first = False
            lo = self.parse_escape() if ch == "\\" else ord(ch)
            if self.peek() == "-" and self.p[self.i + 1 : self.i + 2] not in ("]", ""):
                self.i += 1
                ch2 = self.take()
                hi = self.parse_escape() if ch2 == "\\" else ord(ch2)
                if hi < lo:
                    raise self.error("reversed class range")
            else:
                hi = lo
            if hi > 0x7F:
                raise self.error("non-ASCII class")
            out.update(range(lo, hi + 1))

    @staticmethod
    def literal(cp: int):
        data = chr(cp).encode("utf-8")
        if len(data) == 1:
            return ("bytes", {data[0]})
        return ("cat", [("bytes", {b}) for b in data])


# ---------------------------------------------------------------------------
# Thompson NFA with prioritised unions
# ---------------------------------------------------------------------------
class _NFA:
    def __init__(self) -> None:
        # kinds: "byte" (set, next) | "union" ([alts]) | "eps" (next) | "match"
        self.kind: list[str] = []
        self.data: list = []

    def add(self, kind: str, data) -> int:
        self.kind.append(kind)
        self.data.append(data)
        return len(self.kind) - 1

    def patch(self, sid: int, data) -> None:
        self.data[sid] = data


def _compile(nfa: _NFA, node, out: int) -> int:
    """Compile ``node`` so that it continues to ``out``; return its entry state."""
    tag = node[0]
    if tag == "empty":
        return out
    if tag == "bytes":
        return nfa.add("byte", (frozenset(node[1]), out))
    if tag == "cat":
        nxt = out
        for child in reversed(node[1]):
            nxt = _compile(nfa, child, nxt)
        return nxt
    if tag == "alt":
        entries = [_compile(nfa, child, out) for child in node[1]]
        return nfa.add("union", entries)
    if tag == "rep":
        _, child, lo, hi, greedy = node
        if hi is None:
            # star part: U -> [child -> U, out] (greedy) or [out, child -> U] (lazy)
            loop = nfa.add("union", [])
            body = _compile(nfa, child, loop)
            nfa.patch(loop, [body, out] if greedy else [out, body])
            nxt = loop
        else:
            # (hi - lo) nested optionals: child (child (...)?)?
            nxt = out
            for _ in range(hi - lo):
                body = _compile(nfa, child, nxt)
                nxt = nfa.add("union", [body, out] if greedy else [out, body])
        for _ in range(lo):
            nxt = _compile(nfa, child, nxt)
        return nxt
    raise AssertionError(tag)


def _closure(nfa: _NFA, start: int, into: list[int], seen: set[int]) -> None:
    stack = [start]
    while stack:
        sid = stack.pop()
        while sid not in seen:
            seen.add(sid)
            into.append(sid)
            kind = nfa.kind[sid]
            if kind == "union":
                alts = nfa.data[sid]
                if not alts:
                    break
                stack.extend(reversed(alts[1:]))
                sid = alts[0]
            elif kind == "eps":
                sid = nfa.data[sid]
            else:
                break


# ---------------------------------------------------------------------------
# determinisation
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class ByteDFA:
    """Dense DFA: ``trans[s, byte]``, ``dead`` id, ``start`` id, ``eoi_match[s]``."""

    pattern: str
    trans: np.ndarray  # int32 [n_states, 256]
    dead: int
    start: int
    eoi_match: np.ndarray  # bool [n_states]

    @property
    def n_states(self) -> int:
        return int(self.trans.shape[0])

    def walk(self, state: int, token: bytes) -> int:
        for b in token:
            state = int(self.trans[state, b])
        return state

    def is_dead_state(self, state: int) -> bool:
        return state == self.dead

    def is_match_state(self, state: int) -> bool:
        return state != self.dead and bool(self.eoi_match[state])

    def valid_token_ids(self, state: int, vocabulary) -> tuple[int, ...]:
        return tuple(
            tid
            for tid, tok in enumerate(vocabulary)
            if tok and self.walk(state, tok) != self.dead
        )


def compile_regex_dfa(pattern: str, *, max_states: int = 100_000) -> ByteDFA:
    if not pattern:
        raise ValueError("regex pattern cannot be empty")
    ast = _Parser(pattern).parse()
    nfa = _NFA()
    match = nfa.add("match", None)
    entry = _compile(nfa, ast, match)

    def key_of(ids: list[int], is_match: bool):
        return (is_match, tuple(ids))

    dead_key = key_of([], False)
    index: dict = {dead_key: 0}
    states: list = [dead_key]
    start_ids: list[int] = []
    _closure(nfa, entry, start_ids, set())
    start_key = key_of(start_ids, False)
    if start_key not in index:
        index[start_key] = len(states)
        states.append(start_key)

    def step(ids: tuple[int, ...], byte: int | None):
        nxt: list[int] = []
        seen: set[int] = set()
        is_match = False
        for sid in ids:
            kind = nfa.kind[sid]
            if kind == "match":
                is_match = True
                break  # leftmost-first: drop lower-priority threads
            if kind == "byte" and byte is not None:
                accept, target = nfa.data[sid]
                if byte in accept:
                    _closure(nfa, target, nxt, seen)
        return key_of(nxt, is_match)

    rows: list[list[int]] = []
    eoi: list[bool] = []
    i = 0
    while i < len(states):
        _, ids = states[i]
        row = []
        for byte in range(256):
            k = step(ids, byte)
            if k not in index:
                if len(states) >= max_states:
                    raise ValueError("regex DFA exceeds the state limit")
                index[k] = len(states)
                states.append(k)
            row.append(index[k])
        rows.append(row)
        eoi.append(step(ids, None)[0])
        i += 1

    return ByteDFA(
        pattern=pattern,
        trans=np.asarray(rows, dtype=np.int32),
        dead=0,
        start=index[start_key],
        eoi_match=np.asarray(eoi, dtype=bool),
    )
