"""Generate the golden fixtures in this folder from the reference's own Python code.

Run once where a checkout of the reference (read-only) is available, passing its root
directory; the outputs are committed and the tests only read the JSON files.

* ``regex_parity.json`` -- the reference's frozen regex outcomes
  (onyx_cuda/tests/regex_parity_fixtures.py:22-104, imported as data) plus the vectors
  of the native crate's unit tests (onyx_cuda/rust/src/regex_runtime.rs:271-452),
  transcribed below with their line numbers because Rust tests cannot be imported.
* ``selection_cases.json`` -- masked greedy selection outcomes computed by the
  reference's CPU selector ``select_highest_logit`` (onyx_cuda/src/onyx_cuda/
  generation.py:212-224) over rows masked the way the reference's list masks do
  (onyx_cuda/tests/test_grammar_selection.py:791-798), including the edge rows of the
  CUDA mask tests (onyx_cuda/tests/test_torch_grammar_mask.py:650-809).
* ``sampling_cases.json`` -- the kept ids and probabilities of temperature / top-p
  sampling computed by the reference's ``_filtered_reference_weights``
  (onyx_cuda/src/onyx_cuda/selection.py, the distribution behind
  ``create_reference_sampler``) over masked rows (invalid ids -inf, as mask.apply leaves
  them); an empty valid set or an all -inf support is the mask's rejection
  (torch_grammar_mask.py:182-185), NaN the sampler's.
* ``verify_cases.json`` -- grammar-aware speculative verification outcomes computed by
  ``decide_grammar_masked_target_acceptance`` (grammar_acceptance.py:166) and
  ``decide_grammar_masked_post_acceptance_continuation`` (grammar_continuation.py:102)
  driving a scripted ``FakeGrammarConstraint`` (testing.py:715) whose per-position
  valid sets are the case's bitmasks.
* ``iteration_cases.json`` -- the same pair of reference functions driving a branching
  scripted grammar (tokens lead to different states, some states admit nothing, some
  match), recording both result objects in full: accepted count, replacement, the
  no-decision selections, the committed states (by name) and match facts, the output
  tokens, and how many grammar states are still alive afterwards.

Usage:  python tests/golden/make_golden.py <reference checkout root>
"""

from __future__ import annotations

import json
import math
import struct
import sys
from pathlib import Path

import numpy as np

if len(sys.argv) != 2 or not (Path(sys.argv[1]) / "onyx_cuda" / "src").is_dir():
    raise SystemExit("usage: python tests/golden/make_golden.py <reference checkout root>")
REFERENCE = Path(sys.argv[1])
sys.path.insert(0, str(REFERENCE / "onyx_cuda" / "src"))
sys.path.insert(0, str(REFERENCE / "onyx_cuda" / "tests"))

from onyx_cuda.generation import select_highest_logit  # noqa: E402
from onyx_cuda.grammar_acceptance import decide_grammar_masked_target_acceptance  # noqa: E402
from onyx_cuda.grammar_continuation import (  # noqa: E402
    decide_grammar_masked_post_acceptance_continuation,
)
from onyx_cuda.testing import FakeGrammarConstraint, FakeGrammarProgram  # noqa: E402
from regex_parity_fixtures import REGEX_PARITY_CASES  # noqa: E402
from onyx_cuda.selection import (  # noqa: E402
    SamplingDistributionError,
    TemperatureTopPSelection,
    _filtered_reference_weights,
)

OUT = Path(__file__).resolve().parent

# ---------------------------------------------------------------------------
# regex
# ---------------------------------------------------------------------------
# Vectors of the native crate's unit tests (onyx_cuda/rust/src/regex_runtime.rs).
# Each state is (token path from init, valid ids, is_match, is_dead).
RUST_UNIT_CASES = [
    {
        "name": "rust_branches_and_dead_propagation",  # regex_runtime.rs:413-444
        "vocabulary": [b"a", b"b", b"c", b"ab", b"ac", b"x"],
        "pattern": "(?:ab|ac)",
        "states": [
            ([], [0, 3, 4], False, False),
            ([0], [1, 2], False, False),
            ([5], [], False, True),
            ([5, 0], [], False, True),
        ],
        "match_only": [([0, 1], True), ([0, 2], True)],
    },
    {
        "name": "rust_literal_empty_token_reuse",  # regex_runtime.rs:271-313
        "vocabulary": [b"a", b"b", b"ab", b"x", b"", b"abc", b"c"],
        "pattern": "ab",
        "states": [
            ([4], [0, 2, 5], False, False),
            ([5], [], False, False),
            ([0], [1], False, False),
        ],
        "match_only": [],
    },
]


def _hexbytes(items) -> list[str]:
    return [bytes(b).hex() for b in items]


def regex_fixtures() -> dict:
    cases = []
    for case in REGEX_PARITY_CASES:
        cases.append(
            {
                "name": case.name,
                "source": "onyx_cuda/tests/regex_parity_fixtures.py",
                "pattern": case.pattern,
                "vocabulary_hex": _hexbytes(case.vocabulary),
                "states": [
                    {
                        "token_ids": list(s.token_ids),
                        "valid_token_ids": list(s.valid_token_ids),
                        "is_match": s.is_match,
                        "is_dead": s.is_dead,
                    }
                    for s in case.states
                ],
                "match_only": [],
            }
        )
    for case in RUST_UNIT_CASES:
        cases.append(
            {
                "name": case["name"],
                "source": "onyx_cuda/rust/src/regex_runtime.rs",
                "pattern": case["pattern"],
                "vocabulary_hex": _hexbytes(case["vocabulary"]),
                "states": [
                    {"token_ids": p, "valid_token_ids": v, "is_match": m, "is_dead": d}
                    for p, v, m, d in case["states"]
                ],
                "match_only": [{"token_ids": p, "is_match": m} for p, m in case["match_only"]],
            }
        )
    return {"cases": cases}


# ---------------------------------------------------------------------------
# value encoding: rows are stored as raw bit patterns of their dtype
# ---------------------------------------------------------------------------
def _bf16_bits(x: np.ndarray) -> np.ndarray:
    u = x.astype(np.float32).view(np.uint32)
    rounded = u + 0x7FFF + ((u >> 16) & 1)  # round to nearest even
    bits = (rounded >> 16).astype(np.uint16)
    nan = np.isnan(x)
    bits[nan] = 0x7FC0
    return bits


def _bits_to_floats(bits: list[int], dtype: str) -> list[float]:
    if dtype == "bf16":
        return [struct.unpack("<f", struct.pack("<I", b << 16))[0] for b in bits]
    if dtype == "f16":
        return [float(np.uint16(b).view(np.float16)) for b in bits]
    if dtype == "f32":
        return [struct.unpack("<f", struct.pack("<I", b))[0] for b in bits]
    if dtype == "f64":
        return [struct.unpack("<d", struct.pack("<Q", b))[0] for b in bits]
    raise ValueError(dtype)


def _float_bits(values, dtype: str) -> list[int]:
    arr = np.asarray(values, dtype=np.float64)
    if dtype == "bf16":
        return [int(b) for b in _bf16_bits(arr.astype(np.float32))]
    if dtype == "f16":
        return [int(b) for b in arr.astype(np.float16).view(np.uint16)]
    if dtype == "f32":
        return [int(b) for b in arr.astype(np.float32).view(np.uint32)]
    if dtype == "f64":
        return [int(b) for b in arr.view(np.uint64)]
    raise ValueError(dtype)


def _mask_words(valid: list[int], vocab_size: int) -> list[int]:
    words = [0] * ((vocab_size + 31) // 32)
    for t in valid:
        words[t >> 5] |= 1 << (t & 31)
    return words


def _list_mask(row: list[float], valid: set[int]) -> tuple[float, ...]:
    return tuple(v if i in valid else -math.inf for i, v in enumerate(row))


def _reference_select(row_values: list[float], valid: list[int]):
    """Reference CPU outcome; maps the CUDA boundary's rejections onto status names."""
    if not valid:
        return None, "empty"
    masked = _list_mask(row_values, set(valid))
    if any(math.isnan(v) for v in masked):
        try:
            select_highest_logit(masked)
        except ValueError:
            return None, "nan"
        raise AssertionError("reference selector accepted NaN")
    # TorchCUDAGrammarLogitMask rejects an all -inf support before selection
    # (onyx_cuda/src/onyx_cuda/torch_grammar_mask.py:172-185).
    if all(masked[i] == -math.inf for i in valid):
        return select_highest_logit(masked), "all_neg_inf"
    return select_highest_logit(masked), "ok"


# ---------------------------------------------------------------------------
# selection cases
# ---------------------------------------------------------------------------
def selection_fixtures(rng: np.random.Generator) -> dict:
    cases = []

    def add(name, dtype, values, valid):
        bits = _float_bits(values, dtype)
        floats = _bits_to_floats(bits, dtype)
        idx, status = _reference_select(floats, list(valid))
        cases.append(
            {
                "name": name,
                "dtype": dtype,
                "vocab_size": len(bits),
                "bits": bits,
                "mask_words": _mask_words(list(valid), len(bits)),
                "expected_index": idx,
                "expected_status": status,
            }
        )

    inf, nan = math.inf, math.nan
    for dt in ("f32", "bf16", "f16", "f64"):
        # first-max tie-break (test_torch_grammar_mask.py:758-772)
        add(f"tie_lowest_index_{dt}", dt, [99.0, 7.0, 8.0, 8.0, 8.0, 100.0], [1, 3, 4])
        # +inf ties resolve to the lowest index (:775-794)
        add(f"pos_inf_tie_{dt}", dt, [inf, 4.0, inf, -3.0], [0, 2])
        add(f"single_pos_inf_{dt}", dt, [inf, 4.0, inf, -3.0], [2])
        # disallowed NaN removed, allowed NaN rejected (:797-809)
        add(f"disallowed_nan_{dt}", dt, [nan, 2.0, 1.0], [1, 2])
        add(f"allowed_nan_{dt}", dt, [nan, 2.0, 1.0], [0, 1])
        # signed zeros compare equal: the lowest index wins
        add(f"neg_zero_first_{dt}", dt, [-0.0, 0.0, -1.0], [0, 1, 2])
        add(f"pos_zero_first_{dt}", dt, [0.0, -0.0, -1.0], [0, 1, 2])
        # all -inf support rejected for partial and complete support (:748-755)
        add(f"all_neg_inf_partial_{dt}", dt, [-inf, -inf, -inf], [1])
        add(f"all_neg_inf_complete_{dt}", dt, [-inf, -inf, -inf], [0, 1, 2])
        add(f"neg_inf_and_finite_{dt}", dt, [-inf, -5.0, -inf], [0, 1, 2])
        # empty support: grammar no-decision (grammar_selection.py:122-127)
        add(f"empty_support_{dt}", dt, [1.0, 2.0, 3.0], [])
        # edge values of the bitwise mask test (:650-672)
        add(
            f"edge_values_{dt}",
            dt,
            [-0.0, 0.0, 5.0, inf, nan, -7.0, -inf, 99.0],
            [0, 1, 3, 6],
        )
    # finite extremes (:692-713)
    add("finite_extremes_f32", "f32", [-3.4028234663852886e38, 3.4028234663852886e38, -1.0, 1.0], [0, 1, 2, 3])
    add("finite_extremes_bf16", "bf16", [-3.3895313892515355e38, 3.3895313892515355e38, -1.0, 1.0], [0, 2, 3])
    add("finite_extremes_f16", "f16", [-65504.0, 65504.0, -1.0, 1.0], [0, 1, 3])
    # word-boundary bits: single bits at word 0, last word, bit 31
    for v in (1, 31, 32, 33, 63, 64, 65, 97):
        for pos in sorted({0, v - 1, min(31, v - 1), v // 2}):
            vals = rng.normal(0.0, 3.0, size=v)
            add(f"single_bit_v{v}_at{pos}", "bf16", vals, [pos])
    # random rows of several densities and dtypes, with forced ties
    for k in range(48):
        dt = ("bf16", "f32", "f16", "f64")[k % 4]
        v = int(rng.integers(1, 300))
        vals = rng.normal(0.0, 3.0, size=v)
        if k % 3 == 0 and v > 4:
            top = float(np.max(vals)) + 1.0
            for j in rng.choice(v, size=3, replace=False):
                vals[j] = top
        density = float(rng.uniform(0.005, 0.6))
        valid = [i for i in range(v) if rng.random() < density]
        if not valid and k % 5 != 0:
            valid = [int(rng.integers(0, v))]
        add(f"random_{k}_{dt}_v{v}", dt, vals, valid)
    return {"cases": cases}


# ---------------------------------------------------------------------------
# speculative verify cases through the reference's grammar acceptance
# ---------------------------------------------------------------------------
class _ListMask:
    def __init__(self, vocab_size: int) -> None:
        self.vocab_size = vocab_size

    def apply(self, logits, valid_token_ids, /):
        return _list_mask(list(logits), set(valid_token_ids))


def _chain_constraint(vocab_size: int, per_position_valid: list[list[int]]):
    """Scripted grammar: state s_i admits per_position_valid[i]; every valid token
    moves to s_{i+1}; the state after the last position is a match state."""
    n = len(per_position_valid)
    transitions = []
    valid = []
    match_states = {f"s{n}"}
    for i, ids in enumerate(per_position_valid):
        valid.append((f"s{i}", tuple(ids)))
        for t in ids:
            transitions.append((f"s{i}", t, f"s{i + 1}"))
        if not ids:
            match_states.add(f"s{i}")
    program = FakeGrammarProgram(
        initial_state="s0",
        transitions=tuple(transitions),
        valid_token_ids=tuple(valid),
        match_states=frozenset(match_states),
    )
    vocabulary = tuple(f"t{i}".encode() for i in range(vocab_size))
    return FakeGrammarConstraint(vocabulary, grammar_type="regex", program=program)


def _reference_verify(rows: list[list[float]], valid: list[list[int]], drafts: list[int]):
    vocab_size = len(rows[0])
    for i, r in enumerate(rows):
        masked = _list_mask(r, set(valid[i]))
        # rows the reference would reach with a NaN or all -inf support raise; the
        # fixture only records cases whose decision path avoids them
    constraint = _chain_constraint(vocab_size, valid)
    state = constraint.init_state()
    mask = _ListMask(vocab_size)
    acceptance = decide_grammar_masked_target_acceptance(
        tuple(drafts),
        tuple(tuple(r) for r in rows),
        constraint,
        state,
        mask,
        vocab_size=vocab_size,
        select_token=select_highest_logit,
    )
    accepted = acceptance.accepted_count
    if acceptance.replacement_token_id is not None:
        return accepted, acceptance.replacement_token_id, "ok"
    if not acceptance.decision_made:
        return accepted, None, "empty"
    if acceptance.committed_state is None:
        return accepted, None, "empty"
    cont = decide_grammar_masked_post_acceptance_continuation(
        tuple(drafts),
        tuple(tuple(r) for r in rows),
        acceptance,
        constraint,
        mask,
        vocab_size=vocab_size,
        select_token=select_highest_logit,
    )
    if cont.final_row_no_decision_selection is not None:
        return accepted, None, "empty"
    return accepted, cont.uncached_next_token_id, "ok"


def verify_fixtures(rng: np.random.Generator) -> dict:
    cases = []
    for k in range(72):
        gamma = int(rng.integers(1, 6))
        v = int(rng.integers(8, 200))
        dt = ("bf16", "f32", "f16")[k % 3]
        rows_bits, rows_f, valid = [], [], []
        for i in range(gamma + 1):
            vals = rng.normal(0.0, 3.0, size=v)
            bits = _float_bits(vals, dt)
            rows_bits.append(bits)
            rows_f.append(_bits_to_floats(bits, dt))
            density = float(rng.uniform(0.02, 0.5))
            ids = [j for j in range(v) if rng.random() < density] or [int(rng.integers(0, v))]
            valid.append(ids)
        # sprinkle empty supports (no-decision) into some cases
        if k % 9 == 4:
            valid[int(rng.integers(0, gamma + 1))] = []
        drafts = []
        for i in range(gamma):
            if valid[i]:
                masked = _list_mask(rows_f[i], set(valid[i]))
                best = select_highest_logit(masked)
                if rng.random() < 0.7:
                    drafts.append(best)
                else:
                    others = [j for j in valid[i] if j != best] or [(best + 1) % v]
                    drafts.append(int(rng.choice(others)))
            else:
                drafts.append(int(rng.integers(0, v)))
        accepted, correction, status = _reference_verify(rows_f, valid, drafts)
        cases.append(
            {
                "name": f"verify_{k}_{dt}_g{gamma}_v{v}",
                "dtype": dt,
                "vocab_size": v,
                "gamma": gamma,
                "bits": rows_bits,
                "mask_words": [_mask_words(ids, v) for ids in valid],
                "drafts": drafts,
                "expected_accept_len": accepted,
                "expected_correction": correction,
                "expected_status": status,
            }
        )
    return {"cases": cases}


# ---------------------------------------------------------------------------
# whole speculative iterations (acceptance + continuation) on a branching grammar
# ---------------------------------------------------------------------------
def _branching_constraint(rng: np.random.Generator, vocab_size: int, n_states: int):
    """Scripted grammar of n_states states: each admits a random set of ids (some none),
    each admitted id leads to a random state, some states match."""
    names = [f"q{i}" for i in range(n_states)]
    valid, transitions = [], []
    for name in names:
        if rng.random() < 0.12:
            ids = []
        else:
            density = float(rng.uniform(0.05, 0.6))
            ids = [j for j in range(vocab_size) if rng.random() < density] or [int(rng.integers(0, vocab_size))]
        valid.append((name, tuple(ids)))
        for t in ids:
            transitions.append((name, t, names[int(rng.integers(0, n_states))]))
    # a state that admits nothing must be a match state (the fake's own rule)
    match_states = frozenset(n for (n, ids) in valid if not ids or rng.random() < 0.3)
    program = FakeGrammarProgram(initial_state="q0", transitions=tuple(transitions),
                                 valid_token_ids=tuple(valid), match_states=match_states)
    vocabulary = tuple(f"t{i}".encode() for i in range(vocab_size))
    return FakeGrammarConstraint(vocabulary, grammar_type="regex", program=program), program


def _state_name(constraint, handle):
    return None if handle is None else constraint._states[handle.value]


def iteration_fixtures(rng: np.random.Generator) -> dict:
    cases = []
    for k in range(60):
        gamma = int(rng.integers(1, 6))
        v = int(rng.integers(8, 96))
        n_states = int(rng.integers(3, 9))
        constraint, program = _branching_constraint(rng, v, n_states)
        valid_of = dict(program.valid_token_ids)
        step_of = {(s, t): d for s, t, d in program.transitions}
        start = constraint.init_state()
        # rows of exactly representable f32 values; drafts follow the masked argmax along
        # the grammar 70% of the time, so proposals are often accepted in full
        rows = [[float(np.float32(x)) for x in rng.normal(0.0, 3.0, size=v)] for _ in range(gamma + 1)]
        drafts, state = [], "q0"
        for i in range(gamma):
            ids = valid_of.get(state, ())
            if ids and rng.random() < 0.75:
                best = select_highest_logit(_list_mask(rows[i], set(ids)))
                t = best if rng.random() < 0.8 else int(rng.choice(ids))
            else:
                t = int(rng.integers(0, v))
            drafts.append(t)
            state = step_of.get((state, t), state)
        mask = _ListMask(v)
        acceptance = decide_grammar_masked_target_acceptance(
            tuple(drafts), tuple(tuple(r) for r in rows), constraint, start, mask,
            vocab_size=v, select_token=select_highest_logit)
        nd = acceptance.no_decision_selection
        case = {
            "name": f"iteration_{k}_g{gamma}_v{v}_s{n_states}",
            "vocab_size": v,
            "gamma": gamma,
            "states": [[name, list(ids)] for name, ids in program.valid_token_ids],
            "transitions": [[s, t, d] for s, t, d in program.transitions],
            "match_states": sorted(program.match_states),
            "rows_f32": rows,
            "drafts": drafts,
            "accepted_count": acceptance.accepted_count,
            "replacement_token_id": acceptance.replacement_token_id,
            "no_decision_is_match": None if nd is None else nd.is_match,
            "acceptance_state": _state_name(constraint, acceptance.committed_state),
            "acceptance_is_match": acceptance.committed_state_is_match,
            "continuation": None,
        }
        if acceptance.decision_made:
            state_name = _state_name(constraint, acceptance.committed_state)
            cont = decide_grammar_masked_post_acceptance_continuation(
                tuple(drafts), tuple(tuple(r) for r in rows), acceptance, constraint, mask,
                vocab_size=v, select_token=select_highest_logit)
            fr = cont.final_row_no_decision_selection
            case["acceptance_state"] = state_name
            case["continuation"] = {
                "output_token_ids": list(cont.output_token_ids),
                "uncached_next_token_id": cont.uncached_next_token_id,
                "final_row_no_decision_is_match": None if fr is None else fr.is_match,
                "committed_state": _state_name(constraint, cont.committed_state),
                "committed_is_match": cont.committed_state_is_match,
            }
        case["active_states_after"] = constraint.active_state_count
        cases.append(case)
    return {"cases": cases}


def _reference_kept(row_values: list[float], valid: list[int], temperature: float,
                    top_p: float):
    if not valid:
        return "empty_mask", []
    masked = _list_mask(row_values, set(valid))
    if all(masked[i] == -math.inf for i in valid):
        return "all_neg_inf", []
    policy = TemperatureTopPSelection(temperature=temperature, top_p=top_p, seed=0)
    try:
        kept = _filtered_reference_weights(masked, policy)
    except SamplingDistributionError:
        return "nan_in_support", []
    return "ok", [[int(t), float(p).hex()] for t, p in kept]


def sampling_fixtures(rng: np.random.Generator) -> dict:
    cases = []
    policies = [(1.0, 1.0), (0.8, 0.9), (0.5, 0.5), (2.0, 0.95), (1.3, 0.05), (0.7, 1.0)]
    for n in range(36):
        vocab = int(rng.integers(40, 400))
        dtype = "bf16" if n % 3 else "f32"
        row = (rng.standard_normal(vocab) * 3.0).astype(np.float32)
        valid = sorted(int(i) for i in np.flatnonzero(rng.random(vocab) < rng.uniform(0.05, 0.6)))
        kind = n % 9
        if kind == 1 and valid:  # exact ties among the leaders
            row[valid[: min(4, len(valid))]] = row.max() + 1.0
        elif kind == 2 and valid:  # +inf among the valid ids, and outside them
            row[valid[0]] = np.inf
            row[valid[-1]] = np.inf
            row[0] = np.inf
        elif kind == 3 and valid:  # NaN valid
            row[valid[len(valid) // 2]] = np.nan
        elif kind == 4:  # NaN outside the valid set only
            row[[i for i in range(vocab) if i not in set(valid)][:3]] = np.nan
        elif kind == 5 and valid:  # all valid -inf
            row[valid] = -np.inf
        elif kind == 6:
            valid = []
        elif kind == 7 and valid:  # one valid id
            valid = valid[:1]
        elif kind == 8 and valid:  # some valid -inf, flat values
            row[:] = 0.25
            row[valid[::2]] = -np.inf
        bits = _float_bits(row, dtype)
        values = _bits_to_floats(bits, dtype)
        temperature, top_p = policies[n % len(policies)]
        status, kept = _reference_kept(values, valid, temperature, top_p)
        cases.append({
            "name": f"sample_{n:02d}_kind{kind}", "dtype": dtype, "bits": bits,
            "mask_words": _mask_words(valid, vocab), "temperature": temperature,
            "top_p": top_p, "expected_status": status, "expected_kept": kept,
        })
    return {"source": "onyx_cuda/src/onyx_cuda/selection.py _filtered_reference_weights",
            "cases": cases}


def main() -> None:
    rng = np.random.default_rng(20260714)
    files = {
        "regex_parity.json": regex_fixtures(),
        "selection_cases.json": selection_fixtures(rng),
        "verify_cases.json": verify_fixtures(rng),
        "sampling_cases.json": sampling_fixtures(rng),
        "iteration_cases.json": iteration_fixtures(np.random.default_rng(20261202)),
    }
    for name, payload in files.items():
        payload["generator"] = "tests/golden/make_golden.py"
        (OUT / name).write_text(json.dumps(payload, separators=(",", ":")) + "\n")
        print(f"wrote {name}: {len(payload['cases'])} cases")


if __name__ == "__main__":
    main()
