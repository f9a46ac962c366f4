"""The oracle against every golden vector produced by the reference's own code.

tests/golden/make_golden.py produced the fixtures from the reference (select_highest_logit,
decide_grammar_masked_target_acceptance + post-acceptance continuation, the frozen regex
parity outcomes). Both oracle formulations (C and NumPy) must reproduce all of them before
any GPU result is compared with the oracle.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from oracle import numpy_ref
from oracle.regex_dfa import compile_regex_dfa
from tests.conftest import golden_values, load_golden

SELECTION = load_golden("selection_cases.json")["cases"]
VERIFY = load_golden("verify_cases.json")["cases"]
REGEX = load_golden("regex_parity.json")["cases"]


@pytest.mark.parametrize("case", SELECTION, ids=[c["name"] for c in SELECTION])
def test_c_oracle_selection_matches_reference(case, oracle_lib):
    x = golden_values(case["bits"], case["dtype"])[None]
    m = np.asarray(case["mask_words"], np.uint32)[None]
    idx, st = oracle.masked_argmax(x, m, dtype=case["dtype"])
    assert int(st[0]) == oracle.STATUS_BITS[case["expected_status"]]
    if case["expected_status"] == "ok":
        assert int(idx[0]) == case["expected_index"]


@pytest.mark.parametrize("case", SELECTION, ids=[c["name"] for c in SELECTION])
def test_numpy_oracle_selection_matches_reference(case):
    x = golden_values(case["bits"], case["dtype"])[None]
    m = np.asarray(case["mask_words"], np.uint32)[None]
    idx, st = numpy_ref.masked_argmax(x, m, case["dtype"])
    assert int(st[0]) == oracle.STATUS_BITS[case["expected_status"]]
    if case["expected_status"] == "ok":
        assert int(idx[0]) == case["expected_index"]


@pytest.mark.parametrize("case", VERIFY, ids=[c["name"] for c in VERIFY])
def test_c_oracle_verify_matches_reference(case, oracle_lib):
    x = golden_values(case["bits"], case["dtype"])[None]
    m = np.asarray(case["mask_words"], np.uint32)[None]
    d = np.asarray(case["drafts"], np.int32)[None]
    acc, corr, st = oracle.spec_verify(x, m, d, dtype=case["dtype"])
    assert int(acc[0]) == case["expected_accept_len"]
    expected_corr = -1 if case["expected_correction"] is None else case["expected_correction"]
    assert int(corr[0]) == expected_corr
    assert int(st[0]) == oracle.STATUS_BITS[case["expected_status"]]


def _vocab(case):
    return [bytes.fromhex(h) for h in case["vocabulary_hex"]]


@pytest.mark.parametrize("case", REGEX, ids=[c["name"] for c in REGEX])
def test_regex_dfa_matches_reference_outcomes(case):
    dfa = compile_regex_dfa(case["pattern"])
    vocab = _vocab(case)
    for st in case["states"]:
        s = dfa.start
        for t in st["token_ids"]:
            s = dfa.walk(s, vocab[t])
        assert list(dfa.valid_token_ids(s, vocab)) == st["valid_token_ids"], st
        assert dfa.is_match_state(s) == st["is_match"], st
        assert dfa.is_dead_state(s) == st["is_dead"], st
    for st in case["match_only"]:
        s = dfa.start
        for t in st["token_ids"]:
            s = dfa.walk(s, vocab[t])
        assert dfa.is_match_state(s) == st["is_match"]


@pytest.mark.parametrize("case", REGEX, ids=[c["name"] for c in REGEX])
def test_c_dfa_scan_matches_python_walk(case, oracle_lib):
    dfa = compile_regex_dfa(case["pattern"])
    vocab = _vocab(case)
    for s in range(dfa.n_states):
        words = oracle.dfa_scan_bitmask(dfa, s, vocab)
        bits = numpy_ref.unpack_mask(words, len(vocab))
        assert list(np.flatnonzero(bits)) == list(dfa.valid_token_ids(s, vocab))


def test_invalid_patterns_are_rejected():
    # onyx_cuda/tests/regex_parity_fixtures.py:104 lists "(" and "[z-a]" as invalid
    for pattern in ("(", "[z-a]", ""):
        with pytest.raises(ValueError):
            compile_regex_dfa(pattern)


def test_delayed_match_quirk_for_single_row_grammar():
    """[0-9]{1,8} at init admits d^j (1<=j<=8) and d^j followed by exactly one more byte."""
    dfa = compile_regex_dfa("[0-9]{1,8}")
    vocab = [b"5", b"12345678", b"123456789", b"5a", b"5ab", b"a", b"1234567890", b"", b"55 "]
    assert dfa.valid_token_ids(dfa.start, vocab) == (0, 1, 2, 3, 8)
    assert not dfa.is_match_state(dfa.start)
    assert dfa.is_match_state(dfa.walk(dfa.start, b"12"))


SAMPLING = load_golden("sampling_cases.json")["cases"]


def _float_row(case) -> np.ndarray:
    vals = golden_values(case["bits"], case["dtype"])
    if case["dtype"] == "bf16":
        return (vals.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return vals.astype(np.float64)


@pytest.mark.parametrize("case", SAMPLING, ids=[c["name"] for c in SAMPLING])
def test_sampling_oracle_matches_reference_filtering(case):
    """Kept ids and probabilities (bit for bit) of the reference's _filtered_reference_weights."""
    from oracle import sampling

    row = _float_row(case)
    valid = sampling.unpack_mask(np.asarray(case["mask_words"], np.uint32), row.size)
    status, kept = sampling.kept_weights(row, valid, case["temperature"], case["top_p"])
    names = {0: "ok", 1: "empty_mask", 2: "all_neg_inf", 4: "nan_in_support"}
    assert names[status] == case["expected_status"]
    assert [[t, p.hex()] for t, p in kept] == case["expected_kept"]


def test_philox_known_answers():
    """Philox4x32-10 against the published known-answer vectors of its authors' library."""
    from oracle.sampling import philox4x32_10

    assert philox4x32_10((0, 0, 0, 0), (0, 0)) == (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)
    assert philox4x32_10((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF)) == (
        0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)
    assert philox4x32_10((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344),
                         (0xA4093822, 0x299F31D0)) == (0xD16CFE09, 0x94FDCCEB, 0x5001E420,
                                                       0x24126EA1)
