"""GPU parity of the mask producer (onyx_dfa_state_masks) against the oracle's restatement of
get_valid_token_ids (oracle_cpu.c oracle_dfa_scan / oracle_dfa_table; the DFA compiler in
oracle/regex_dfa.py is pinned by the reference's regex fixtures). Bit-exact."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from onyx_b200 import dfa_masks, masked_selection as ms, workloads
from oracle.regex_dfa import compile_regex_dfa
from tests.conftest import load_golden
from tests.gpu_util import host, masks_to_device, requires_cuda, to_device

pytestmark = [pytest.mark.gpu, requires_cuda]

REGEX = load_golden("regex_parity.json")["cases"]


def _edge_tokens(rng) -> list[bytes]:
    return [b"", b"0" * 40, bytes(range(0x80, 0x90)), b"12345678", b"123456789", b"7a",
            bytes([0x30, 0xFF, 0x31]), bytes(rng.integers(0x20, 0x7F, 19, dtype=np.uint8))]


@pytest.mark.parametrize("case", REGEX, ids=[c["name"] for c in REGEX])
def test_fixture_patterns_every_state(case, cuda_lib):
    dfa = compile_regex_dfa(case["pattern"])
    vocab = [bytes.fromhex(h) for h in case["vocabulary_hex"]]
    want = oracle.dfa_table(dfa, vocab)
    got = dfa_masks.DfaMaskBuilder(dfa.trans, dfa.dead, vocab).table()
    np.testing.assert_array_equal(host(got).view(np.uint32), want)


@pytest.mark.parametrize("pattern", ["[0-9]{1,8}", "-?(0|[1-9][0-9]*)(\\.[0-9]+)?([eE][-+]?[0-9]+)?",
                                     "(true|false|null)", "\"[a-z_]{0,12}\""])
def test_large_vocabulary_every_state(pattern, cuda_lib):
    rng = np.random.default_rng(len(pattern))
    vocab = workloads.synthetic_vocabulary(rng, 128256 - 8) + _edge_tokens(rng)
    dfa = compile_regex_dfa(pattern)
    want = oracle.dfa_table(dfa, vocab)
    builder = dfa_masks.DfaMaskBuilder(dfa.trans, dfa.dead, vocab)
    assert builder.absorbing
    got = host(builder.table()).view(np.uint32)
    np.testing.assert_array_equal(got, want)
    # one state at a time, in any order, with repeats
    states = [dfa.start, dfa.dead, dfa.start, dfa.n_states - 1]
    got_rows = host(builder.masks(states)).view(np.uint32)
    np.testing.assert_array_equal(got_rows, want[states])


def test_single_row_grammar_workload_mask(cuda_lib):
    """The single-row workload's mask ([0-9]{1,8} at the start state over a 32,000-token
    synthetic vocabulary) built on the GPU."""
    w = workloads.single_row()
    dfa = compile_regex_dfa("[0-9]{1,8}")
    want = oracle.dfa_scan_bitmask(dfa, dfa.start, w["vocabulary"])
    got = dfa_masks.DfaMaskBuilder(dfa.trans, dfa.dead, w["vocabulary"]).masks([dfa.start])
    np.testing.assert_array_equal(host(got)[0].view(np.uint32), want)


def test_dead_state_not_absorbing_uses_the_final_state(cuda_lib):
    """A table whose dead state has ways out: a walk may pass through dead and leave it, so
    only the final state decides (no early stop)."""
    rng = np.random.default_rng(8)
    S = 37
    trans = rng.integers(0, S, size=(S, 256), dtype=np.int32)
    dead = 5
    trans[:, rng.integers(0, 256, 40)] = dead
    vocab = workloads.synthetic_vocabulary(rng, 5000) + _edge_tokens(rng)

    class _Dfa:  # the oracle's scan only reads these fields
        pass

    dfa = _Dfa()
    dfa.trans, dfa.dead = trans, dead
    want = oracle.dfa_table(dfa, vocab)
    builder = dfa_masks.DfaMaskBuilder(trans, dead, vocab)
    assert not builder.absorbing
    np.testing.assert_array_equal(host(builder.table()).view(np.uint32), want)


def test_malformed_input_stays_in_bounds(cuda_lib):
    """Out-of-range transitions count as dead and out-of-range state ids give empty rows."""
    rng = np.random.default_rng(9)
    S = 6
    trans = rng.integers(0, S, size=(S, 256), dtype=np.int32)
    trans[0, :] = 0
    dead = 0
    trans[2, 0x61] = 1000  # 'a' from state 2 leaves the table
    trans[3, 0x62] = -4  # 'b' from state 3 too
    vocab = [b"a", b"b", b"ab", b"ba", b"", b"cc", b"a" * 20]
    builder = dfa_masks.DfaMaskBuilder(trans, dead, vocab)
    got = host(builder.masks([2, 3, -1, S, 4])).view(np.uint32)

    def walk(state, tok):  # restated on the host, out-of-range transitions as dead
        for b in tok:
            nxt = int(trans[state, b])
            state = nxt if 0 <= nxt < S else dead
        return state

    for row, state in enumerate([2, 3, -1, S, 4]):
        want = 0
        for t, tok in enumerate(vocab):
            if 0 <= state < S and tok and walk(state, tok) != dead:
                want |= 1 << t
        assert int(got[row, 0]) == want, (row, state)


def test_built_table_feeds_the_gather(cuda_lib):
    """DFA table on the GPU -> gather masked argmax == the oracle on the oracle's table."""
    rng = np.random.default_rng(10)
    vocab = workloads.synthetic_vocabulary(rng, 32000)
    dfa = compile_regex_dfa("-?(0|[1-9][0-9]*)(\\.[0-9]+)?")
    table = dfa_masks.DfaMaskBuilder(dfa.trans, dfa.dead, vocab).table()
    ids = rng.integers(0, dfa.n_states, 48).astype(np.int32)
    x = workloads.normal_bf16(rng, (48, 32000))
    idx_ref, st_ref = oracle.gather_masked_argmax(x, oracle.dfa_table(dfa, vocab), ids,
                                                  dtype="bf16")
    r = ms.gather_masked_argmax(to_device(x, "bf16"), table, torch.from_numpy(ids).cuda())
    np.testing.assert_array_equal(host(r.token_ids), idx_ref)
    np.testing.assert_array_equal(host(r.status).astype(np.uint32), st_ref)
