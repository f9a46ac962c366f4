"""GPU parity: masked argmax / gather through the C ABI against the oracle and the golden
vectors produced by the reference's own selector. Bit-exact (integer outputs)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from onyx_b200 import _lib
from onyx_b200 import masked_selection as ms
from onyx_b200 import workloads
from oracle.regex_dfa import compile_regex_dfa
from tests.conftest import golden_values, load_golden
from tests.gpu_util import host, masks_to_device, requires_cuda, to_device

pytestmark = [pytest.mark.gpu, requires_cuda]

SELECTION = load_golden("selection_cases.json")["cases"]
STATUS = oracle.STATUS_BITS


def _check(idx_gpu, st_gpu, idx_ref, st_ref):
    idx_gpu, st_gpu = host(idx_gpu).astype(np.int64), host(st_gpu).astype(np.int64)
    np.testing.assert_array_equal(st_gpu, st_ref.astype(np.int64))
    np.testing.assert_array_equal(idx_gpu, idx_ref.astype(np.int64))


@pytest.mark.parametrize("case", SELECTION, ids=[c["name"] for c in SELECTION])
def test_golden_selection(case, cuda_lib):
    x = golden_values(case["bits"], case["dtype"])
    m = np.asarray(case["mask_words"], np.uint32)
    r = ms.masked_argmax(to_device(x[None], case["dtype"]), masks_to_device(m[None]))
    assert int(host(r.status)[0]) == STATUS[case["expected_status"]]
    if case["expected_status"] == "ok":
        assert int(host(r.token_ids)[0]) == case["expected_index"]


def _random_case(rng, rows, vocab, dtype, density):
    if dtype == "bf16":
        x = workloads.normal_bf16(rng, (rows, vocab))
    else:
        np_dt = {"f32": np.float32, "f16": np.float16, "f64": np.float64}[dtype]
        x = (rng.standard_normal((rows, vocab)) * 3.0).astype(np_dt)
    m = workloads.bernoulli_masks(rng, np.full(rows, density), vocab)
    return x, m


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32", "f64"])
@pytest.mark.parametrize("vocab", [1, 7, 31, 32, 33, 1000, 4097, 16385, 32000, 128256, 151665])
def test_random_rows_match_oracle(dtype, vocab, cuda_lib):
    rng = np.random.default_rng(vocab * 7 + len(dtype))
    rows = 5
    x, m = _random_case(rng, rows, vocab, dtype, 0.05)
    # forced ties: equal maxima in two segments of row 0
    if vocab > 40000:
        hi = x[0].max() if dtype != "bf16" else None
        if dtype == "bf16":
            x[0, [3, 20000, vocab - 1]] = workloads.bf16_bits(np.array([50.0] * 3, np.float32))
        else:
            x[0, [3, 20000, vocab - 1]] = hi + 50
        for j in (3, 20000, vocab - 1):
            m[0, j >> 5] |= np.uint32(1 << (j & 31))
    idx_ref, st_ref = oracle.masked_argmax(x, m, dtype=dtype)
    r = ms.masked_argmax(to_device(x, dtype), masks_to_device(m))
    _check(r.token_ids, r.status, idx_ref, st_ref)
    if vocab > 40000:
        assert int(host(r.token_ids)[0]) == 3


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_unaligned_rows_take_the_generic_path(dtype, cuda_lib):
    """Row stride 151665 (odd) and an offset base: rows are not 16-byte aligned."""
    rng = np.random.default_rng(5)
    rows, vocab = 3, 151665
    x, m = _random_case(rng, rows, vocab + 1, dtype, 0.03)
    t = to_device(x, dtype)[:, 1:]  # base shifted by one element, stride vocab+1
    m = m.copy()
    idx_ref, st_ref = oracle.masked_argmax(np.ascontiguousarray(x[:, 1:]),
                                           _shift_masks(m, vocab + 1), dtype=dtype)
    r = ms.masked_argmax(t, masks_to_device(_shift_masks(m, vocab + 1)))
    _check(r.token_ids, r.status, idx_ref, st_ref)


def _shift_masks(m, vocab_plus_one):
    """Masks for columns 1..V of a row (drop bit 0)."""
    from onyx_b200 import bitmask

    bits = bitmask.unpack(m, vocab_plus_one)[:, 1:]
    return bitmask.pack_bool(bits)


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_unmasked_argmax_matches_first_max(dtype, cuda_lib):
    rng = np.random.default_rng(3)
    x, _ = _random_case(rng, 4, 70000, dtype, 0.1)
    idx_ref, st_ref = oracle.masked_argmax(x, None, dtype=dtype)
    r = ms.masked_argmax(to_device(x, dtype), None)
    _check(r.token_ids, r.status, idx_ref, st_ref)


def test_edge_masks_empty_single_bits_and_all_ones(cuda_lib):
    rng = np.random.default_rng(9)
    vocab = 128256
    x = workloads.normal_bf16(rng, (6, vocab))
    m = np.zeros((6, vocab // 32), np.uint32)
    m[1, 0] = 1  # id 0
    m[2, -1] = np.uint32(1 << 31)  # last id
    m[3, 2000] = np.uint32(1 << 31)  # bit 31 mid-row
    m[4, :] = 0xFFFFFFFF
    m[5, 17] = np.uint32(0x80000001)
    idx_ref, st_ref = oracle.masked_argmax(x, m, dtype="bf16")
    r = ms.masked_argmax(to_device(x, "bf16"), masks_to_device(m))
    _check(r.token_ids, r.status, idx_ref, st_ref)
    assert int(host(r.status)[0]) == ms.STATUS_EMPTY_MASK
    assert int(host(r.token_ids)[2]) == vocab - 1


def test_special_values_across_segments(cuda_lib):
    """NaN in one segment, +inf ties across segments, all -inf rows, signed zeros."""
    vocab = 128256
    rows = 5
    x = np.zeros((rows, vocab), np.float32)
    x[:] = -1.0
    x[0, 50000] = np.nan
    x[0, 70000] = 5.0
    x[1, [1000, 90000]] = np.inf
    x[2, :] = -np.inf
    x[3, 5] = -0.0
    x[3, 6] = 0.0
    x[4, 100000] = 0.0
    x[4, 100001] = -0.0
    m = np.full((rows, vocab // 32), 0xFFFFFFFF, np.uint32)
    m[4, :] = 0
    m[4, 100000 >> 5] = np.uint32((1 << (100000 & 31)) | (1 << (100001 & 31)))
    for dt in ("f32", "bf16"):
        xv = x if dt == "f32" else workloads.bf16_bits(x)
        idx_ref, st_ref = oracle.masked_argmax(xv, m, dtype=dt)
        r = ms.masked_argmax(to_device(xv, dt), masks_to_device(m))
        _check(r.token_ids, r.status, idx_ref, st_ref)
        st = host(r.status)
        assert st[0] == ms.STATUS_NAN_IN_SUPPORT and st[2] == ms.STATUS_ALL_NEG_INF
        assert host(r.token_ids)[1] == 1000 and host(r.token_ids)[3] == 5
        assert host(r.token_ids)[4] == 100000


def test_single_row_grammar_workload(cuda_lib):
    """fp32 [1, 32000] under the [0-9]{1,8} grammar's initial-state mask."""
    w = workloads.single_row()
    dfa = compile_regex_dfa(w["pattern"])
    words = oracle.dfa_scan_bitmask(dfa, dfa.start, w["vocabulary"])
    assert words.shape == (1000,)
    idx_ref, st_ref = oracle.masked_argmax(w["logits"], words[None], dtype="f32")
    r = ms.masked_argmax(to_device(w["logits"], "f32"), masks_to_device(words[None]))
    _check(r.token_ids, r.status, idx_ref, st_ref)
    assert st_ref[0] == 0


def test_batched_workload_full_size(cuda_lib):
    w = workloads.batched()
    idx_ref, st_ref = oracle.masked_argmax(w["logits_bf16"], w["masks"], dtype="bf16")
    r = ms.masked_argmax(to_device(w["logits_bf16"], "bf16"), masks_to_device(w["masks"]))
    _check(r.token_ids, r.status, idx_ref, st_ref)
    # repeated calls reuse the self-resetting workspace and give identical results
    for _ in range(3):
        r2 = ms.masked_argmax(to_device(w["logits_bf16"], "bf16"), masks_to_device(w["masks"]))
        _check(r2.token_ids, r2.status, idx_ref, st_ref)


def test_table_gather_workload_full_size(cuda_lib):
    w = workloads.table_gather()
    idx_ref, st_ref = oracle.gather_masked_argmax(w["logits_bf16"], w["table"], w["state_ids"],
                                                  dtype="bf16")
    r = ms.gather_masked_argmax(to_device(w["logits_bf16"], "bf16"), masks_to_device(w["table"]),
                                torch.from_numpy(w["state_ids"]).cuda())
    _check(r.token_ids, r.status, idx_ref, st_ref)
    # gather == masked argmax with the rows gathered on the host
    r2 = ms.masked_argmax(to_device(w["logits_bf16"], "bf16"),
                          masks_to_device(w["table"][w["state_ids"]]))
    _check(r2.token_ids, r2.status, idx_ref, st_ref)


def test_gather_rejects_out_of_range_states(cuda_lib):
    rng = np.random.default_rng(2)
    x = workloads.normal_bf16(rng, (4, 5000))
    table = workloads.bernoulli_masks(rng, np.full(3, 0.1), 5000)
    ids = np.array([0, -1, 3, 2], np.int32)
    idx_ref, st_ref = oracle.gather_masked_argmax(x, table, ids, dtype="bf16")
    r = ms.gather_masked_argmax(to_device(x, "bf16"), masks_to_device(table),
                                torch.from_numpy(ids).cuda())
    _check(r.token_ids, r.status, idx_ref, st_ref)
    assert list(host(r.status)[1:3]) == [ms.STATUS_BAD_STATE] * 2


def test_results_are_independent_of_the_stream(cuda_lib):
    w = workloads.batched(rows=16)
    x, m = to_device(w["logits_bf16"], "bf16"), masks_to_device(w["masks"])
    ref = ms.masked_argmax(x, m)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        other = ms.masked_argmax(x, m)
    s.synchronize()
    assert torch.equal(ref.token_ids, other.token_ids) and torch.equal(ref.status, other.status)


def test_workspace_is_left_zeroed_across_layouts(cuda_lib):
    """Calls of different shapes share one workspace per stream; each must leave it zeroed
    (counters, flags and partials), whatever layout the previous call used."""
    rng = np.random.default_rng(12)
    for rows, vocab, dtype in ((4, 16385, "f64"), (4, 40000, "bf16"), (64, 128256, "bf16"),
                               (3, 151665, "f32"), (1, 256000, "f16"), (7, 99999, "bf16")):
        x, m = _random_case(rng, rows, vocab, dtype, 0.05)
        idx_ref, st_ref = oracle.masked_argmax(x, m, dtype=dtype)
        r = ms.masked_argmax(to_device(x, dtype), masks_to_device(m))
        _check(r.token_ids, r.status, idx_ref, st_ref)
        out, st = ms.mask_apply(to_device(x, dtype), masks_to_device(m))
        torch.cuda.synchronize()
        for buf in ms._WORKSPACES._buffers.values():
            assert int(torch.count_nonzero(buf)) == 0


@pytest.mark.parametrize("path", ["cluster", "ticket"])
def test_both_cross_cta_combines_match_oracle(path, cuda_lib):
    """Rows that fit one thread-block cluster merge CTA partials through distributed shared
    memory; the CLUSTER option off forces the global-ticket merge. Both must agree with the
    oracle for argmax, gather and shard keys."""
    with _lib.option_override({_lib.OPTION_CLUSTER: 1 if path == "cluster" else 0}):
        _combine_cases()


def _combine_cases():
    w = workloads.batched(rows=16)
    x, m = to_device(w["logits_bf16"], "bf16"), masks_to_device(w["masks"])
    idx_ref, st_ref = oracle.masked_argmax(w["logits_bf16"], w["masks"], dtype="bf16")
    r = ms.masked_argmax(x, m)
    _check(r.token_ids, r.status, idx_ref, st_ref)
    ids = np.array([3, 0, 15, 7] * 4, np.int32)
    idx_g, st_g = oracle.gather_masked_argmax(w["logits_bf16"], w["masks"], ids, dtype="bf16")
    g = ms.gather_masked_argmax(x, m, torch.from_numpy(ids).cuda())
    _check(g.token_ids, g.status, idx_g, st_g)
    keys = ms.vocab_partial_keys(x, m, 0)
    c = ms.combine_partial_keys(keys[None])
    _check(c.token_ids, c.status, idx_ref, st_ref)
    # 256,000-token rows need 125 warp segments: 8 CTAs of 16 warps in one cluster
    w2 = workloads.scaling(rows=4)
    idx2, st2 = oracle.masked_argmax(w2["logits_bf16"], w2["masks"], dtype="bf16")
    r2 = ms.masked_argmax(to_device(w2["logits_bf16"], "bf16"), masks_to_device(w2["masks"]))
    _check(r2.token_ids, r2.status, idx2, st2)
