"""GPU parity of masked temperature / top-p sampling (onyx_masked_sample) against the oracle
(oracle/sampling.py: the reference's _filtered_reference_weights, pinned to fixtures made
by the reference, plus the Philox4x32-10 draw), and the reference's sampler tests
(test_torch_grammar_mask.py:758-794: replay, confinement to the valid set, +inf rules).

Same arguments give the same draw on both sides; the token ids must be equal. (Block
reductions round differently from the oracle's sequential sums by a few units in the last
place; none of these seeded cases puts a draw that close to a boundary.)"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sampling as osamp
from onyx_b200 import _lib
from onyx_b200 import masked_selection as ms
from onyx_b200 import sampling, workloads
from tests.conftest import golden_values, load_golden
from tests.gpu_util import host, masks_to_device, requires_cuda, to_device

pytestmark = [pytest.mark.gpu, requires_cuda]

# Kernel forms: the default (a cluster of CTAs per row, sized from the batch), the one-CTA
# kernel, and clusters of 3 and 16 CTAs (the library option ONYX_OPTION_SAMPLE_FORM).
FORMS = {"default": 0, "single": -1, "cluster:3": 3, "cluster:16": 16}


@pytest.fixture(params=list(FORMS))
def form(request, cuda_lib):
    with _lib.option_override({_lib.OPTION_SAMPLE_FORM: FORMS[request.param]}):
        yield request.param


def _float64(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return (x.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return x.astype(np.float64)


def _check(x, m, dtype, temperature, top_p, seed, call):
    r = sampling.masked_sample(to_device(x, dtype), None if m is None else masks_to_device(m),
                               temperature=temperature, top_p=top_p, seed=seed, call=call)
    idx_ref, st_ref = osamp.masked_sample(_float64(x, dtype), m, temperature, top_p, seed, call)
    np.testing.assert_array_equal(host(r.status).astype(np.uint32), st_ref)
    np.testing.assert_array_equal(host(r.token_ids), idx_ref)
    return host(r.token_ids)


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("policy", [(1.0, 1.0), (0.8, 0.9), (0.5, 0.3), (2.0, 0.99), (1.0, 0.02)])
def test_random_rows_match_oracle(dtype, policy, form, cuda_lib):
    rng = np.random.default_rng(len(dtype) * 100 + int(policy[1] * 1000))
    vocab = 5003
    rows = 12
    if dtype == "bf16":
        x = workloads.normal_bf16(rng, (rows, vocab))
    else:
        x = (rng.standard_normal((rows, vocab)) * 3.0).astype(
            np.float16 if dtype == "f16" else np.float32)
    m = workloads.bernoulli_masks(rng, rng.uniform(0.002, 0.5, rows), vocab)
    for call in (0, 1, 7):
        _check(x, m, dtype, policy[0], policy[1], 1234, call)


def test_full_vocabulary_rows(form, cuda_lib):
    w = workloads.batched(rows=8)
    for seed, (t, tp) in ((5, (0.8, 0.9)), (6, (1.0, 1.0)), (7, (0.3, 0.5))):
        _check(w["logits_bf16"], w["masks"], "bf16", t, tp, seed, 3)
    # unmasked: every id valid
    _check(w["logits_bf16"], None, "bf16", 1.0, 0.95, 11, 0)


def test_batch_of_full_rows_dense_and_sparse_masks(cuda_lib):
    """64 full-vocabulary rows, two CTAs per row in the default form: masks from 0.5 % to
    60 % dense, so some warps work from their list of valid ids and others, with more valid
    ids than a list holds, walk their whole range; unmasked rows too."""
    rng = np.random.default_rng(64)
    x = workloads.normal_bf16(rng, (64, 128256))
    dens = np.concatenate([rng.uniform(0.005, 0.2, 40), rng.uniform(0.2, 0.6, 24)])
    m = workloads.bernoulli_masks(rng, dens, 128256)
    for t, tp, call in ((0.8, 0.9, 0), (0.6, 0.99, 2)):
        _check(x, m, "bf16", t, tp, 2024, call)
    _check(x[:8], None, "bf16", 0.8, 0.9, 5, 0)


def test_special_rows(form, cuda_lib):
    vocab = 300
    x = np.zeros((8, vocab), np.float32)
    rng = np.random.default_rng(3)
    x[:] = rng.standard_normal((8, vocab)) * 2
    m = np.full((8, (vocab + 31) // 32), 0xFFFFFFFF, np.uint32)
    m[:, -1] &= np.uint32((1 << (vocab % 32)) - 1)
    x[0, [3, 40, 41, 299]] = 50.0           # exact ties among the leaders
    x[1, [7, 100]] = np.inf                  # +inf ids share the mass
    x[2, 17] = np.nan                        # NaN valid
    x[3, :] = -np.inf                        # all -inf
    m[4, :] = 0                              # empty mask
    x[5, :] = 0.5                            # flat: top_p keeps a prefix of the ids
    x[6, ::3] = -np.inf                      # some -inf, the rest finite
    x[7, 250] = 1e30                         # one id takes all the mass; others underflow
    for tp in (0.05, 0.5, 1.0):
        for call in range(4):
            got = _check(x, m, "f32", 0.7, tp, 99, call)
            assert got[1] in (7, 100)
    st = host(sampling.masked_sample(to_device(x, "f32"), masks_to_device(m), temperature=1.0,
                                     top_p=1.0, seed=1).status)
    assert list(st[2:5]) == [ms.STATUS_NAN_IN_SUPPORT, ms.STATUS_ALL_NEG_INF, ms.STATUS_EMPTY_MASK]


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_wide_value_ranges(dtype, form, cuda_lib):
    """Candidates on both sides of zero and over many exponents (a hot temperature or a
    top_p near 1): the radix select starts at the sign bit and takes several levels."""
    rng = np.random.default_rng(77)
    rows, vocab = 6, 9001
    x = rng.standard_normal((rows, vocab)) * np.array([[0.3], [3.0], [30.0], [1.0], [8.0], [0.01]])
    x = x.astype(np.float32)
    if dtype == "bf16":
        x = workloads.bf16_bits(x)
    elif dtype == "f16":
        x = x.astype(np.float16)
    m = workloads.bernoulli_masks(rng, rng.uniform(0.05, 1.0, rows), vocab)
    for t, tp in ((50.0, 0.9), (5.0, 0.999), (1.0, 0.5), (0.05, 0.95)):
        for call in (0, 3):
            _check(x, m, dtype, t, tp, 4242, call)


def test_unaligned_rows(form, cuda_lib):
    """Rows whose start is not 16-byte aligned (a column slice) stage element by element."""
    rng = np.random.default_rng(5)
    full = workloads.normal_bf16(rng, (4, 3001))
    xt = to_device(full, "bf16")[:, 1:]
    x = full[:, 1:]
    m = workloads.bernoulli_masks(rng, np.array([0.5, 0.1, 1.0, 0.02]), 3000)
    for call in range(3):
        r = sampling.masked_sample(xt, masks_to_device(m), temperature=0.9, top_p=0.8,
                                   seed=8, call=call)
        idx_ref, st_ref = osamp.masked_sample(_float64(x, "bf16"), m, 0.9, 0.8, 8, call)
        np.testing.assert_array_equal(host(r.status).astype(np.uint32), st_ref)
        np.testing.assert_array_equal(host(r.token_ids), idx_ref)


def test_many_ties_at_the_cut(form, cuda_lib):
    """Hundreds of ids share the value the cut falls on; the kept ones are the first in id
    order, spread over several warps and CTAs."""
    vocab = 20000
    x = np.full((3, vocab), -5.0, np.float32)
    x[:, ::7] = 1.0     # 2858 ties at the top
    x[1, 100] = 2.0     # one id above them
    x[2, ::5000] = 3.0  # four ids above them
    for tp in (0.1, 0.5, 0.97):
        for call in range(4):
            _check(x, None, "f32", 1.0, tp, 31, call)


@pytest.mark.parametrize("case", load_golden("sampling_cases.json")["cases"][:18],
                         ids=lambda c: c["name"])
def test_reference_fixture_rows_sample_inside_the_kept_set(case, cuda_lib):
    """Every draw on a reference fixture row is one of the ids the reference keeps."""
    x = golden_values(case["bits"], case["dtype"])[None]
    m = np.asarray(case["mask_words"], np.uint32)[None]
    kept = {t for t, _ in case["expected_kept"]}
    for call in range(6):
        r = sampling.masked_sample(to_device(x, case["dtype"]), masks_to_device(m),
                                   temperature=case["temperature"], top_p=case["top_p"],
                                   seed=17, call=call)
        tok, st = int(host(r.token_ids)[0]), int(host(r.status)[0])
        if case["expected_status"] == "ok":
            assert st == 0 and tok in kept
        else:
            assert st != 0 and tok == -1


def test_draws_follow_the_distribution(cuda_lib):
    """4,000 calls on one row: the frequencies match the kept probabilities (chi-square)."""
    x = np.array([[2.0, 1.0, 0.5, 0.0, -1.0, 3.0, -np.inf, 1.5]], np.float32)
    xt = to_device(x, "f32")
    _, kept = osamp.kept_weights(x[0].astype(np.float64), np.ones(8, bool), 1.2, 0.9)
    counts = np.zeros(8)
    for call in range(4000):
        counts[int(host(sampling.masked_sample(xt, temperature=1.2, top_p=0.9, seed=3,
                                                call=call).token_ids)[0])] += 1
    total = sum(p for _, p in kept)
    expected = np.zeros(8)
    for t, p in kept:
        expected[t] = 4000 * p / total
    assert counts[expected == 0].sum() == 0
    nz = expected > 0
    chi2 = float((((counts - expected) ** 2)[nz] / expected[nz]).sum())
    assert chi2 < 25.0, (counts, expected)  # 99.9th percentile of chi-square, <= 6 dof: 22.5


def test_reference_sampler_contract(cuda_lib):
    """The reference's CUDA sampler tests, on this sampler."""
    from onyx_b200 import select_cuda_argmax
    from onyx_b200.torch_grammar_mask import create_cuda_grammar_logit_mask

    mask = create_cuda_grammar_logit_mask(6)
    logits = torch.tensor((99.0, 7.0, 8.0, 8.0, 8.0, 100.0), device="cuda:0")
    valid = (1, 3, 4)
    masked = mask.apply(logits, valid)
    assert select_cuda_argmax(masked) == 3
    policy = sampling.TemperatureTopPSelection(temperature=0.8, top_p=0.9, seed=23)
    first = sampling.create_cuda_sampler(policy)
    second = sampling.create_cuda_sampler(policy)
    a = tuple(first(masked) for _ in range(20))
    b = tuple(second(masked) for _ in range(20))
    assert a == b and set(a) <= set(valid)

    mask4 = create_cuda_grammar_logit_mask(4)
    logits4 = torch.tensor((float("inf"), 4.0, float("inf"), -3.0), device="cuda:0")
    one = mask4.apply(logits4, (2,))
    for seed in (0, 1, 99):
        for top_p in (0.1, 0.5, 1.0):
            s = sampling.create_cuda_sampler(sampling.TemperatureTopPSelection(1.0, top_p, seed))
            assert tuple(s(one) for _ in range(5)) == (2,) * 5
    both = mask4.apply(logits4, (0, 2))
    s1 = sampling.create_cuda_sampler(sampling.TemperatureTopPSelection(1.0, 1.0, 7))
    s2 = sampling.create_cuda_sampler(sampling.TemperatureTopPSelection(1.0, 1.0, 7))
    seq1 = tuple(s1(both) for _ in range(12))
    assert seq1 == tuple(s2(both) for _ in range(12)) and set(seq1) <= {0, 2}
