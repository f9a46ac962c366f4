"""GPU parity: grammar-aware speculative verify against the reference's acceptance code
(golden vectors) and the oracle at the full 32 x 5 x 151,936 workload."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from onyx_b200 import masked_selection as ms
from onyx_b200 import workloads
from tests.conftest import golden_values, load_golden
from tests.gpu_util import host, masks_to_device, requires_cuda, to_device

pytestmark = [pytest.mark.gpu, requires_cuda]

VERIFY = load_golden("verify_cases.json")["cases"]


@pytest.mark.parametrize("case", VERIFY, ids=[c["name"] for c in VERIFY])
def test_golden_verify(case, cuda_lib):
    x = golden_values(case["bits"], case["dtype"])[None]
    m = np.asarray(case["mask_words"], np.uint32)[None]
    d = torch.tensor([case["drafts"]], dtype=torch.int32, device="cuda:0")
    r = ms.spec_verify(to_device(x, case["dtype"]), masks_to_device(m), d)
    assert int(host(r.accept_len)[0]) == case["expected_accept_len"]
    exp = -1 if case["expected_correction"] is None else case["expected_correction"]
    assert int(host(r.correction)[0]) == exp
    assert int(host(r.status)[0]) == oracle.STATUS_BITS[case["expected_status"]]


def _oracle_argmax(x, m):
    return oracle.masked_argmax(x, m, dtype="bf16")[0]


@pytest.fixture(scope="module")
def verify_workload():
    return workloads.spec_verify(_oracle_argmax)


@pytest.mark.parametrize("bonus", [True, False])
def test_full_workload_matches_oracle(verify_workload, bonus, cuda_lib):
    w = verify_workload
    acc_ref, corr_ref, st_ref = oracle.spec_verify(w["logits_bf16"], w["masks"], w["drafts"],
                                                   bonus=bonus, dtype="bf16")
    r = ms.spec_verify(to_device(w["logits_bf16"], "bf16"), masks_to_device(w["masks"]),
                       torch.from_numpy(w["drafts"]).cuda(), bonus=bonus)
    np.testing.assert_array_equal(host(r.accept_len), acc_ref)
    np.testing.assert_array_equal(host(r.correction), corr_ref)
    np.testing.assert_array_equal(host(r.status).astype(np.uint32), st_ref)
    # the drafts follow the masked argmax 70% of the time: every accept length occurs
    assert len(set(acc_ref.tolist())) > 2


def test_verify_equals_per_row_selection(verify_workload, cuda_lib):
    """accept/correction recomputed on the host from the batched per-row selections."""
    w = verify_workload
    b, g1, v = w["logits_bf16"].shape
    rows = ms.masked_argmax(to_device(w["logits_bf16"].reshape(b * g1, v), "bf16"),
                            masks_to_device(w["masks"].reshape(b * g1, -1)))
    sel = host(rows.token_ids).reshape(b, g1)
    r = ms.spec_verify(to_device(w["logits_bf16"], "bf16"), masks_to_device(w["masks"]),
                       torch.from_numpy(w["drafts"]).cuda())
    acc, corr = host(r.accept_len), host(r.correction)
    for i in range(b):
        k = 0
        while k < g1 - 1 and sel[i, k] == w["drafts"][i, k]:
            k += 1
        assert acc[i] == k and corr[i] == sel[i, k]


def test_padded_vocabulary_view_and_strides(cuda_lib):
    """Rows sliced out of a padded [B, G+1, 151936] model output (the reference's
    raw_logits[0, i, :vocab] view), real vocabulary 151,665."""
    rng = np.random.default_rng(4)
    b, g1, vpad, v = 3, 4, 151936, 151665
    x = workloads.normal_bf16(rng, (b, g1, vpad))
    m = workloads.bernoulli_masks(rng, np.full(b * g1, 0.02), v).reshape(b, g1, -1)
    best = oracle.masked_argmax(np.ascontiguousarray(x[:, :, :v]).reshape(b * g1, v),
                                m.reshape(b * g1, -1), dtype="bf16")[0].reshape(b, g1)
    d = best[:, : g1 - 1].astype(np.int32).copy()
    d[1, 1] = (d[1, 1] + 1) % v
    acc_ref, corr_ref, st_ref = oracle.spec_verify(np.ascontiguousarray(x[:, :, :v]), m, d,
                                                   dtype="bf16")
    t = to_device(x, "bf16")[:, :, :v]
    r = ms.spec_verify(t, masks_to_device(m), torch.from_numpy(d).cuda())
    np.testing.assert_array_equal(host(r.accept_len), acc_ref)
    np.testing.assert_array_equal(host(r.correction), corr_ref)
    assert list(acc_ref) == [g1 - 1, 1, g1 - 1]


def test_empty_support_and_nan_rows_end_the_decision(cuda_lib):
    rng = np.random.default_rng(8)
    b, g1, v = 4, 5, 40000
    x = workloads.normal_bf16(rng, (b, g1, v))
    m = workloads.bernoulli_masks(rng, np.full(b * g1, 0.05), v).reshape(b, g1, -1)
    best = oracle.masked_argmax(x.reshape(b * g1, v), m.reshape(b * g1, -1), dtype="bf16")[0]
    d = best.reshape(b, g1)[:, :4].astype(np.int32).copy()
    m[0, 2, :] = 0  # no-decision at position 2
    m[1, 4, :] = 0  # empty bonus row
    x[2, 1, 123] = 0x7FC0  # NaN in the support of position 1
    m[2, 1, 123 >> 5] |= np.uint32(1 << (123 & 31))
    x[3, 0, :] = 0xFF80  # all -inf at position 0
    acc_ref, corr_ref, st_ref = oracle.spec_verify(x, m, d, dtype="bf16")
    r = ms.spec_verify(to_device(x, "bf16"), masks_to_device(m), torch.from_numpy(d).cuda())
    np.testing.assert_array_equal(host(r.accept_len), acc_ref)
    np.testing.assert_array_equal(host(r.correction), corr_ref)
    np.testing.assert_array_equal(host(r.status).astype(np.uint32), st_ref)
    assert list(st_ref) == [ms.STATUS_EMPTY_MASK, ms.STATUS_EMPTY_MASK,
                            ms.STATUS_NAN_IN_SUPPORT, ms.STATUS_ALL_NEG_INF]
    assert list(acc_ref) == [2, 4, 1, 0]


def test_invalid_shapes_are_rejected(cuda_lib):
    x = torch.zeros(2, 1, 64, dtype=torch.bfloat16, device="cuda:0")
    with pytest.raises(ValueError, match="at least one draft"):
        ms.spec_verify(x, torch.zeros(2, 1, 2, dtype=torch.int32, device="cuda:0"),
                       torch.zeros(2, 0, dtype=torch.int32, device="cuda:0"))
