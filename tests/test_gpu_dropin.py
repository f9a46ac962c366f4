"""The reference's mask and selector contracts, replayed on the drop-in boundary
(cases of onyx_cuda/tests/test_torch_grammar_mask.py:650-852) plus mask-apply parity."""

from __future__ import annotations

import gc
import weakref

import numpy as np
import pytest
import torch

import oracle
from onyx_b200 import masked_selection as ms
from onyx_b200 import workloads
from onyx_b200.torch_backend import TorchBackendInvariantError, select_cuda_argmax
from onyx_b200.torch_grammar_mask import (
    TorchGrammarMaskInvariantError,
    create_cuda_grammar_logit_mask,
)
from tests.gpu_util import host, masks_to_device, requires_cuda, to_device

pytestmark = [pytest.mark.gpu, requires_cuda]


def _bitwise_equal(a, b):
    return torch.equal(a.contiguous().view(torch.uint8), b.contiguous().view(torch.uint8))


class _Timing:
    def __init__(self):
        self.records = []

    def record_mask_timing(self, transfer, application):
        self.records.append((transfer, application))


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32", "float64"])
def test_mask_preserves_allowed_edge_values_bitwise(dtype):
    mask = create_cuda_grammar_logit_mask(8)
    logits = torch.tensor((-0.0, 0.0, 5.0, float("inf"), float("nan"), -7.0, float("-inf"), 99.0),
                          dtype=getattr(torch, dtype), device="cuda:0")
    original = logits.clone()
    valid = (0, 1, 3, 4, 6)
    result = mask.apply(logits, valid)
    idx = torch.tensor(valid, device="cuda:0")
    dis = torch.tensor((2, 5, 7), device="cuda:0")
    assert _bitwise_equal(result[idx], original[idx])
    assert torch.isneginf(result[dis]).all().item()
    assert _bitwise_equal(logits, original)
    assert result.shape == logits.shape and result.dtype == logits.dtype
    assert result.untyped_storage().data_ptr() != logits.untyped_storage().data_ptr()


def test_timed_mask_matches_untimed():
    mask = create_cuda_grammar_logit_mask(4, device_index=0)
    logits = torch.tensor((1.0, 5.0, 3.0, -2.0), device="cuda:0")
    timing = _Timing()
    untimed = mask.apply(logits, (1, 3))
    timed = mask.apply_with_timing(logits, (1, 3), timing)
    assert _bitwise_equal(timed, untimed)
    assert len(timing.records) == 1 and all(t > 0 for t in timing.records[0])


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32", "float64"])
def test_finite_extremes_with_all_and_all_but_one_support(dtype):
    tdt = getattr(torch, dtype)
    lim = torch.finfo(tdt)
    logits = torch.tensor((lim.min, lim.max, -1.0, 1.0), dtype=tdt, device="cuda:0")
    mask = create_cuda_grammar_logit_mask(4)
    complete = mask.apply(logits, (0, 1, 2, 3))
    almost = mask.apply(logits, (0, 1, 3))
    assert _bitwise_equal(complete, logits)
    keep = torch.tensor((0, 1, 3), device="cuda:0")
    assert _bitwise_equal(almost[keep], logits[keep]) and torch.isneginf(almost[2]).item()


def test_production_vocabulary_ceiling_and_padding_rejected():
    mask = create_cuda_grammar_logit_mask(151_665)
    logits = torch.zeros(151_665, dtype=torch.float16, device="cuda:0")
    logits[0] = 100.0
    result = mask.apply(logits, (151_664,))
    assert select_cuda_argmax(result) == 151_664
    with pytest.raises(TorchGrammarMaskInvariantError, match="151665"):
        mask.apply(torch.zeros(151_936, dtype=torch.float16, device="cuda:0"), (151_664,))


@pytest.mark.parametrize(
    ("make", "message"),
    [
        (lambda: torch.empty(0, device="cuda:0"), "configured vocabulary shape"),
        (lambda: torch.zeros((1, 4), device="cuda:0"), "configured vocabulary shape"),
        (lambda: torch.zeros(4), "non-CUDA"),
        (lambda: torch.zeros(4, dtype=torch.int64, device="cuda:0"), "floating-point"),
        (lambda: torch.zeros(4, dtype=torch.bool, device="cuda:0"), "floating-point"),
        (lambda: torch.zeros(4, dtype=torch.complex64, device="cuda:0"), "floating-point"),
    ],
)
def test_invalid_logits_rejected(make, message):
    with pytest.raises(TorchGrammarMaskInvariantError, match=message):
        create_cuda_grammar_logit_mask(4).apply(make(), (1,))


def test_all_negative_infinity_support_rejected():
    mask = create_cuda_grammar_logit_mask(3)
    logits = torch.full((3,), float("-inf"), device="cuda:0")
    for valid in ((1,), (0, 1, 2)):
        with pytest.raises(TorchGrammarMaskInvariantError, match="no logit support"):
            mask.apply(logits, valid)


def test_first_max_tie_break_and_infinity_ties():
    mask = create_cuda_grammar_logit_mask(6)
    logits = torch.tensor((99.0, 7.0, 8.0, 8.0, 8.0, 100.0), device="cuda:0")
    assert select_cuda_argmax(mask.apply(logits, (1, 3, 4))) == 3
    mask4 = create_cuda_grammar_logit_mask(4)
    inf_row = torch.tensor((float("inf"), 4.0, float("inf"), -3.0), device="cuda:0")
    assert select_cuda_argmax(mask4.apply(inf_row, (2,))) == 2
    assert select_cuda_argmax(mask4.apply(inf_row, (0, 2))) == 0


def test_disallowed_nan_removed_allowed_nan_rejected():
    mask = create_cuda_grammar_logit_mask(3)
    logits = torch.tensor((float("nan"), 2.0, 1.0), device="cuda:0")
    assert select_cuda_argmax(mask.apply(logits, (1, 2))) == 1
    allowed = mask.apply(logits, (0, 1))
    assert torch.isnan(allowed[0]).item()
    with pytest.raises(TorchBackendInvariantError, match="NaN"):
        select_cuda_argmax(allowed)


def test_no_rng_advance_and_no_state_between_calls():
    mask = create_cuda_grammar_logit_mask(5)
    logits = torch.arange(5, dtype=torch.float32, device="cuda:0")
    original = torch.cuda.get_rng_state(0).clone()
    try:
        torch.cuda.manual_seed(723)
        before = torch.cuda.get_rng_state(0).clone()
        first = mask.apply(logits, (0, 2))
        second = mask.apply(logits, (1, 4))
        assert torch.equal(torch.cuda.get_rng_state(0), before)
    finally:
        torch.cuda.set_rng_state(original, 0)
    assert torch.isneginf(first[1]).item() and torch.isneginf(second[2]).item()
    assert select_cuda_argmax(first) == 2 and select_cuda_argmax(second) == 4


def test_no_retained_references():
    mask = create_cuda_grammar_logit_mask(3)
    logits = torch.tensor((1.0, 2.0, 3.0), device="cuda:0")
    result = mask.apply(logits, (1,))
    lref, rref = weakref.ref(logits), weakref.ref(result)
    del logits, result
    gc.collect()
    assert lref() is None and rref() is None


def test_selector_rejects_nan_anywhere_and_returns_python_int():
    row = torch.tensor((1.0, float("nan"), 0.5), device="cuda:0")
    with pytest.raises(TorchBackendInvariantError, match="NaN"):
        select_cuda_argmax(row)
    ok = select_cuda_argmax(torch.tensor((-0.0, 0.0, -1.0), device="cuda:0"))
    assert ok == 0 and type(ok) is int
    assert select_cuda_argmax(torch.full((7,), float("-inf"), device="cuda:0")) == 0


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32", "f64"])
@pytest.mark.parametrize("vocab", [5, 33, 4097, 151665])
def test_mask_apply_matches_oracle(dtype, vocab):
    rng = np.random.default_rng(vocab)
    rows = 3
    if dtype == "bf16":
        x = workloads.normal_bf16(rng, (rows, vocab))
    else:
        x = (rng.standard_normal((rows, vocab)) * 3).astype(
            {"f16": np.float16, "f32": np.float32, "f64": np.float64}[dtype])
    m = workloads.bernoulli_masks(rng, np.full(rows, 0.1), vocab)
    m[2, :] = 0
    out_ref, st_ref = oracle.mask_apply(x, m, dtype=dtype)
    out, st = ms.mask_apply(to_device(x, dtype), masks_to_device(m))
    got = host(out.view(torch.int16) if dtype == "bf16" else out)
    if dtype == "bf16":
        got = got.view(np.uint16)
    assert got.tobytes() == np.ascontiguousarray(out_ref).tobytes()
    np.testing.assert_array_equal(host(st).astype(np.uint32), st_ref)
