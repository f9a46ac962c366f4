"""The cluster path's one wait is bounded: rank 0 of a row's cluster waits on an mbarrier for
the other CTAs' keys, and gives up after 0.5 s with ONYX_STATUS_WAIT_TIMEOUT instead of
hanging. The test option ONYX_OPTION_TEST_WITHHELD_KEY_BYTES makes rank 0 expect key bytes
that no CTA sends, so the wait runs out; nothing faults, and the context stays usable
afterwards."""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import oracle
from onyx_b200 import _lib
from onyx_b200 import masked_selection as ms
from onyx_b200 import workloads
from tests.gpu_util import host, masks_to_device, requires_cuda, to_device

pytestmark = [pytest.mark.gpu, requires_cuda]


def _inputs(rows, vocab=128256, seed=4):
    rng = np.random.default_rng(seed)
    x = workloads.normal_bf16(rng, (rows, vocab))
    m = workloads.bernoulli_masks(rng, np.full(rows, 0.05), vocab)
    return x, m


def test_withheld_keys_time_out_and_the_context_recovers(cuda_lib):
    x, m = _inputs(2)
    xd, md = to_device(x, "bf16"), masks_to_device(m)
    with _lib.option_override({_lib.OPTION_CLUSTER: 1, _lib.OPTION_TEST_WITHHELD_KEY_BYTES: 8}):
        _withheld_calls(xd, md)

    idx_ref, st_ref = oracle.masked_argmax(x, m, dtype="bf16")
    r2 = ms.masked_argmax(xd, md)
    np.testing.assert_array_equal(host(r2.token_ids).astype(np.int64), idx_ref.astype(np.int64))
    np.testing.assert_array_equal(host(r2.status).astype(np.int64), st_ref.astype(np.int64))


def _withheld_calls(xd, md):
    t0 = time.perf_counter()
    r = ms.masked_argmax(xd, md)
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert list(host(r.status)) == [ms.STATUS_WAIT_TIMEOUT] * 2
    assert list(host(r.token_ids)) == [-1, -1]
    assert 0.3 < waited < 20.0

    # verify: the timed-out row decides the group with its status
    v = ms.spec_verify(xd.view(1, 2, -1), md.view(1, 2, -1),
                       torch.zeros((1, 1), dtype=torch.int32, device=xd.device))
    assert int(host(v.status)[0]) == ms.STATUS_WAIT_TIMEOUT
    assert int(host(v.accept_len)[0]) == 0 and int(host(v.correction)[0]) == -1

    # shard keys: the timed-out shard's key wins the combine and carries the status
    keys = ms.vocab_partial_keys(xd, md, 0)
    c = ms.combine_partial_keys(keys[None])
    assert list(host(c.status)) == [ms.STATUS_WAIT_TIMEOUT] * 2
