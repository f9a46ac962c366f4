"""GPU parity of the streaming form (one CTA per SM, a shared-memory ring fed by bulk copies,
split rows merged by 128-bit compare-and-swap in the workspace) against the oracle.

The STREAM option forces the form on every shape it can serve, so these cases cover shapes
far below the size from which it is chosen by default: rows split over many CTAs, rows
inside one CTA, ties across pieces and CTAs, empty / all -inf / NaN supports, gather rows
with bad DFA state ids, every verify decision, and the workspace left zero-filled."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from onyx_b200 import _lib
from onyx_b200 import masked_selection as ms
from onyx_b200 import workloads
from tests.gpu_util import host, masks_to_device, requires_cuda, to_device

pytestmark = [pytest.mark.gpu, requires_cuda]


@pytest.fixture
def stream_always(cuda_lib):
    with _lib.option_override({_lib.OPTION_STREAM: _lib.STREAM_ALWAYS}):
        yield


def _check(idx_gpu, st_gpu, idx_ref, st_ref):
    np.testing.assert_array_equal(host(st_gpu).astype(np.int64), st_ref.astype(np.int64))
    np.testing.assert_array_equal(host(idx_gpu).astype(np.int64), idx_ref.astype(np.int64))


def _case(rng, rows, vocab, dtype, density):
    if dtype == "bf16":
        x = workloads.normal_bf16(rng, (rows, vocab))
    else:
        np_dt = {"f32": np.float32, "f16": np.float16}[dtype]
        x = (rng.standard_normal((rows, vocab)) * 3.0).astype(np_dt)
    m = workloads.bernoulli_masks(rng, np.full(rows, density), vocab)
    return x, m


def _set(x, dtype, cols, value):
    if dtype == "bf16":
        x[cols] = workloads.bf16_bits(np.full(np.size(cols), value, np.float32))
    else:
        x[cols] = value


def _allow(m, row, cols):
    for j in np.atleast_1d(cols):
        m[row, j >> 5] |= np.uint32(1 << (int(j) & 31))


def _workspace_zero():
    torch.cuda.synchronize()
    for buf in ms._WORKSPACES._buffers.values():
        assert int(torch.count_nonzero(buf)) == 0


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("rows,vocab", [(1, 128), (1, 32000), (3, 4096), (5, 128256),
                                        (64, 128256), (150, 1024), (300, 8320), (7, 151936)])
def test_random_rows(dtype, rows, vocab, stream_always):
    rng = np.random.default_rng(rows * 1000 + vocab + len(dtype))
    x, m = _case(rng, rows, vocab, dtype, 0.05)
    idx_ref, st_ref = oracle.masked_argmax(x, m, dtype=dtype)
    r = ms.masked_argmax(to_device(x, dtype), masks_to_device(m))
    _check(r.token_ids, r.status, idx_ref, st_ref)
    _workspace_zero()


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_ties_across_pieces_and_ctas_resolve_lowest(dtype, stream_always):
    """Equal maxima in different pieces of one warp, in different CTAs and at both ends of
    a row: the lowest index wins. Signed zeros tie."""
    rng = np.random.default_rng(31)
    rows, vocab = 6, 128256
    x, m = _case(rng, rows, vocab, dtype, 0.02)
    spots = [7, 16384 + 7, 40000, 90001, vocab - 1]
    for r in range(rows):
        cols = spots[r % 3:]
        _set(x[r], dtype, cols, 60.0)
        _allow(m, r, cols)
    # row 5: every valid value is +0.0 or -0.0
    m[5] = 0
    zeros = np.array([100, 20000, 70000, 128000])
    _allow(m, 5, zeros)
    _set(x[5], dtype, zeros[[0, 2]], -0.0)
    _set(x[5], dtype, zeros[[1, 3]], 0.0)
    idx_ref, st_ref = oracle.masked_argmax(x, m, dtype=dtype)
    r = ms.masked_argmax(to_device(x, dtype), masks_to_device(m))
    _check(r.token_ids, r.status, idx_ref, st_ref)
    assert list(host(r.token_ids)) == [7, 16384 + 7, 40000, 7, 16384 + 7, 100]


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_status_rows(dtype, stream_always):
    """Empty mask, all -inf support, NaN in the support (and NaN outside it, ignored),
    +inf ties, a single valid id at the very end."""
    rng = np.random.default_rng(77)
    rows, vocab = 8, 151936
    x, m = _case(rng, rows, vocab, dtype, 0.03)
    m[0] = 0                                              # empty
    m[1] = 0
    _allow(m, 1, [5, 70000, 151935])
    _set(x[1], dtype, [5, 70000, 151935], -np.inf)        # all -inf
    _set(x[2], dtype, [90000], np.nan)
    _allow(m, 2, [90000])                                 # NaN in the support
    m[3, 2000 >> 5] &= ~np.uint32(1 << (2000 & 31))
    _set(x[3], dtype, [2000], np.nan)                     # NaN outside the support
    _set(x[4], dtype, [30, 100000], np.inf)
    _allow(m, 4, [30, 100000])                            # +inf tie -> lowest
    m[5] = 0
    _allow(m, 5, [151935])                                # last id only
    idx_ref, st_ref = oracle.masked_argmax(x, m, dtype=dtype)
    r = ms.masked_argmax(to_device(x, dtype), masks_to_device(m))
    _check(r.token_ids, r.status, idx_ref, st_ref)
    st = host(r.status)
    assert st[0] == ms.STATUS_EMPTY_MASK and st[1] == ms.STATUS_ALL_NEG_INF
    assert st[2] == ms.STATUS_NAN_IN_SUPPORT and st[3] == 0
    assert int(host(r.token_ids)[4]) == 30 and int(host(r.token_ids)[5]) == 151935
    _workspace_zero()


def test_gather_with_bad_states(stream_always):
    w = workloads.table_gather(rows=64, states=512)
    ids = w["state_ids"].copy()
    ids[[0, 17, 63]] = [-1, 512, 1 << 30]
    idx_ref, st_ref = oracle.gather_masked_argmax(w["logits_bf16"], w["table"], ids, dtype="bf16")
    g = ms.gather_masked_argmax(to_device(w["logits_bf16"], "bf16"), masks_to_device(w["table"]),
                                torch.from_numpy(ids).cuda())
    _check(g.token_ids, g.status, idx_ref, st_ref)
    assert all(host(g.status)[[0, 17, 63]] == ms.STATUS_BAD_STATE)
    _workspace_zero()


def test_full_gather_workload(stream_always):
    w = workloads.table_gather()
    idx_ref, st_ref = oracle.gather_masked_argmax(w["logits_bf16"], w["table"], w["state_ids"],
                                                  dtype="bf16")
    g = ms.gather_masked_argmax(to_device(w["logits_bf16"], "bf16"), masks_to_device(w["table"]),
                                torch.from_numpy(w["state_ids"]).cuda())
    _check(g.token_ids, g.status, idx_ref, st_ref)


@pytest.mark.parametrize("bonus", [True, False])
@pytest.mark.parametrize("batch,gamma,vocab", [(32, 4, 151936), (3, 1, 4096), (5, 7, 32000),
                                               (2, 31, 1024), (40, 2, 128)])
def test_verify(batch, gamma, vocab, bonus, stream_always):
    rng = np.random.default_rng(batch * 100 + gamma)
    g1 = gamma + 1
    x = workloads.normal_bf16(rng, (batch, g1, vocab))
    m = workloads.bernoulli_masks(rng, rng.uniform(0.01, 0.1, batch * g1), vocab)
    m = m.reshape(batch, g1, -1)
    best = oracle.masked_argmax(x.reshape(batch * g1, vocab), m.reshape(batch * g1, -1),
                                dtype="bf16")[0].reshape(batch, g1)
    d = best[:, :gamma].astype(np.int32).copy()
    # mismatches at varied positions; an empty mask (status) in entry 1
    for b in range(batch):
        if b % 3 == 1:
            d[b, b % gamma] = (d[b, b % gamma] + 1) % vocab
    if batch > 1:
        m[1, min(1, gamma - 1)] = 0
    acc_ref, corr_ref, st_ref = oracle.spec_verify(x, m, d, bonus=bonus, dtype="bf16")
    r = ms.spec_verify(to_device(x, "bf16"), masks_to_device(m), torch.from_numpy(d).cuda(),
                       bonus=bonus)
    np.testing.assert_array_equal(host(r.accept_len), acc_ref)
    np.testing.assert_array_equal(host(r.correction), corr_ref)
    np.testing.assert_array_equal(host(r.status).astype(np.uint32), st_ref)
    _workspace_zero()


def test_vocab_shard_keys(stream_always):
    w = workloads.scaling(rows=16, vocab=256000)
    x, m = w["logits_bf16"], w["masks"]
    keys = []
    for lo, hi in ((0, 64000), (64000, 128000), (128000, 192000), (192000, 256000)):
        keys.append(ms.vocab_partial_keys(to_device(np.ascontiguousarray(x[:, lo:hi]), "bf16"),
                                          masks_to_device(np.ascontiguousarray(m[:, lo // 32:hi // 32])),
                                          lo))
    c = ms.combine_partial_keys(torch.stack(keys))
    idx_ref, st_ref = oracle.masked_argmax(x, m, dtype="bf16")
    _check(c.token_ids, c.status, idx_ref, st_ref)


def test_default_and_forced_forms_agree(cuda_lib):
    """The headline shape under every form: default choice, streaming forced, streaming off."""
    w = workloads.batched()
    x, m = to_device(w["logits_bf16"], "bf16"), masks_to_device(w["masks"])
    idx_ref, st_ref = oracle.masked_argmax(w["logits_bf16"], w["masks"], dtype="bf16")
    for mode in (_lib.STREAM_AUTO, _lib.STREAM_ALWAYS, _lib.STREAM_NEVER):
        with _lib.option_override({_lib.OPTION_STREAM: mode}):
            for _ in range(2):  # the second call runs on the workspace the first left behind
                r = ms.masked_argmax(x, m)
                _check(r.token_ids, r.status, idx_ref, st_ref)
