"""The allocation-free masked argmax against the workspace entry point, through the C ABI.

``onyx_masked_argmax_noalloc`` exists for callers that cannot allocate device memory when
they call (a serving process whose GPU memory is pre-reserved by its own pool, or a binding
that only receives pointers to buffers allocated elsewhere), so it cannot take a workspace
and keeps its split-row scratch in a fixed array inside the library instead. Its outputs
must equal those of ``onyx_masked_argmax`` exactly (token ids and status bits are
integers), on consecutive calls that reuse the same scratch. This file sorts last so that a
run stopping at the first failure has already run every other test.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from onyx_b200 import _lib, workloads
from tests.gpu_util import masks_to_device, requires_cuda, to_device

pytestmark = [pytest.mark.gpu, requires_cuda]


def _with_workspace(lib, x, m):
    rows, vocab = x.shape
    idx = torch.empty(rows, dtype=torch.int32, device=x.device)
    st = torch.empty(rows, dtype=torch.int32, device=x.device)
    need = lib.onyx_masked_argmax_workspace_size(rows, vocab, _lib.DTYPE_BF16)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=x.device)
    rc = lib.onyx_masked_argmax(
        x.data_ptr(), _lib.DTYPE_BF16, rows, vocab, x.stride(0), m.data_ptr(), m.stride(0),
        idx.data_ptr(), st.data_ptr(), ws.data_ptr(), ws.numel(),
        torch.cuda.current_stream().cuda_stream,
    )
    assert rc == _lib.OK
    return idx, st


def _without_workspace(lib, x, m):
    rows, vocab = x.shape
    idx = torch.full((rows,), -7, dtype=torch.int32, device=x.device)
    st = torch.full((rows,), -7, dtype=torch.int32, device=x.device)
    rc = lib.onyx_masked_argmax_noalloc(
        x.data_ptr(), _lib.DTYPE_BF16, rows, vocab, x.stride(0),
        None if m is None else m.data_ptr(), 0 if m is None else m.stride(0),
        idx.data_ptr(), st.data_ptr(), torch.cuda.current_stream().cuda_stream,
    )
    assert rc == _lib.OK, lib.onyx_error_string(rc)
    return idx, st


@pytest.mark.parametrize("cluster", [1, 0], ids=["cluster-combine", "scratch-combine"])
def test_noalloc_matches_workspace_entry_point_on_consecutive_calls(cluster, cuda_lib):
    """With the cluster option on, rows that fit one cluster combine in distributed shared
    memory and the scratch is not touched; with it off, every split row goes through the
    fixed scratch array. Both must match the workspace entry point, call after call."""
    lib = cuda_lib
    first = workloads.batched()  # 64 x 128,256 bf16: rows split over 63 warps each
    second = workloads.batched(seed=77, rows=40, vocab=151936)
    with _lib.option_override({_lib.OPTION_CLUSTER: cluster}):
        for w in (first, second, first):
            x = to_device(w["logits_bf16"], "bf16")
            m = masks_to_device(w["masks"])
            ref_idx, ref_st = _with_workspace(lib, x, m)
            got_idx, got_st = _without_workspace(lib, x, m)
            torch.cuda.synchronize()
            assert torch.equal(got_idx, ref_idx)
            assert torch.equal(got_st, ref_st)


def test_noalloc_rows_longer_than_a_cluster_use_the_scratch(cuda_lib):
    """300,000-column rows need 147 warp segments, more than one cluster holds: their CTAs
    combine through the fixed scratch even with the cluster option on."""
    w = workloads.batched(seed=5, rows=6, vocab=300000)
    x = to_device(w["logits_bf16"], "bf16")
    m = masks_to_device(w["masks"])
    for _ in range(2):
        ref_idx, ref_st = _with_workspace(cuda_lib, x, m)
        got_idx, got_st = _without_workspace(cuda_lib, x, m)
        torch.cuda.synchronize()
        assert torch.equal(got_idx, ref_idx) and torch.equal(got_st, ref_st)


def test_noalloc_unmasked_rows(cuda_lib):
    rng = np.random.default_rng(3)
    x = to_device(workloads.normal_bf16(rng, (8, 100000)), "bf16")
    a = _without_workspace(cuda_lib, x, None)
    b = _without_workspace(cuda_lib, x, None)
    ref = torch.argmax(x.float(), dim=1).to(torch.int32)
    torch.cuda.synchronize()
    assert torch.equal(a[0], ref) and torch.equal(b[0], ref)
    assert int(torch.count_nonzero(a[1])) == 0


def test_noalloc_rejects_requests_beyond_its_scratch(cuda_lib):
    """With the cluster option off, a request whose split-row partials exceed the fixed
    scratch is refused before any launch. The buffers are real and sized for the request,
    so nothing could read out of bounds even if the call were accepted."""
    with _lib.option_override({_lib.OPTION_CLUSTER: 0}):
        _rejects_beyond_scratch(cuda_lib)


def _rejects_beyond_scratch(lib):
    rows, vocab = 32768, 16385  # 9 warp segments -> 2 CTAs per row: 32,768 * (4 + 32) B > 1 MiB
    count_bytes = (rows * 4 + 255) // 256 * 256
    assert count_bytes + rows * 2 * 16 > _lib.NOALLOC_SCRATCH_BYTES
    x = torch.empty((rows, vocab), dtype=torch.bfloat16, device="cuda:0")
    m = torch.zeros((rows, (vocab + 31) // 32), dtype=torch.int32, device="cuda:0")
    idx = torch.empty(rows, dtype=torch.int32, device="cuda:0")
    st = torch.empty(rows, dtype=torch.int32, device="cuda:0")
    rc = lib.onyx_masked_argmax_noalloc(
        x.data_ptr(), _lib.DTYPE_BF16, rows, vocab, x.stride(0), m.data_ptr(), m.stride(0),
        idx.data_ptr(), st.data_ptr(), torch.cuda.current_stream().cuda_stream,
    )
    torch.cuda.synchronize()
    assert rc == _lib.ERR_SCRATCH_LIMIT
    assert b"scratch" in lib.onyx_error_string(rc)
