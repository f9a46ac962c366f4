"""GPU parity of the vocabulary-sharded path: shard keys + combine == unsharded selection.

The shards are emulated on one GPU (each shard a separate column slice and kernel call);
the multi-process NCCL version runs when more than one GPU is visible."""

from __future__ import annotations

import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from onyx_b200 import masked_selection as ms
from onyx_b200 import vocab_parallel, workloads
from tests.gpu_util import host, masks_to_device, requires_cuda, to_device

pytestmark = [pytest.mark.gpu, requires_cuda]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_sharded_keys_combine_to_unsharded(world, cuda_lib):
    w = workloads.scaling(rows=64)
    x, m = w["logits_bf16"], w["masks"]
    vocab = x.shape[1]
    # a tie straddling shard boundaries
    j1, j2 = 5, vocab - 5
    x[0, [j1, j2]] = workloads.bf16_bits(np.array([40.0, 40.0], np.float32))
    for j in (j1, j2):
        m[0, j >> 5] |= np.uint32(1 << (j & 31))
    idx_ref, st_ref = oracle.masked_argmax(x, m, dtype="bf16")
    xt, mt = to_device(x, "bf16"), masks_to_device(m)
    keys = []
    for r in range(world):
        lo, hi = vocab_parallel.vocab_shard_bounds(vocab, r, world)
        keys.append(ms.vocab_partial_keys(xt[:, lo:hi], mt[:, lo // 32 : (hi + 31) // 32], lo))
    res = ms.combine_partial_keys(torch.stack(keys))
    np.testing.assert_array_equal(host(res.status).astype(np.uint32), st_ref)
    np.testing.assert_array_equal(host(res.token_ids), idx_ref)
    assert int(host(res.token_ids)[0]) == j1


def test_scaling_workload_batch_shards_full_width(cuda_lib):
    """1024 x 256,000 bf16 at 5% density: per-shard-of-rows kernels == oracle."""
    w = workloads.scaling()
    idx_ref, st_ref = oracle.masked_argmax(w["logits_bf16"], w["masks"], dtype="bf16")
    xt, mt = to_device(w["logits_bf16"], "bf16"), masks_to_device(w["masks"])
    got_i, got_s = [], []
    for r in range(8):
        lo, hi = vocab_parallel.batch_shard_bounds(1024, r, 8)
        res = ms.masked_argmax(xt[lo:hi], mt[lo:hi])
        got_i.append(host(res.token_ids))
        got_s.append(host(res.status))
    np.testing.assert_array_equal(np.concatenate(got_i), idx_ref)
    np.testing.assert_array_equal(np.concatenate(got_s).astype(np.uint32), st_ref)


_NCCL_WORKER = r"""
import os, sys, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, os.environ["ONYX_ROOT"])
from onyx_b200 import vocab_parallel, workloads
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
w = workloads.scaling(rows=128, vocab=32000 * world)
x, m = w["logits_bf16"], w["masks"]
lo, hi = vocab_parallel.vocab_shard_bounds(x.shape[1], rank, world)
xt = torch.from_numpy(np.ascontiguousarray(x[:, lo:hi]).view(np.int16)).cuda().view(torch.bfloat16)
mt = torch.from_numpy(np.ascontiguousarray(m[:, lo // 32:(hi + 31) // 32]).view(np.int32)).cuda()
res = vocab_parallel.vocab_parallel_masked_argmax(xt, mt, lo)
out = torch.stack((res.token_ids, res.status)).cpu().numpy()
if rank == 0:
    np.save(os.environ["ONYX_OUT"], out)
dist.barrier()
dist.destroy_process_group()
"""


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_nccl_vocab_parallel_multi_rank(tmp_path, cuda_lib):
    """One rank per GPU of the box (2 to 8): shards of a 32,000 x world vocabulary."""
    world = min(torch.cuda.device_count(), 8)
    script = tmp_path / "worker.py"
    script.write_text(_NCCL_WORKER)
    out = tmp_path / "out.npy"
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, ONYX_ROOT=str(Path(__file__).resolve().parents[1]), ONYX_OUT=str(out),
               NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(port), str(script)]
    subprocess.run(["timeout", "-k", "30", "300", *cmd], check=True, env=env)
    got = np.load(out)
    w = workloads.scaling(rows=128, vocab=32000 * world)
    idx_ref, st_ref = oracle.masked_argmax(w["logits_bf16"], w["masks"], dtype="bf16")
    np.testing.assert_array_equal(got[0], idx_ref)
    np.testing.assert_array_equal(got[1].astype(np.uint32), st_ref)


def test_peer_exchange_single_rank_matches_oracle(cuda_lib):
    """world = 1: the key kernel stores into the rank's own exchange buffer, the exchange
    kernel raises and reads its own flag; consecutive calls alternate the two parities."""
    import ctypes
    from onyx_b200 import _lib
    lib = cuda_lib
    rows, rows_cap = 64, 96
    nbytes = lib.onyx_exchange_buffer_bytes(1, rows_cap)
    handle = ctypes.create_string_buffer(lib.onyx_ipc_handle_bytes())
    own = ctypes.c_void_p()
    assert lib.onyx_ipc_alloc(nbytes, ctypes.byref(own), handle) == _lib.OK
    bases = (ctypes.c_void_p * 1)(own.value)
    try:
        for seed in (3, 4, 5):  # three calls: both parities, then the first again
            w = workloads.scaling(seed=seed, rows=rows, vocab=32000)
            x, m = w["logits_bf16"], w["masks"]
            idx_ref, st_ref = oracle.masked_argmax(x, m, dtype="bf16")
            res = ms.vocab_exchange_argmax(to_device(x, "bf16"), masks_to_device(m), 0, world=1,
                                           rank=0, exchange_bases=bases, rows_cap=rows_cap)
            np.testing.assert_array_equal(host(res.token_ids), idx_ref)
            np.testing.assert_array_equal(host(res.status).astype(np.uint32), st_ref)
        # captured in a CUDA graph: the device-side call count keeps the parities right
        w = workloads.scaling(seed=6, rows=rows, vocab=32000)
        idx_ref, st_ref = oracle.masked_argmax(w["logits_bf16"], w["masks"], dtype="bf16")
        xt, mt = to_device(w["logits_bf16"], "bf16"), masks_to_device(w["masks"])
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            ms.vocab_exchange_argmax(xt, mt, 0, world=1, rank=0, exchange_bases=bases,
                                     rows_cap=rows_cap)  # workspace and library warm-up
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            outs = [ms.vocab_exchange_argmax(xt, mt, 0, world=1, rank=0, exchange_bases=bases,
                                             rows_cap=rows_cap) for _ in range(3)]
        for _ in range(2):
            g.replay()
            torch.cuda.synchronize()
            for res in outs:
                np.testing.assert_array_equal(host(res.token_ids), idx_ref)
                np.testing.assert_array_equal(host(res.status).astype(np.uint32), st_ref)
    finally:
        torch.cuda.synchronize()
        assert lib.onyx_ipc_free(own.value) == _lib.OK


def test_peer_exchange_wait_times_out_and_stays_failed(cuda_lib):
    """A peer whose flag never rises: rank 0 of a two-rank world whose second buffer is a
    zero-filled local allocation that no kernel ever raises. The exchange kernel's bounded
    wait (2 s) gives up and every row reports WAIT_TIMEOUT; the failure is sticky, so the
    next call reports it at once and stores no key into the other buffer. Nothing faults or
    hangs: one kernel waits, for a flag nothing sets, and gives up."""
    import ctypes
    import time

    from onyx_b200 import _lib
    lib = cuda_lib
    rows, rows_cap, world = 16, 16, 2
    nbytes = lib.onyx_exchange_buffer_bytes(world, rows_cap)
    handle = ctypes.create_string_buffer(lib.onyx_ipc_handle_bytes())
    own = ctypes.c_void_p()
    assert lib.onyx_ipc_alloc(nbytes, ctypes.byref(own), handle) == _lib.OK
    peer = torch.zeros(nbytes, dtype=torch.uint8, device="cuda:0")
    bases = (ctypes.c_void_p * world)(own.value, peer.data_ptr())
    w = workloads.scaling(seed=9, rows=rows, vocab=32000)
    lo, hi = vocab_parallel.vocab_shard_bounds(32000, 0, world)
    xt = to_device(np.ascontiguousarray(w["logits_bf16"][:, lo:hi]), "bf16")
    mt = masks_to_device(np.ascontiguousarray(w["masks"][:, lo // 32:hi // 32]))
    try:
        t0 = time.perf_counter()
        res = ms.vocab_exchange_argmax(xt, mt, lo, world=world, rank=0, exchange_bases=bases,
                                       rows_cap=rows_cap)
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 > 1.5  # the bounded wait ran out
        assert list(host(res.status)) == [ms.STATUS_WAIT_TIMEOUT] * rows
        assert list(host(res.token_ids)) == [-1] * rows
        peer.zero_()
        t0 = time.perf_counter()
        res2 = ms.vocab_exchange_argmax(xt, mt, lo, world=world, rank=0, exchange_bases=bases,
                                        rows_cap=rows_cap)
        torch.cuda.synchronize()
        assert time.perf_counter() - t0 < 1.0  # failed already: no second wait
        assert list(host(res2.status)) == [ms.STATUS_WAIT_TIMEOUT] * rows
        assert int(torch.count_nonzero(peer)) == 0  # neither keys nor flags were stored
    finally:
        torch.cuda.synchronize()
        assert lib.onyx_ipc_free(own.value) == _lib.OK


def test_peer_exchange_rejects_bad_arguments(cuda_lib):
    import ctypes
    from onyx_b200 import _lib
    lib = cuda_lib
    bases = (ctypes.c_void_p * 1)(None)
    x = torch.zeros((2, 64), dtype=torch.bfloat16, device="cuda:0")
    m = torch.zeros((2, 2), dtype=torch.int32, device="cuda:0")
    out = torch.empty(2, dtype=torch.int32, device="cuda:0")
    args = [x.data_ptr(), _lib.DTYPE_BF16, 2, 64, 64, m.data_ptr(), 2, 0]
    # a null buffer, rank outside the world, more rows than the buffers hold, world > 8
    for world, rank, cap in ((1, 0, 4), (1, 1, 4), (1, 0, 1), (9, 0, 4)):
        rc = lib.onyx_vocab_exchange_argmax(*args, world, rank, bases, cap, out.data_ptr(),
                                            out.data_ptr(), None, 0, None)
        assert rc == _lib.ERR_INVALID_ARGUMENT
    assert lib.onyx_exchange_buffer_bytes(9, 4) == 0


_PEER_WORKER = r"""
import os, sys, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, os.environ["ONYX_ROOT"])
from onyx_b200 import vocab_parallel, workloads
rank = int(os.environ["RANK"]); world = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
ex = vocab_parallel.PeerExchange(rows_cap=128)
outs = []
for seed in (11, 12, 13):  # three calls: both parities, then the first again
    w = workloads.scaling(seed=seed, rows=128, vocab=32000 * world)
    x, m = w["logits_bf16"], w["masks"]
    lo, hi = vocab_parallel.vocab_shard_bounds(x.shape[1], rank, world)
    xt = torch.from_numpy(np.ascontiguousarray(x[:, lo:hi]).view(np.int16)).cuda().view(torch.bfloat16)
    mt = torch.from_numpy(np.ascontiguousarray(m[:, lo // 32:(hi + 31) // 32]).view(np.int32)).cuda()
    res = vocab_parallel.vocab_parallel_masked_argmax(xt, mt, lo, exchange=ex)
    ref = vocab_parallel.vocab_parallel_masked_argmax(xt, mt, lo)  # NCCL all-gather
    assert torch.equal(res.token_ids, ref.token_ids) and torch.equal(res.status, ref.status)
    outs.append(torch.stack((res.token_ids, res.status)).cpu().numpy())
ex.close()
if rank == 0:
    np.save(os.environ["ONYX_OUT"], np.stack(outs))
dist.barrier()
dist.destroy_process_group()
"""


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_exchange_multi_rank(tmp_path, cuda_lib):
    """One rank per GPU of the box (2 to 8): keys over NVLink peer stores, three calls."""
    world = min(torch.cuda.device_count(), 8)
    script = tmp_path / "peer_worker.py"
    script.write_text(_PEER_WORKER)
    out = tmp_path / "peer_out.npy"
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, ONYX_ROOT=str(Path(__file__).resolve().parents[1]), ONYX_OUT=str(out),
               NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(port), str(script)]
    subprocess.run(["timeout", "-k", "30", "300", *cmd], check=True, env=env)
    got = np.load(out)
    for k, seed in enumerate((11, 12, 13)):
        w = workloads.scaling(seed=seed, rows=128, vocab=32000 * world)
        idx_ref, st_ref = oracle.masked_argmax(w["logits_bf16"], w["masks"], dtype="bf16")
        np.testing.assert_array_equal(got[k, 0], idx_ref)
        np.testing.assert_array_equal(got[k, 1].astype(np.uint32), st_ref)
