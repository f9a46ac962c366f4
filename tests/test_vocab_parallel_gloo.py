"""World-size-2 CPU (gloo) test of the vocabulary-sharded exchange and combine.

Each rank reduces its column shard to 64-bit keys (oracle restatement, CPU), the keys are
all-gathered through a real gloo process group exactly as the GPU path all-gathers them
through NCCL, and every rank combines them; all ranks must agree with the unsharded oracle.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, result_q) -> None:
    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import oracle
    from onyx_b200 import vocab_parallel, workloads
    from tests.test_host_logic import _oracle_keys

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(11)
        rows, vocab = 16, 2048
        x = workloads.normal_bf16(rng, (rows, vocab))
        masks = workloads.bernoulli_masks(rng, np.full(rows, 0.05), vocab)
        lo, hi = vocab_parallel.vocab_shard_bounds(vocab, rank, world)
        mine = torch.tensor(
            [k - (1 << 64) if k >= 1 << 63 else k for k in _oracle_keys(x, masks, lo, hi)],
            dtype=torch.int64,
        )
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
        got = vocab_parallel.combine_keys_host([[int(v) & ((1 << 64) - 1) for v in g] for g in gathered])
        idx, st = oracle.masked_argmax(x, masks, dtype="bf16")
        ok = all(
            got[r][1] == int(st[r]) and (int(st[r]) not in (0, 2) or got[r][0] == int(idx[r]))
            for r in range(rows)
        )
        result_q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_exchange_matches_unsharded():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}
