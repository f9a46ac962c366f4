"""Multi-GPU masked selection: batch sharding and vocabulary sharding.

The reference is single-device (everything runs on ``cuda:0``,
onyx_cuda/src/onyx_cuda/torch_backend.py:105-107); these two layouts spread the same
selection over one process per GPU:

* **batch-sharded**: rows are independent, so each rank selects its own slice of rows
  with :func:`onyx_b200.masked_selection.masked_argmax`; there is no communication
  (:func:`batch_shard_bounds` gives each rank's slice).
* **vocabulary-sharded**: each rank holds columns ``[col_offset, col_offset + V/n)`` of
  every row. It reduces them to one packed 8-byte key per row (order code of the masked
  maximum, complemented global id); an all-gather of ``rows x 8`` bytes per rank
  (NCCL over NVLink on GPUs, gloo on CPU for the host-logic tests) and one combine kernel
  give every rank the same selections as the unsharded kernel, bit for bit, because the
  key order (value, then lowest id, with NaN above all and signed zeros folded) is total.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import masked_selection as _ms

__all__ = [
    "batch_shard_bounds",
    "vocab_shard_bounds",
    "vocab_parallel_masked_argmax",
    "combine_keys_host",
]


def batch_shard_bounds(rows: int, rank: int, world_size: int) -> tuple[int, int]:
    """Contiguous row slice ``[lo, hi)`` of ``rank`` (first ranks take the remainder)."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("rank must lie in [0, world_size)")
    base, extra = divmod(rows, world_size)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def vocab_shard_bounds(vocab: int, rank: int, world_size: int) -> tuple[int, int]:
    """Column slice ``[lo, hi)`` of ``rank``; every boundary is a multiple of 32 so each
    shard's mask words are whole words of the unsharded mask."""
    if world_size <= 0 or not 0 <= rank < world_size:
        raise ValueError("rank must lie in [0, world_size)")
    words = (vocab + 31) // 32
    wlo, whi = batch_shard_bounds(words, rank, world_size)
    return min(wlo * 32, vocab), min(whi * 32, vocab)


def vocab_parallel_masked_argmax(
    logits_shard: torch.Tensor,
    mask_shard: torch.Tensor,
    col_offset: int,
    group: dist.ProcessGroup | None = None,
) -> _ms.MaskedArgmaxResult:
    """Masked greedy selection over a vocabulary split across the ranks of ``group``.

    Every rank passes its own shard and receives the full-vocabulary selections.
    """
    world = dist.get_world_size(group)
    if logits_shard.shape[-1] == 0:
        # a rank past the end of a small vocabulary holds no columns: key 0 = no token
        keys = torch.zeros(logits_shard.shape[0], dtype=torch.int64, device=logits_shard.device)
    else:
        keys = _ms.vocab_partial_keys(logits_shard, mask_shard, col_offset)
    gathered = torch.empty((world, keys.shape[0]), dtype=keys.dtype, device=keys.device)
    dist.all_gather_into_tensor(gathered, keys, group=group)
    return _ms.combine_partial_keys(gathered)


_MASK64 = (1 << 64) - 1


def combine_keys_host(keys_by_shard: list[list[int]]) -> list[tuple[int, int]]:
    """Host restatement of the combine step on unsigned 64-bit keys: (id, status) per row.

    Used where the keys travel through a CPU process group; the GPU path uses the combine
    kernel. Keys are compared as unsigned integers; 0 means "no valid token in the shard".
    """
    rows = len(keys_by_shard[0])
    out = []
    for r in range(rows):
        best = max(int(k[r]) & _MASK64 for k in keys_by_shard)
        if best == 0:
            out.append((-1, _ms.STATUS_EMPTY_MASK))
            continue
        if best == _MASK64:  # a shard whose in-kernel wait gave up
            out.append((-1, _ms.STATUS_WAIT_TIMEOUT))
            continue
        order = best >> 32
        if order == 0xFFFFFFFF:
            out.append((-1, _ms.STATUS_NAN_IN_SUPPORT))
            continue
        idx = 0xFFFFFFFF - (best & 0xFFFFFFFF)
        out.append((idx, _ms.STATUS_ALL_NEG_INF if order == 0x007FFFFF else 0))
    return out
