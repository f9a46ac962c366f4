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

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from . import masked_selection as _ms

__all__ = [
    "batch_shard_bounds",
    "vocab_shard_bounds",
    "PeerExchange",
    "vocab_parallel_masked_argmax",
    "combine_keys_host",
]

MAX_EXCHANGE_RANKS = 8


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


class PeerExchange:
    """Exchange buffers of one process group for vocabulary-sharded selection over NVLink
    peer memory: each rank's buffer is mapped into every other rank (CUDA IPC), the shard
    kernel writes its row keys straight into all of them, and a small kernel swaps flags
    and combines -- one fused step instead of an all-gather plus a combine.

    Collective: every rank of ``group`` constructs it with the same ``rows_cap`` (the most
    rows one call may select), makes the same calls in the same order, and closes it. The
    call count lives on the device, so calls may be captured in a CUDA graph.
    """

    def __init__(self, rows_cap: int, group: dist.ProcessGroup | None = None,
                 device: torch.device | int | None = None) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if not 1 <= self.world <= MAX_EXCHANGE_RANKS:
            raise ValueError(f"peer exchange supports 1..{MAX_EXCHANGE_RANKS} ranks")
        if rows_cap < 1:
            raise ValueError("rows_cap must be positive")
        self.rows_cap = int(rows_cap)
        if device is None:
            device = torch.cuda.current_device()
        self.device = device if isinstance(device, torch.device) else torch.device("cuda", device)
        self._lib = lib = _lib.load()
        nbytes = lib.onyx_exchange_buffer_bytes(self.world, self.rows_cap)
        handle = ctypes.create_string_buffer(lib.onyx_ipc_handle_bytes())
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check("onyx_ipc_alloc", lib.onyx_ipc_alloc(nbytes, ctypes.byref(own), handle))
        handles: list[bytes | None] = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self._opened: list[int] = []
        bases = []
        with torch.cuda.device(self.device):
            for i, h in enumerate(handles):
                if i == self.rank:
                    bases.append(own.value)
                    continue
                ptr = ctypes.c_void_p()
                _lib.check("onyx_ipc_open", lib.onyx_ipc_open(h, ctypes.byref(ptr)))
                self._opened.append(ptr.value)
                bases.append(ptr.value)
        self._own = own.value
        self.bases = (ctypes.c_void_p * self.world)(*bases)
        dist.barrier(group)  # every mapping exists before any rank stores into it

    def select(self, logits_shard: torch.Tensor, mask_shard: torch.Tensor,
               col_offset: int) -> _ms.MaskedArgmaxResult:
        """This call's full-vocabulary selections (same call on every rank)."""
        if self._own is None:
            raise RuntimeError("the peer exchange is closed")
        if logits_shard.shape[-1] == 0:
            raise ValueError("every rank of a peer exchange must hold at least one column")
        return _ms.vocab_exchange_argmax(
            logits_shard, mask_shard, col_offset, world=self.world, rank=self.rank,
            exchange_bases=self.bases, rows_cap=self.rows_cap)

    def close(self) -> None:
        """Collective: unmaps the peers' buffers and frees this rank's."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)  # no rank still stores into another's buffer
        with torch.cuda.device(self.device):
            for ptr in self._opened:
                _lib.check("onyx_ipc_close", self._lib.onyx_ipc_close(ptr))
            dist.barrier(self.group)
            _lib.check("onyx_ipc_free", self._lib.onyx_ipc_free(self._own))
        self._own = None
        self._opened = []


def vocab_parallel_masked_argmax(
    logits_shard: torch.Tensor,
    mask_shard: torch.Tensor,
    col_offset: int,
    group: dist.ProcessGroup | None = None,
    exchange: PeerExchange | None = None,
) -> _ms.MaskedArgmaxResult:
    """Masked greedy selection over a vocabulary split across the ranks of ``group``.

    Every rank passes its own shard and receives the full-vocabulary selections. With a
    :class:`PeerExchange` the keys travel through NVLink peer memory inside the selection
    step; without one they travel by ``all_gather_into_tensor`` (any backend).
    """
    if exchange is not None:
        return exchange.select(logits_shard, mask_shard, col_offset)
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
