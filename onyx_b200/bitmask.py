"""Host-side packing of valid-token sets into the library's uint32 bitmask layout.

The reference hands the mask boundary a sorted tuple of valid ids
(onyx_cuda/src/onyx_cuda/torch_grammar_mask.py:69-86); the B200 kernels read the same set
as packed words: token ``t`` valid iff bit ``t & 31`` of word ``t >> 5`` is set.
"""

from __future__ import annotations

from collections.abc import Iterable

import numpy as np

__all__ = ["words_for", "pack_ids", "pack_bool", "unpack"]


def words_for(vocab_size: int) -> int:
    return (int(vocab_size) + 31) // 32


def pack_ids(ids: Iterable[int], vocab_size: int, out: np.ndarray | None = None) -> np.ndarray:
    """Pack valid ids (any order, in range) into ``uint32[words_for(vocab_size)]``."""
    w = words_for(vocab_size)
    if out is None:
        out = np.zeros(w, dtype=np.uint32)
    else:
        out[:w] = 0
    arr = np.fromiter(ids, dtype=np.int64) if not isinstance(ids, np.ndarray) else ids.astype(np.int64)
    if arr.size:
        if arr.min() < 0 or arr.max() >= vocab_size:
            raise ValueError(f"token ids must lie in [0, {vocab_size})")
        np.bitwise_or.at(out, arr >> 5, (np.uint32(1) << (arr & 31).astype(np.uint32)))
    return out


def pack_bool(valid: np.ndarray) -> np.ndarray:
    """Pack a boolean matrix ``[..., V]`` into ``uint32[..., ceil(V/32)]`` (tail bits zero)."""
    valid = np.asarray(valid, dtype=bool)
    v = valid.shape[-1]
    w = words_for(v)
    padded = np.zeros(valid.shape[:-1] + (w * 32,), dtype=bool)
    padded[..., :v] = valid
    return np.packbits(padded, axis=-1, bitorder="little").view("<u4").astype(np.uint32)


def unpack(words: np.ndarray, vocab_size: int) -> np.ndarray:
    """Inverse of :func:`pack_bool`: boolean ``[..., vocab_size]``."""
    w = np.ascontiguousarray(words, dtype="<u4")
    bits = np.unpackbits(w.view(np.uint8), axis=-1, bitorder="little")
    return bits[..., :vocab_size].astype(bool)
