"""NumPy restatement of masked greedy selection -- TEST INFRASTRUCTURE ONLY.

The masked row is ``np.where(bit, x, -inf)`` (onyx_cuda/src/onyx_cuda/
torch_grammar_mask.py:155-171: allowed values kept, everything else -inf) and the
selection is NumPy's first-occurrence ``argmax`` after NaN rejection
(onyx_cuda/src/onyx_cuda/torch_backend.py:991-998; generation.py:219-224). bf16 rows are
passed as their uint16 bit patterns and widened exactly with ``u16 << 16``.
Used to cross-check ``oracle_cpu.c`` on small inputs.
"""

from __future__ import annotations

import numpy as np


def to_float(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return (x.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return x.astype(np.float64)


def unpack_mask(mask_words: np.ndarray, vocab_size: int) -> np.ndarray:
    bits = np.unpackbits(
        np.ascontiguousarray(mask_words, dtype="<u4").view(np.uint8), axis=-1, bitorder="little"
    )
    return bits[..., :vocab_size].astype(bool)


def masked_argmax(logits: np.ndarray, mask_words: np.ndarray, dtype: str):
    """Returns (index int32[B], status uint32[B]) with the oracle's status bits."""
    x = to_float(np.atleast_2d(logits), dtype)
    B, V = x.shape
    bits = unpack_mask(np.atleast_2d(mask_words), V)
    masked = np.where(bits, x, -np.inf)
    idx = np.full(B, -1, np.int32)
    st = np.zeros(B, np.uint32)
    for r in range(B):
        if not bits[r].any():
            st[r] = 1
            continue
        if np.isnan(masked[r]).any():
            st[r] = 4
            continue
        if np.all(masked[r][bits[r]] == -np.inf):
            # rejected by the mask boundary; the index reported is the first support id
            st[r] = 2
            idx[r] = int(np.flatnonzero(bits[r])[0])
            continue
        # -0.0 == +0.0 under float comparison, so argmax keeps the first of them
        idx[r] = int(np.argmax(masked[r]))
    return idx, st
