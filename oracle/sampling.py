"""Masked temperature / top-p sampling -- TEST INFRASTRUCTURE ONLY (the oracle).

Only tests and the CPU-baseline leg of the benchmark use this module, as the checker.

Restates the reference's sampling distribution, onyx_cuda/src/onyx_cuda/selection.py
(``_filtered_reference_weights``, used by ``create_reference_sampler``):

* NaN among the values -> rejected;
* any +inf -> every +inf id with equal weight 1/k;
* otherwise weight exp((v - max) / T) for every finite value (max over the finite ones),
  -inf -> weight 0; probabilities weight / total; zero-weight ids drop out;
* rank by (-probability, id); keep the shortest prefix whose cumulative probability
  reaches top_p (the token that crosses is kept).

The grammar mask comes first: invalid ids are -inf (torch_grammar_mask.py:145-186), an
empty valid set or an all -inf support is rejected.

The uniform draw comes from Philox4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel Random
Numbers: As Easy as 1, 2, 3", SC 2011) with key = seed (64 bits) and counter = (call counter,
row), turned into a double in [0, 1) from 53 bits (a * 2^26 + b) / 2^53 with a = x0 >> 5,
b = x1 >> 6. The sampled id is the first kept id, walking kept ids in increasing id order,
whose cumulative kept probability exceeds u times the kept total. (The reference's CPU
sampler walks in ranked order with Python's Mersenne Twister; its CUDA sampler uses torch's
generator. Neither stream is reproducible elsewhere, so the build fixes its own: the
distribution and the top-p set are the reference's.)

Arithmetic is float64 and sequential in the orders stated above; the normalising total is
Python's sum() (compensated from Python 3.12), as in the reference.
"""

from __future__ import annotations

import math

import numpy as np

STATUS_OK = 0
STATUS_EMPTY_MASK = 1
STATUS_ALL_NEG_INF = 2
STATUS_NAN_IN_SUPPORT = 4

_M0, _M1 = 0xD2511F53, 0xCD9E8D57
_W0, _W1 = 0x9E3779B9, 0xBB67AE85
_MASK32 = 0xFFFFFFFF


def philox4x32_10(counter: tuple[int, int, int, int], key: tuple[int, int]) -> tuple[int, ...]:
    """Philox4x32 with 10 rounds (the published algorithm)."""
    c0, c1, c2, c3 = (int(c) & _MASK32 for c in counter)
    k0, k1 = (int(k) & _MASK32 for k in key)
    for r in range(10):
        if r:
            k0 = (k0 + _W0) & _MASK32
            k1 = (k1 + _W1) & _MASK32
        p0 = _M0 * c0
        p1 = _M1 * c2
        hi0, lo0 = p0 >> 32, p0 & _MASK32
        hi1, lo1 = p1 >> 32, p1 & _MASK32
        c0, c1, c2, c3 = hi1 ^ c1 ^ k0, lo1, hi0 ^ c3 ^ k1, lo0
    return c0, c1, c2, c3


def uniform(seed: int, call: int, row: int) -> float:
    """The draw of `row` in call `call` of a session seeded with `seed`, in [0, 1)."""
    x = philox4x32_10((call & _MASK32, (call >> 32) & _MASK32, row & _MASK32, 0),
                      (seed & _MASK32, (seed >> 32) & _MASK32))
    a, b = x[0] >> 5, x[1] >> 6
    return (a * 67108864.0 + b) / 9007199254740992.0


def kept_weights(values: np.ndarray, valid: np.ndarray, temperature: float,
                 top_p: float) -> tuple[int, list[tuple[int, float]]]:
    """(status, [(id, probability)] of the kept ids in ranked order) of one masked row."""
    vals = [float(v) for v in np.asarray(values, dtype=np.float64)]
    ids = [i for i in range(len(vals)) if valid[i]]
    if not ids:
        return STATUS_EMPTY_MASK, []
    if any(math.isnan(vals[i]) for i in ids):
        return STATUS_NAN_IN_SUPPORT, []
    pos_inf = [i for i in ids if vals[i] == math.inf]
    if pos_inf:
        w = 1.0 / len(pos_inf)
        probs = [(i, w) for i in pos_inf]
    else:
        finite = [vals[i] for i in ids if vals[i] != -math.inf]
        if not finite:
            return STATUS_ALL_NEG_INF, []
        m = max(finite)
        weights = [0.0] * len(vals)
        for i in ids:
            if vals[i] != -math.inf:
                weights[i] = math.exp((vals[i] - m) / float(temperature))
        # every weight in index order, with Python's own sum(): from Python 3.12 it adds
        # floats with Neumaier's compensated summation, which the reference's sum(...) gets
        total = sum(weights)
        probs = [(i, weights[i] / total) for i in range(len(vals)) if weights[i] > 0.0]
    ranked = sorted(probs, key=lambda item: (-item[1], item[0]))
    kept = []
    cumulative = 0.0
    for tid, p in ranked:
        kept.append((tid, p))
        cumulative += p
        if cumulative >= float(top_p):
            break
    return STATUS_OK, kept


def sample_row(values, valid, temperature: float, top_p: float, u: float) -> tuple[int, int]:
    """(token id or -1, status) for one masked row and uniform draw u."""
    status, kept = kept_weights(values, valid, temperature, top_p)
    if status:
        return -1, status
    kept_by_id = sorted(kept)
    total = 0.0
    for _, p in kept_by_id:
        total += p
    threshold = u * total
    cumulative = 0.0
    for tid, p in kept_by_id:
        cumulative += p
        if threshold < cumulative:
            return tid, STATUS_OK
    return kept_by_id[-1][0], STATUS_OK


def unpack_mask(words: np.ndarray, vocab: int) -> np.ndarray:
    bits = np.unpackbits(np.ascontiguousarray(words, dtype="<u4").view(np.uint8),
                         bitorder="little")
    return bits[:vocab].astype(bool)


def masked_sample(values: np.ndarray, masks: np.ndarray | None, temperature: float,
                  top_p: float, seed: int, call: int) -> tuple[np.ndarray, np.ndarray]:
    """Batched: row r draws uniform(seed, call, r). values [B, V] float; masks [B, W]."""
    values = np.asarray(values)
    B, V = values.shape
    idx = np.empty(B, np.int32)
    st = np.empty(B, np.uint32)
    for r in range(B):
        valid = np.ones(V, bool) if masks is None else unpack_mask(masks[r], V)
        idx[r], st[r] = sample_row(values[r], valid, temperature, top_p, uniform(seed, call, r))
    return idx, st
