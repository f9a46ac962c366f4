"""Seeded synthetic inputs with the shapes and value distributions of the five workloads.

No public dataset is involved; the shapes stand in for Llama-3 (V=128,256), Qwen2.5
(V=151,936 model rows) and a 256,000-token vocabulary. Logits are N(0, 3); token masks are
per-row Bernoulli bitmasks (token id t -> bit t&31 of word t>>5), at least one bit set,
tail bits zero. bf16 values are produced by round-to-nearest-even from float32 and carried
as ``uint16`` bit patterns so that the CPU oracle and the GPU see identical bits.

1. ``single_row``   fp32 [1, 32000]; 256 single bytes + 31,744 printable-ASCII strings of
                    2-8 bytes (seeded); the mask comes from the grammar ``[0-9]{1,8}`` at its
                    initial state (computed by the caller).
2. ``batched``      bf16 [64, 128256]; density ~ U[0.5%, 20%] per row.
3. ``spec_verify``  bf16 [32, 5, 151936]; masks [32, 5, 4748] at U[1%, 10%]; drafts int32
                    [32, 4]: 70% the position's masked argmax, else another valid id.
4. ``table_gather`` table uint32 [4096, 4008] at U[0.1%, 30%] per state; state ids int32
                    [256] ~ U{0..4095}; logits bf16 [256, 128256].
5. ``scaling``      bf16 [1024, 256000], density 5%.
"""

from __future__ import annotations

from collections.abc import Callable

import numpy as np

from .bitmask import words_for

__all__ = [
    "SEEDS",
    "bf16_bits",
    "bf16_bits_to_f32",
    "normal_bf16",
    "bernoulli_masks",
    "synthetic_vocabulary",
    "single_row",
    "batched",
    "spec_verify",
    "table_gather",
    "scaling",
]

SEEDS = {1: 1001, 2: 1002, 3: 1003, 4: 1004, 5: 1005}


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (NaN -> quiet NaN)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    bits = (rounded >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        bits[nan] = 0x7FC0
    return bits


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << np.uint32(16)).view(np.float32)


def normal_bf16(rng: np.random.Generator, shape, scale: float = 3.0, chunk_rows: int = 64) -> np.ndarray:
    """N(0, scale) as bf16 bits, generated in row chunks to bound host memory."""
    shape = tuple(shape)
    out = np.empty(shape, dtype=np.uint16)
    flat = out.reshape(-1, shape[-1])
    for lo in range(0, flat.shape[0], chunk_rows):
        hi = min(lo + chunk_rows, flat.shape[0])
        flat[lo:hi] = bf16_bits(rng.standard_normal((hi - lo, shape[-1]), dtype=np.float32) * scale)
    return out


def bernoulli_masks(rng: np.random.Generator, densities: np.ndarray, vocab: int,
                    chunk_rows: int = 64) -> np.ndarray:
    """One packed mask row per density; each row gets at least one valid id."""
    densities = np.asarray(densities, dtype=np.float32).reshape(-1)
    rows = densities.shape[0]
    w = words_for(vocab)
    out = np.zeros((rows, w), dtype=np.uint32)
    for lo in range(0, rows, chunk_rows):
        hi = min(lo + chunk_rows, rows)
        valid = rng.random((hi - lo, vocab), dtype=np.float32) < densities[lo:hi, None]
        empty = ~valid.any(axis=1)
        if empty.any():
            for r in np.flatnonzero(empty):
                valid[r, rng.integers(0, vocab)] = True
        padded = np.zeros((hi - lo, w * 32), dtype=bool)
        padded[:, :vocab] = valid
        out[lo:hi] = np.packbits(padded, axis=1, bitorder="little").view("<u4")
    return out


def synthetic_vocabulary(rng: np.random.Generator, size: int = 32000) -> list[bytes]:
    """256 single-byte tokens followed by random printable-ASCII strings of 2-8 bytes."""
    vocab = [bytes([b]) for b in range(256)]
    n = size - 256
    lengths = rng.integers(2, 9, size=n)
    chars = rng.integers(0x20, 0x7F, size=int(lengths.sum()), dtype=np.uint8).tobytes()
    pos = 0
    for ln in lengths:
        vocab.append(chars[pos : pos + ln])
        pos += int(ln)
    return vocab


def synthetic_dfa(rng: np.random.Generator, states: int = 64, live: float = 0.2) -> dict:
    """Dense byte DFA with an absorbing dead state 0 and start state 1: every other
    (state, byte) transition goes to a uniformly drawn live state with probability `live`,
    else to dead (a grammar that admits a few bytes per state, like a JSON or number
    pattern)."""
    trans = rng.integers(1, states, size=(states, 256), dtype=np.int32)
    trans[rng.random((states, 256)) >= live] = 0
    trans[0, :] = 0
    return {"trans": trans, "dead": 0, "start": 1}


def digits_dfa(max_len: int = 8) -> dict:
    """Dense byte DFA of the anchored pattern ``[0-9]{1,max_len}`` as the reference's
    leftmost-first dense DFA behaves (matches reported one byte late), built directly:

    * 0 dead; 1 start; 1 + j after j digits (j = 1..max_len); ``m`` = max_len + 2, the
      delayed-match state a match that has ended moves to on any byte;
    * start: digit -> 2, anything else -> dead;
    * after j < max_len digits: digit -> j + 1 digits, anything else -> m;
    * after max_len digits: any byte -> m;  m: any byte -> dead.

    So a token is valid from the start state iff it is d^j (1 <= j <= max_len) or d^j followed
    by one more byte of any kind."""
    n = max_len + 3
    m = max_len + 2
    trans = np.zeros((n, 256), np.int32)
    digits = np.arange(ord("0"), ord("9") + 1)
    trans[1, digits] = 2
    for j in range(1, max_len + 1):
        s = 1 + j
        trans[s, :] = m
        if j < max_len:
            trans[s, digits] = s + 1
    trans[m, :] = 0
    return {"trans": trans, "dead": 0, "start": 1}


def single_row(seed: int = SEEDS[1]) -> dict:
    rng = np.random.default_rng(seed)
    vocabulary = synthetic_vocabulary(rng, 32000)
    logits = (rng.standard_normal((1, 32000), dtype=np.float32) * 3.0).astype(np.float32)
    return {"vocabulary": vocabulary, "pattern": "[0-9]{1,8}", "logits": logits}


def batched(seed: int = SEEDS[2], rows: int = 64, vocab: int = 128256) -> dict:
    rng = np.random.default_rng(seed)
    logits = normal_bf16(rng, (rows, vocab))
    dens = rng.uniform(0.005, 0.20, size=rows)
    masks = bernoulli_masks(rng, dens, vocab)
    return {"logits_bf16": logits, "masks": masks, "densities": dens}


def spec_verify(argmax_fn: Callable[[np.ndarray, np.ndarray], np.ndarray], seed: int = SEEDS[3],
                batch: int = 32, gamma: int = 4, vocab: int = 151936) -> dict:
    """``argmax_fn(logits_bf16 [R, V], masks [R, W]) -> int32 [R]`` supplies the masked
    argmax the drafts are drawn from (70% of the time)."""
    rng = np.random.default_rng(seed)
    g1 = gamma + 1
    logits = normal_bf16(rng, (batch, g1, vocab))
    dens = rng.uniform(0.01, 0.10, size=batch * g1)
    masks = bernoulli_masks(rng, dens, vocab).reshape(batch, g1, -1)
    best = argmax_fn(logits.reshape(batch * g1, vocab), masks.reshape(batch * g1, -1))
    best = np.asarray(best, dtype=np.int64).reshape(batch, g1)
    drafts = np.empty((batch, gamma), dtype=np.int32)
    for b in range(batch):
        for i in range(gamma):
            if rng.random() < 0.7:
                drafts[b, i] = best[b, i]
                continue
            words = masks[b, i]
            bits = np.unpackbits(words.view(np.uint8), bitorder="little")[:vocab]
            ids = np.flatnonzero(bits)
            ids = ids[ids != best[b, i]]
            drafts[b, i] = int(rng.choice(ids)) if ids.size else (int(best[b, i]) + 1) % vocab
    return {"logits_bf16": logits, "masks": masks, "drafts": drafts, "gamma": gamma}


def table_gather(seed: int = SEEDS[4], states: int = 4096, rows: int = 256,
                 vocab: int = 128256) -> dict:
    rng = np.random.default_rng(seed)
    dens = rng.uniform(0.001, 0.30, size=states)
    table = bernoulli_masks(rng, dens, vocab)
    state_ids = rng.integers(0, states, size=rows).astype(np.int32)
    logits = normal_bf16(rng, (rows, vocab))
    return {"table": table, "state_ids": state_ids, "logits_bf16": logits}


def scaling(seed: int = SEEDS[5], rows: int = 1024, vocab: int = 256000,
            density: float = 0.05) -> dict:
    rng = np.random.default_rng(seed)
    logits = normal_bf16(rng, (rows, vocab))
    masks = bernoulli_masks(rng, np.full(rows, density), vocab)
    return {"logits_bf16": logits, "masks": masks}
