"""CPU oracle for the grammar-masked selection path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
(including ``bench.py --impl reference``) import this package, and only as the checker or
as the timed CPU reference. The CUDA product in ``onyx_b200`` never imports it.

Contents:

* ``oracle_cpu.c`` -- scalar C restatement of the reference's mask / first-max select /
  speculative verify / table gather / vocabulary-sharded select, plus the dense-DFA valid
  token scan (citations in that file). Built into ``oracle/_build/liboracle_cpu.so`` by
  ``oracle/build.py`` (OpenMP over rows).
* ``numpy_ref.py`` -- the same selection contract in NumPy
  (``np.where(bits, x, -inf)`` + first-occurrence ``argmax``), used to cross-check the C
  restatement on small cases.
* ``regex_dfa.py`` -- restated ``regex-automata`` dense-DFA semantics for the pattern
  subset the workloads use.

Parity pins: ``tests/golden/*.json`` were produced by the reference's own Python code
(``tests/golden/make_golden.py``); the oracle is checked against every one of them in
``tests/test_oracle_golden.py`` before any GPU result is compared with it.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "_build" / "liboracle_cpu.so"

DTYPE_CODES = {"f32": 0, "f16": 1, "bf16": 2, "f64": 3}
STATUS_BITS = {"ok": 0, "empty": 1, "all_neg_inf": 2, "nan": 4, "bad_state": 8}

_lib = None


class OraclePartial(ctypes.Structure):
    _fields_ = [
        ("found", ctypes.c_int32),
        ("nan", ctypes.c_int32),
        ("best", ctypes.c_double),
        ("idx", ctypes.c_int64),
    ]


def load() -> ctypes.CDLL:
    """Load the compiled C oracle, building it first if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        from .build import build

        build()
    lib = ctypes.CDLL(str(LIB_PATH))
    i64, i32, vp = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p
    lib.oracle_masked_argmax.argtypes = [vp, i32, i64, i64, i64, vp, i64, vp, vp, i32]
    lib.oracle_gather_masked_argmax.argtypes = [vp, i32, i64, i64, i64, vp, i64, i64, vp, vp, vp, i32]
    lib.oracle_spec_verify.argtypes = [
        vp, i32, i64, i64, i64, i64, i64, vp, i64, i64, vp, i64, i32, vp, vp, vp, i32,
    ]
    lib.oracle_mask_apply.argtypes = [vp, i32, i64, i64, i64, vp, i64, vp, i64, vp]
    lib.oracle_vocab_shard_select.argtypes = [vp, i32, i64, i64, i64, vp, i64, i64, vp]
    lib.oracle_vocab_combine.argtypes = [vp, i64, i64, vp, vp]
    lib.oracle_dfa_scan.argtypes = [vp, i32, i32, i32, vp, vp, i64, vp]
    lib.oracle_dfa_table.argtypes = [vp, i32, i32, vp, vp, i64, vp, i32]
    lib.oracle_max_threads.argtypes = []
    for name in (
        "oracle_masked_argmax",
        "oracle_gather_masked_argmax",
        "oracle_spec_verify",
        "oracle_mask_apply",
        "oracle_vocab_shard_select",
        "oracle_vocab_combine",
        "oracle_dfa_scan",
        "oracle_dfa_table",
        "oracle_max_threads",
    ):
        getattr(lib, name).restype = ctypes.c_int
    _lib = lib
    return lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def _dtype_code(arr: np.ndarray, dtype: str | None) -> int:
    if dtype is not None:
        return DTYPE_CODES[dtype]
    if arr.dtype == np.float32:
        return DTYPE_CODES["f32"]
    if arr.dtype == np.float64:
        return DTYPE_CODES["f64"]
    if arr.dtype == np.float16:
        return DTYPE_CODES["f16"]
    raise TypeError("pass dtype='bf16' for uint16 bf16 bit patterns")


def default_threads() -> int:
    return len(os.sched_getaffinity(0))


def masked_argmax(logits: np.ndarray, mask: np.ndarray | None, *, dtype: str | None = None,
                  threads: int = 0) -> tuple[np.ndarray, np.ndarray]:
    """First-max masked select per row. ``logits`` [B,V] (bf16 as uint16 bits)."""
    lib = load()
    logits = np.ascontiguousarray(logits)
    B, V = logits.shape
    idx = np.empty(B, np.int32)
    st = np.empty(B, np.uint32)
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.uint32)
    rc = lib.oracle_masked_argmax(
        _ptr(logits), _dtype_code(logits, dtype), B, V, V,
        _ptr(mask) if mask is not None else None, mask.shape[1] if mask is not None else 0,
        _ptr(idx), _ptr(st), threads,
    )
    if rc:
        raise ValueError("oracle_masked_argmax rejected its arguments")
    return idx, st


def gather_masked_argmax(logits, table, state_ids, *, dtype=None, threads=0):
    lib = load()
    logits = np.ascontiguousarray(logits)
    table = np.ascontiguousarray(table, dtype=np.uint32)
    state_ids = np.ascontiguousarray(state_ids, dtype=np.int32)
    B, V = logits.shape
    idx = np.empty(B, np.int32)
    st = np.empty(B, np.uint32)
    rc = lib.oracle_gather_masked_argmax(
        _ptr(logits), _dtype_code(logits, dtype), B, V, V, _ptr(table), table.shape[0],
        table.shape[1], _ptr(state_ids), _ptr(idx), _ptr(st), threads,
    )
    if rc:
        raise ValueError("oracle_gather_masked_argmax rejected its arguments")
    return idx, st


def spec_verify(logits, masks, drafts, *, bonus=True, dtype=None, threads=0):
    """``logits`` [B,G+1,V], ``masks`` [B,G+1,W], ``drafts`` [B,G]."""
    lib = load()
    logits = np.ascontiguousarray(logits)
    masks = np.ascontiguousarray(masks, dtype=np.uint32)
    drafts = np.ascontiguousarray(drafts, dtype=np.int32)
    B, G1, V = logits.shape
    G = G1 - 1
    acc = np.empty(B, np.int32)
    corr = np.empty(B, np.int32)
    st = np.empty(B, np.uint32)
    rc = lib.oracle_spec_verify(
        _ptr(logits), _dtype_code(logits, dtype), B, G, V, G1 * V, V, _ptr(masks),
        G1 * masks.shape[2], masks.shape[2], _ptr(drafts), drafts.shape[1] if drafts.ndim == 2 else 0,
        1 if bonus else 0, _ptr(acc), _ptr(corr), _ptr(st), threads,
    )
    if rc:
        raise ValueError("oracle_spec_verify rejected its arguments")
    return acc, corr, st


def mask_apply(logits, mask, *, dtype=None):
    lib = load()
    logits = np.ascontiguousarray(logits)
    mask = np.ascontiguousarray(mask, dtype=np.uint32)
    B, V = logits.shape
    out = np.empty_like(logits)
    st = np.empty(B, np.uint32)
    lib.oracle_mask_apply(
        _ptr(logits), _dtype_code(logits, dtype), B, V, V, _ptr(mask), mask.shape[1], _ptr(out),
        V, _ptr(st),
    )
    return out, st


def vocab_shard_select(logits_shard, mask_shard, col_offset, *, dtype=None):
    lib = load()
    logits_shard = np.ascontiguousarray(logits_shard)
    mask_shard = np.ascontiguousarray(mask_shard, dtype=np.uint32)
    B, Vs = logits_shard.shape
    out = (OraclePartial * B)()
    lib.oracle_vocab_shard_select(
        _ptr(logits_shard), _dtype_code(logits_shard, dtype), B, Vs, Vs, _ptr(mask_shard),
        mask_shard.shape[1], col_offset, ctypes.addressof(out),
    )
    return out


def vocab_combine(partials_by_shard) -> tuple[np.ndarray, np.ndarray]:
    lib = load()
    n = len(partials_by_shard)
    B = len(partials_by_shard[0])
    flat = (OraclePartial * (n * B))()
    for s, part in enumerate(partials_by_shard):
        for r in range(B):
            flat[s * B + r] = part[r]
    idx = np.empty(B, np.int32)
    st = np.empty(B, np.uint32)
    lib.oracle_vocab_combine(ctypes.addressof(flat), n, B, _ptr(idx), _ptr(st))
    return idx, st


def pack_vocabulary(vocabulary) -> tuple[np.ndarray, np.ndarray]:
    """CSR layout (bytes uint8[], offsets int64[V+1]) of a byte-string vocabulary."""
    offsets = np.zeros(len(vocabulary) + 1, np.int64)
    offsets[1:] = np.cumsum([len(t) for t in vocabulary])
    data = np.frombuffer(b"".join(vocabulary), dtype=np.uint8).copy()
    if data.size == 0:
        data = np.zeros(1, np.uint8)
    return data, offsets


def dfa_scan_bitmask(dfa, state: int, vocabulary, *, packed=None) -> np.ndarray:
    """Packed valid-token bitmask of ``state`` (restating get_valid_token_ids). ``packed``:
    ``pack_vocabulary(vocabulary)`` done once by the caller, for repeated scans."""
    lib = load()
    data, offsets = packed if packed is not None else pack_vocabulary(vocabulary)
    trans = np.ascontiguousarray(dfa.trans, dtype=np.int32)
    V = len(vocabulary)
    out = np.zeros((V + 31) // 32, np.uint32)
    rc = lib.oracle_dfa_scan(_ptr(trans), trans.shape[0], dfa.dead, state, _ptr(data),
                             _ptr(offsets), V, _ptr(out))
    if rc:
        raise ValueError("oracle_dfa_scan rejected its arguments")
    return out


def dfa_table(dfa, vocabulary, *, threads: int = 0) -> np.ndarray:
    lib = load()
    data, offsets = pack_vocabulary(vocabulary)
    trans = np.ascontiguousarray(dfa.trans, dtype=np.int32)
    V = len(vocabulary)
    out = np.zeros((trans.shape[0], (V + 31) // 32), np.uint32)
    lib.oracle_dfa_table(_ptr(trans), trans.shape[0], dfa.dead, _ptr(data), _ptr(offsets), V,
                         _ptr(out), threads)
    return out


def status_name(bits: int) -> str:
    for name, value in STATUS_BITS.items():
        if value == bits:
            return name
    return f"bits:{bits}"
